"""The CPU oracle is pinned against golden vectors produced by running the
reference package itself (tests/golden/make_golden.py)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as orc

TOL = dict(rtol=1e-10, atol=1e-10)


@pytest.mark.parametrize("k", [1, 3, 5])
def test_stride1_matches_reference(golden, k):
    g = golden("depthwise.npz")
    t = f"s1_k{k}/"
    np.testing.assert_allclose(orc.dw_fwd(g[t + "x"], g[t + "w"], g[t + "b"], k), g[t + "y"], **TOL)
    np.testing.assert_allclose(orc.dw_dgrad(g[t + "dy"], g[t + "w"], k), g[t + "dx"], **TOL)
    dw, db = orc.dw_wgrad(g[t + "x"], g[t + "dy"], k)
    np.testing.assert_allclose(dw, g[t + "dw"], **TOL)
    np.testing.assert_allclose(db, g[t + "db"], **TOL)


@pytest.mark.parametrize("k", [3, 5])
def test_stride2_matches_reference(golden, k):
    g = golden("depthwise.npz")
    t = f"s2_k{k}/"
    x = g[t + "x"]
    np.testing.assert_allclose(orc.s2_fwd(x, g[t + "w"], g[t + "b"], k), g[t + "y"], **TOL)
    np.testing.assert_allclose(orc.s2_dgrad(g[t + "dy"], g[t + "w"], x.shape[2:], k), g[t + "dx"], **TOL)
    dw, db = orc.s2_wgrad(x, g[t + "dy"], k)
    np.testing.assert_allclose(dw, g[t + "dw"], **TOL)
    np.testing.assert_allclose(db, g[t + "db"], **TOL)


@pytest.mark.parametrize("k", [3, 5])
def test_transpose_matches_reference(golden, k):
    g = golden("depthwise.npz")
    t = f"t_k{k}/"
    np.testing.assert_allclose(orc.t_fwd(g[t + "x"], g[t + "w"], g[t + "b"], k), g[t + "y"], **TOL)
    np.testing.assert_allclose(orc.t_dgrad(g[t + "dy"], g[t + "w"], k), g[t + "dx"], **TOL)
    dw, db = orc.t_wgrad(g[t + "x"], g[t + "dy"], k)
    np.testing.assert_allclose(dw, g[t + "dw"], **TOL)
    np.testing.assert_allclose(db, g[t + "db"], **TOL)


@pytest.mark.parametrize("tag,kind", [("regular_k3", "regular"), ("regular_k5", "regular"), ("down_k3", "down"),
                                      ("up_k3", "up")])
def test_block_matches_reference(golden, tag, kind):
    g = golden("blocks.npz")
    state = {k[len(tag) + 7:]: g[k] for k in g.files if k.startswith(f"{tag}/param/")}
    p = orc.BlockParams.from_state(state)
    x, dy = g[f"{tag}/x"], g[f"{tag}/dy"]
    addend = None
    if kind == "down":
        # residual branch: 1x1 stride-2 conv of x
        rw, rb = state["residual.weight"], state["residual.bias"]
        addend = orc.pointwise_fwd(x[:, :, ::2, ::2, ::2], rw, rb)
    elif kind == "up":
        rw, rb = state["residual.weight"], state["residual.bias"]
        n, c, d, h, w = x.shape
        # 1x1 transposed stride-2 conv: scatter x into even positions of a (2S-1) grid
        up = np.zeros((n, c, 2 * d - 1, 2 * h - 1, 2 * w - 1))
        up[:, :, ::2, ::2, ::2] = x
        addend = orc.pointwise_fwd(up, np.transpose(rw, (1, 0, 2, 3, 4)), None)
        addend += rb.reshape(1, -1, 1, 1, 1)
    y, grads = orc.block_reference(x, dy if kind != "up" else dy[:, :, 1:, 1:, 1:], p, kind, addend=addend,
                                   residual_is_input=(kind == "regular"), round_bf16_steps=False)
    want_y = g[f"{tag}/y"]
    if kind == "up":
        want_y = want_y[:, :, 1:, 1:, 1:]
        assert np.all(g[f"{tag}/y"][:, :, 0] == 0) and np.all(g[f"{tag}/y"][:, :, :, 0] == 0)
    np.testing.assert_allclose(y, want_y, rtol=1e-9, atol=1e-9)
    for name in ("depthwise.weight", "depthwise.bias", "norm.weight", "norm.bias", "expand.weight", "expand.bias",
                 "project.weight", "project.bias"):
        np.testing.assert_allclose(grads[name], g[f"{tag}/grad/{name}"], rtol=1e-8, atol=1e-8, err_msg=name)
    if kind == "regular":
        np.testing.assert_allclose(grads["dx"], g[f"{tag}/dx"], rtol=1e-9, atol=1e-9)


def test_bf16_rounding_is_nearest_even():
    vals = np.array([1.0, 1.0 + 2**-8, 1.0 + 2**-8 + 2**-9, 1.0 + 3 * 2**-8, -2.5, 0.0])
    got = orc.round_bf16(vals)
    np.testing.assert_array_equal(got, [1.0, 1.0, 1.0 + 2**-7, 1.0 + 2**-6, -2.5, 0.0])


def test_gelu_grad_matches_finite_difference():
    x = np.linspace(-4, 4, 41)
    h = 1e-6
    fd = (orc.gelu(x + h) - orc.gelu(x - h)) / (2 * h)
    np.testing.assert_allclose(orc.gelu_grad(x), fd, rtol=1e-6, atol=1e-8)


def test_grn_oracle_matches_reference(golden):
    """The v2 GRN restatement against the reference's GlobalResponseNorm3d forward and
    autograd backward (tests/golden/grn.npz), zero-norm channel included."""
    fx = golden("grn.npz")
    for case in (0, 1):
        g = lambda k: fx[f"{case}/{k}"]  # noqa: E731
        y, norm, den = orc.grn_fwd(g("x"), g("gamma"), g("beta"), 1e-6)
        np.testing.assert_allclose(y, g("y"), rtol=1e-12, atol=1e-12)
        dx, dgamma, dbeta = orc.grn_bwd(g("dy"), g("x"), g("gamma"), norm, den)
        np.testing.assert_allclose(dx, g("dx"), rtol=1e-11, atol=1e-12)
        np.testing.assert_allclose(dgamma, g("dgamma").reshape(-1), rtol=1e-11, atol=1e-12)
        np.testing.assert_allclose(dbeta, g("dbeta").reshape(-1), rtol=1e-11, atol=1e-12)

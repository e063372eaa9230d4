"""v2 Global Response Norm on the sm_100a kernels, through the C ABI.

* float32 on the GPU against the reference's own float64 forward/backward
  (tests/golden/grn.npz, zero-norm channel included): relative error <= 1e-5;
* bfloat16 / float16 against the fp64 oracle evaluated on the same rounded inputs,
  over ragged sizes (voxel counts that are not multiples of 8, rows shorter and
  longer than one work item): relative L2 <= 4e-3 for the 16-bit outputs (their
  rounding), 1e-4 for the float32 dgamma / dbeta;
* the policy wrapper routes a training step to the fused op, and its gradients
  match the reference formula's autograd (relative L2 <= 2e-2 under autocast);
* every result is bitwise reproducible;
* the shape of the v2 Wide stage-0 expansion (2 x 192 x 160^3, bf16) against the
  reference formula on the GPU.
"""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

import mednext_accel_b200 as mx
from mednext_accel_b200 import _native as nat
from mednext_accel_b200.grn import grn_backward, grn_forward
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den > 0 else float(np.linalg.norm(a - b))


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().double().cpu().numpy()


@pytest.mark.parametrize("case", [0, 1])
def test_float32_matches_reference_golden(golden, case):
    fx = golden("grn.npz")
    g = lambda k: torch.from_numpy(fx[f"{case}/{k}"])  # noqa: E731
    x = g("x").float().cuda()
    gamma = g("gamma").float().cuda().contiguous()
    beta = g("beta").float().cuda().contiguous()
    dy = g("dy").float().cuda()
    y, norm, den = grn_forward(x, gamma, beta, 1e-6)
    dx, dgamma, dbeta = grn_backward(dy, x, gamma, norm, den)
    torch.cuda.synchronize()
    for got, want in ((y, "y"), (dx, "dx"), (dgamma, "dgamma"), (dbeta, "dbeta")):
        ref = fx[f"{case}/{want}"]
        scale = max(np.abs(ref).max(), 1e-30)
        assert np.abs(_np(got) - ref).max() / scale <= 1e-5, want


SHAPES = [
    (1, 1, (3, 5, 7)),        # 105 voxels: the scalar path, one short row
    (2, 3, (16, 16, 16)),     # 4096 voxels: rows shorter than a work item
    (3, 5, (33, 35, 37)),     # 42735 voxels, not a multiple of 8: scalar path, 3 items per row
    (2, 7, (40, 40, 41)),     # 65600 voxels: vector path with a ragged last item
    (1, 64, (32, 32, 32)),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n,c,spatial", SHAPES)
def test_16bit_matches_oracle(n, c, spatial, dtype):
    gen = torch.Generator().manual_seed(n * 1000 + c)
    x = torch.randn((n, c, *spatial), generator=gen).to(dtype)
    dy = torch.randn((n, c, *spatial), generator=gen).to(dtype)
    gamma = torch.randn((1, c, 1, 1, 1), generator=gen)
    beta = torch.randn((1, c, 1, 1, 1), generator=gen)
    y, norm, den = grn_forward(x.cuda(), gamma.cuda(), beta.cuda(), 1e-6)
    dx, dgamma, dbeta = grn_backward(dy.cuda(), x.cuda(), gamma.cuda(), norm, den)
    torch.cuda.synchronize()
    oy, onorm, oden = orc.grn_fwd(_np(x), _np(gamma), _np(beta), 1e-6)
    odx, odg, odb = orc.grn_bwd(_np(dy), _np(x), _np(gamma), onorm, oden)
    assert _rel_l2(_np(norm), onorm) <= 1e-5
    assert _rel_l2(_np(den), oden) <= 1e-5
    assert _rel_l2(_np(y), oy) <= 4e-3
    assert _rel_l2(_np(dx), odx) <= 4e-3
    assert _rel_l2(_np(dgamma).ravel(), odg) <= 1e-4
    assert _rel_l2(_np(dbeta).ravel(), odb) <= 1e-4


def test_results_are_bitwise_reproducible():
    gen = torch.Generator().manual_seed(5)
    x = torch.randn((2, 24, 40, 40, 40), generator=gen).to(torch.bfloat16).cuda()
    dy = torch.randn_like(x.float()).to(torch.bfloat16)
    gamma = torch.randn((1, 24, 1, 1, 1), generator=gen).cuda()
    beta = torch.randn((1, 24, 1, 1, 1), generator=gen).cuda()
    first = grn_forward(x, gamma, beta, 1e-6)
    back = grn_backward(dy, x, gamma, first[1], first[2])
    for _ in range(2):
        again = grn_forward(x, gamma, beta, 1e-6)
        back2 = grn_backward(dy, x, gamma, again[1], again[2])
        for a, b in zip((*first, *back), (*again, *back2), strict=True):
            assert torch.equal(a, b)


def test_wrapper_routes_training_to_the_fused_op_and_matches_reference_autograd():
    from torch.utils._python_dispatch import TorchDispatchMode

    class Spy(TorchDispatchMode):
        def __init__(self):
            super().__init__()
            self.ops = []

        def __torch_dispatch__(self, func, types, args=(), kwargs=None):
            self.ops.append(func._schema.name)
            return func(*args, **(kwargs or {}))

    torch.manual_seed(3)
    layer = mx.GlobalResponseNorm3d(48)
    with torch.no_grad():
        layer.gamma.normal_()
        layer.beta.normal_()
    ref = copy.deepcopy(layer).cuda()
    model = torch.nn.Sequential(copy.deepcopy(layer))
    from mednext_accel_b200.adaptive import ModelOptimizationContext

    assert mx.install_adaptive_operators(model, resolver=mx.PolicyResolver(),
                                         model_context=ModelOptimizationContext("mednext_v2", "wide", "none")) == 1
    model = model.cuda().train()
    x = torch.randn((2, 48, 24, 24, 24), device="cuda").to(torch.bfloat16)
    dy = torch.randn_like(x)
    xa = x.clone().requires_grad_()
    with Spy() as spy:
        y = model(xa)
    assert "mednext_accel_b200::grn_forward" in spy.ops
    y.backward(dy)
    xb = x.clone().requires_grad_()
    yr = ref(xb)
    yr.backward(dy)
    assert _rel_l2(_np(y), _np(yr)) <= 2e-2
    assert _rel_l2(_np(xa.grad), _np(xb.grad)) <= 2e-2
    assert _rel_l2(_np(model[0].gamma.grad), _np(ref.gamma.grad)) <= 2e-2
    assert _rel_l2(_np(model[0].beta.grad), _np(ref.beta.grad)) <= 2e-2
    # evaluation and no-grad calls use the reference formula
    model.eval()
    with Spy() as spy, torch.no_grad():
        model(x)
    assert "mednext_accel_b200::grn_forward" not in spy.ops


def test_v2_wide_stage0_expansion_shape_against_reference_formula():
    """2 x 192 x 160^3 bf16 (the v2 Wide stage-0 expansion; 3.1 GB per tensor)."""
    torch.manual_seed(4)
    x = torch.randn((2, 192, 160, 160, 160), device="cuda", dtype=torch.bfloat16)
    gamma = torch.randn((1, 192, 1, 1, 1), device="cuda")
    beta = torch.randn((1, 192, 1, 1, 1), device="cuda")
    y, norm, den = grn_forward(x, gamma, beta, 1e-6)
    want = mx.global_response_norm3d_reference(x, gamma, beta, 1e-6)
    diff = (y.float() - want.float()).norm() / want.float().norm()
    assert diff.item() <= 4e-3
    want_norm = torch.linalg.vector_norm(x.float(), dim=(2, 3, 4))
    assert torch.allclose(norm, want_norm, rtol=1e-4)
    del want
    dy = torch.randn_like(x)
    dx, dgamma, dbeta = grn_backward(dy, x, gamma, norm, den)
    torch.cuda.synchronize()
    assert torch.isfinite(dx.float()).all() and torch.isfinite(dgamma).all()
    # dbeta is the per-channel sum of dy over samples and voxels
    assert torch.allclose(dbeta.reshape(-1), dy.float().sum(dim=(0, 2, 3, 4)), rtol=1e-3, atol=1e-1)
    assert nat.device_error() == 0

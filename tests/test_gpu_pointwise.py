"""tcgen05 pointwise GEMMs (forward / input-grad / weight-grad with the fused
prologues and epilogues) against the CPU oracle on the same bf16 inputs."""

from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

from mednext_accel_b200 import _native as nat
from mednext_accel_b200.pointwise import gn_stats, pointwise_conv3d, pw_gemm, pw_wgrad
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def rand(shape, seed, dtype=torch.bfloat16, scale=1.0):
    gen = torch.Generator().manual_seed(zlib.crc32(repr((shape, seed)).encode()) % 100_000)
    return (torch.randn(shape, generator=gen, dtype=torch.float64) * scale).to(dtype)


def h(t):
    return t.detach().double().cpu().numpy()


def assert_close_bf16(got, want, what, rel_l2=4e-3, max_rel=2e-2):
    g = h(got)
    rl, mr = orc.rel_l2(g, want), orc.max_rel(g, want)
    assert rl <= rel_l2 and mr <= max_rel, f"{what}: rel_l2 {rl:.3e} max_rel {mr:.3e}"


GEMM_SHAPES = [
    # (n, cin, cout, spatial)
    (1, 32, 64, (16, 16, 16)),
    (2, 64, 32, (8, 8, 8)),
    (1, 1, 32, (16, 16, 16)),        # stem: K=1
    (2, 96, 192, (5, 7, 9)),         # odd voxel count, non-multiple-of-64 K
    (1, 128, 512, (8, 8, 8)),        # two N tiles, two K stages
    (1, 512, 2048, (4, 4, 4)),       # 8 N tiles, 8 K stages, 64 voxels
    (1, 2048, 512, (4, 4, 3)),       # deep K
    (1, 64, 128, (15, 15, 15)),      # up-block volume 15^3
]


@pytest.mark.parametrize("n,cin,cout,spatial", GEMM_SHAPES)
def test_forward_bias(n, cin, cout, spatial):
    x = rand((n, cin, *spatial), 1)
    w = rand((cout, cin), 2, scale=1 / np.sqrt(cin))
    b = rand((cout,), 3, torch.float32)
    y, _ = pw_gemm(x.cuda(), w.cuda(), cout, bias=b.cuda())
    want = orc.pointwise_fwd(h(x), h(w), h(b))
    assert_close_bf16(y, want, "y")


@pytest.mark.parametrize("n,cin,cout,spatial", GEMM_SHAPES[:5])
def test_forward_groupnorm_prologue_gelu_epilogue_chain(n, cin, cout, spatial):
    """expand(GroupNorm(t)) then project(gelu(u)) + residual, as in the block."""
    t = (rand((n, cin, *spatial), 4).double() * 3 + 1.5).to(torch.bfloat16)
    gamma = (1 + 0.2 * rand((cin,), 5, torch.float64)).float()
    beta = (0.2 * rand((cin,), 6, torch.float64)).float()
    we = rand((cout, cin), 7, scale=1 / np.sqrt(cin))
    be = rand((cout,), 8, torch.float32)
    tg = t.cuda()
    stats = gn_stats(tg, 1e-5)
    u, _ = pw_gemm(tg, we.cuda(), cout, prologue=nat.PRO_GROUPNORM, pro_stats=stats, pro_gamma=gamma.cuda(),
                   pro_beta=beta.cuda(), bias=be.cuda())
    z, mean, rstd = orc.groupnorm_fwd(h(t), h(gamma), h(beta))
    np.testing.assert_allclose(h(stats)[:, 0], mean, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(h(stats)[:, 1], rstd, rtol=1e-4, atol=1e-5)
    want_u = orc.pointwise_fwd(orc.round_bf16(z), h(we), h(be))
    assert_close_bf16(u, want_u, "u")
    wp = rand((cin, cout), 9, scale=1 / np.sqrt(cout))
    bp = rand((cin,), 10, torch.float32)
    res = rand((n, cin, *spatial), 11)
    y, _ = pw_gemm(u, wp.cuda(), cin, prologue=nat.PRO_GELU, bias=bp.cuda(), residual=res.cuda())
    want_y = orc.pointwise_fwd(orc.round_bf16(orc.gelu(h(u))), h(wp), h(bp)) + h(res)
    assert_close_bf16(y, want_y, "y")


@pytest.mark.parametrize("n,cin,cout,spatial", GEMM_SHAPES[:4])
def test_dgrad_gelu_grad_epilogue(n, cin, cout, spatial):
    dy = rand((n, cin, *spatial), 12)
    wt = rand((cout, cin), 13, scale=1 / np.sqrt(cin))  # already transposed weight
    u = rand((n, cout, *spatial), 14)
    du, _ = pw_gemm(dy.cuda(), wt.cuda(), cout, aux=u.cuda(), gelu_grad=True)
    want = orc.round_bf16(orc.pointwise_fwd(h(dy), h(wt), None)) * orc.gelu_grad(h(u))
    assert_close_bf16(du, want, "du")


@pytest.mark.parametrize("n,cin,cout,spatial", GEMM_SHAPES[:4])
def test_dgrad_groupnorm_backward_partials(n, cin, cout, spatial):
    du = rand((n, cin, *spatial), 15)
    wt = rand((cout, cin), 16, scale=1 / np.sqrt(cin))
    t = rand((n, cout, *spatial), 17)
    stats = gn_stats(t.cuda(), 1e-5)
    dz, part = pw_gemm(du.cuda(), wt.cuda(), cout, aux=t.cuda(), gn_bwd_stats=stats)
    from mednext_accel_b200.pointwise import gn_backward_from_partials

    gamma = (1 + 0.1 * rand((cout,), 18, torch.float64)).float().cuda()
    dt, dg, db = gn_backward_from_partials(dz, t.cuda(), stats, gamma, part)
    dzr = orc.round_bf16(orc.pointwise_fwd(h(du), h(wt), None))
    assert_close_bf16(dz, dzr, "dz")
    mean, rstd = h(stats)[:, 0], h(stats)[:, 1]
    want_dt, want_dg, want_db = orc.groupnorm_bwd(h(dz), h(t), mean, rstd, h(gamma))
    assert_close_bf16(dt, want_dt, "dt")
    np.testing.assert_allclose(h(dg), want_dg, rtol=2e-4, atol=2e-3)
    np.testing.assert_allclose(h(db), want_db, rtol=2e-4, atol=2e-3)


@pytest.mark.parametrize("n,cin,cout,spatial", GEMM_SHAPES)
@pytest.mark.parametrize("prologue", [nat.PRO_NONE, nat.PRO_GELU, nat.PRO_GROUPNORM])
def test_wgrad(n, cin, cout, spatial, prologue):
    g = rand((n, cout, *spatial), 19)
    a = rand((n, cin, *spatial), 20)
    kw = {}
    a_eff = h(a)
    if prologue == nat.PRO_GELU:
        a_eff = orc.round_bf16(orc.gelu(a_eff))
    elif prologue == nat.PRO_GROUPNORM:
        gamma = (1 + 0.1 * rand((cin,), 21, torch.float64)).float()
        beta = (0.1 * rand((cin,), 22, torch.float64)).float()
        stats = gn_stats(a.cuda(), 1e-5)
        kw = dict(pro_stats=stats, pro_gamma=gamma.cuda(), pro_beta=beta.cuda())
        z, _, _ = orc.groupnorm_fwd(a_eff, h(gamma), h(beta))
        a_eff = orc.round_bf16(z)
    dw, db = pw_wgrad(g.cuda(), a.cuda(), prologue=prologue, **kw)
    _, want_dw, want_db = orc.pointwise_bwd(h(g), a_eff, np.zeros((cout, cin)))
    assert orc.rel_l2(h(dw), want_dw) <= 2e-3, orc.rel_l2(h(dw), want_dw)
    assert orc.rel_l2(h(db), want_db) <= 1e-5


def test_wgrad_is_deterministic():
    g = rand((2, 64, 32, 32, 32), 23).cuda()
    a = rand((2, 128, 32, 32, 32), 24).cuda()
    a1 = pw_wgrad(g, a)
    a2 = pw_wgrad(g, a)
    assert torch.equal(a1[0], a2[0]) and torch.equal(a1[1], a2[1])


def test_pointwise_op_autograd():
    x = rand((2, 32, 8, 8, 8), 25).cuda().requires_grad_()
    w = rand((64, 32, 1, 1, 1), 26, scale=0.2).cuda().requires_grad_()
    b = rand((64,), 27).cuda().requires_grad_()
    y = pointwise_conv3d(x, w, b)
    dy = rand(tuple(y.shape), 28).cuda()
    dx, dw, db = torch.autograd.grad(y, (x, w, b), dy)
    want_y = orc.pointwise_fwd(h(x), h(w), h(b))
    assert_close_bf16(y, want_y, "y")
    wdx, wdw, wdb = orc.pointwise_bwd(h(dy), h(x), h(w))
    assert_close_bf16(dx, wdx, "dx")
    assert_close_bf16(dw.reshape(64, 32), wdw, "dw")
    assert_close_bf16(db, wdb, "db")


@pytest.mark.parametrize("cin,cout", [(64, 256), (256, 64), (32, 64)])
def test_epilogue_rings_wrap_many_times_per_cta(cin, cout):
    """2 x 64^3 voxels: every persistent CTA handles dozens of tiles, so the TMEM
    accumulators and the epilogue-operand ring (1, 2 or 4 slots, one or two
    epilogue groups depending on the tile width) wrap many times."""
    n, vox = 2, 64**3
    a = rand((n, cin, vox), 41)
    w = rand((cout, cin), 42, scale=cin**-0.5)
    u = rand((n, cout, vox), 43)
    t = rand((n, cout, vox), 44)
    stats = gn_stats(t.cuda(), 1e-5)
    ag, wg, ug, tg = a.cuda(), w.cuda(), u.cuda(), t.cuda()
    acc = torch.einsum("jk,skv->sjv", wg.float(), ag.float())
    # GELU' epilogue: round the GEMM to bf16, then multiply by GELU'(u) (fp32)
    du, _ = pw_gemm(ag, wg, cout, aux=ug, gelu_grad=True)
    uu = ug.float().requires_grad_()
    (gp,) = torch.autograd.grad(torch.nn.functional.gelu(uu), uu, torch.ones_like(uu))
    want = (acc.to(torch.bfloat16).float() * gp).to(torch.bfloat16)
    assert orc.rel_l2(h(du), h(want)) <= 4e-3
    # GroupNorm-backward partial sums against torch on the same dz
    from mednext_accel_b200.pointwise import gn_backward_from_partials

    dz, part = pw_gemm(ag, wg, cout, aux=tg, gn_bwd_stats=stats)
    assert orc.rel_l2(h(dz), h(acc.to(torch.bfloat16))) <= 2e-3
    _, dg, db = gn_backward_from_partials(dz, tg, stats, torch.ones(cout, device="cuda"), part)
    xhat = (tg.float() - stats[:, 0].view(n, cout, 1)) * stats[:, 1].view(n, cout, 1)
    for got, terms in ((db, dz.float()), (dg, dz.float() * xhat)):
        want, scale = terms.sum(dim=(0, 2)), terms.abs().sum(dim=(0, 2))
        assert bool(((got - want).abs() <= 1e-5 * scale + 1e-3).all())
    assert nat.device_error() == 0


def _all_finite_bf16(channels):
    """Every finite bf16 value once, laid out as [1, channels, vox] (zero padded)."""
    bits = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    vals = bits[torch.isfinite(bits.float())]
    vox = -(-vals.numel() // channels)
    vox = -(-vox // 64) * 64
    flat = torch.zeros(channels * vox, dtype=torch.bfloat16)
    flat[: vals.numel()] = vals
    return flat.view(1, channels, vox).cuda(), vals.numel()


def _compare_to_torch(got, want, what):
    """Same bf16 rounding as torch's erf-form GELU except within one bf16 ulp on
    a small fraction of elements, or within 2e-6 absolute (the far negative tail,
    where fp32 1 + erf(x) loses its digits in the reference formula)."""
    g, w = got.float().cpu().flatten(), want.float().cpu().flatten()
    ulp = torch.maximum(w.abs(), torch.full_like(w, 1e-30)) * 2.0**-7
    ok = ((g - w).abs() <= ulp) | ((g - w).abs() <= 2e-6)
    assert bool(ok.all()), f"{what}: worst {(g - w).abs().max().item():.3e} at {w[~ok][:4].tolist()}"
    differ = (g != w).float().mean().item()
    assert differ <= 5e-3, f"{what}: {differ:.2e} of the elements differ in the last bf16 bit"


def test_gelu_prologue_matches_torch_on_every_bf16_value():
    a, count = _all_finite_bf16(16)
    eye = torch.eye(16, dtype=torch.bfloat16, device="cuda")
    y, _ = pw_gemm(a, eye, 16, prologue=nat.PRO_GELU)  # identity weight: y = bf16(gelu(a))
    want = torch.nn.functional.gelu(a.float()).to(torch.bfloat16)
    _compare_to_torch(y.flatten()[:count], want.flatten()[:count], "gelu")


def test_gelu_grad_epilogue_matches_torch_on_every_bf16_value():
    u, count = _all_finite_bf16(16)
    ones = torch.ones_like(u)
    eye = torch.eye(16, dtype=torch.bfloat16, device="cuda")
    du, _ = pw_gemm(ones, eye, 16, aux=u, gelu_grad=True)  # 1 * gelu'(u)
    uu = u.float().requires_grad_()
    (want,) = torch.autograd.grad(torch.nn.functional.gelu(uu), uu, torch.ones_like(uu))
    _compare_to_torch(du.flatten()[:count], want.to(torch.bfloat16).flatten()[:count], "gelu'")


PRO_OUT_SHAPES = [
    (1, 32, 64, (16, 16, 16)),
    (2, 64, 32, (8, 8, 8)),
    (2, 96, 192, (5, 7, 9)),     # odd voxel count: first-generation kernel + separate prologue output
    (1, 128, 512, (8, 8, 8)),    # two K stages per tile
    (1, 64, 32, (64, 64, 64)),   # 2048 tiles: every ring stage is stored and released many times
]


@pytest.mark.parametrize("n,cin,cout,spatial", PRO_OUT_SHAPES)
@pytest.mark.parametrize("prologue", [nat.PRO_GELU, nat.PRO_GROUPNORM])
def test_prologue_output(n, cin, cout, spatial, prologue):
    """pro_out holds pro(a) exactly as the GEMM consumed it; y is unchanged by asking for it."""
    a = (rand((n, cin, *spatial), 21).double() * 2 + 0.5).to(torch.bfloat16).cuda()
    w = rand((cout, cin), 22, scale=1 / np.sqrt(cin)).cuda()
    b = rand((cout,), 23, torch.float32).cuda()
    kw = {}
    if prologue == nat.PRO_GROUPNORM:
        gamma = (1 + 0.2 * rand((cin,), 24, torch.float64)).float().cuda()
        beta = (0.2 * rand((cin,), 25, torch.float64)).float().cuda()
        kw = dict(pro_stats=gn_stats(a, 1e-5), pro_gamma=gamma, pro_beta=beta)
    y0, _ = pw_gemm(a, w, cout, prologue=prologue, bias=b, **kw)
    g = torch.full_like(a, float("nan"))
    y1, _ = pw_gemm(a, w, cout, prologue=prologue, bias=b, pro_out=g, **kw)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)
    if prologue == nat.PRO_GELU:
        want = orc.round_bf16(orc.gelu(h(a)))
    else:
        z, _, _ = orc.groupnorm_fwd(h(a), h(kw["pro_gamma"]), h(kw["pro_beta"]))
        want = orc.round_bf16(z)
    assert not torch.isnan(g).any()
    assert_close_bf16(g, want, "pro_out", rel_l2=2e-3, max_rel=1e-2)
    # the same prologue through the identity GEMM is bit-identical to pro_out
    if cin <= 256:
        eye = torch.eye(cin, dtype=torch.bfloat16, device="cuda")
        yi, _ = pw_gemm(a, eye, cin, prologue=prologue, **kw)
        assert torch.equal(yi, g)


def test_gelu_prologue_output_on_every_bf16_value():
    a, count = _all_finite_bf16(16)
    eye = torch.eye(16, dtype=torch.bfloat16, device="cuda")
    g = torch.empty_like(a)
    y, _ = pw_gemm(a, eye, 16, prologue=nat.PRO_GELU, pro_out=g)
    assert torch.equal(y, g)


GELU_BWD_SHAPES = [
    # (n, c = dy channels, h = GEMM output channels, spatial)
    (1, 32, 64, (16, 16, 16)),
    (2, 64, 64, (8, 8, 8)),
    (1, 32, 112, (16, 16, 16)),
    (2, 32, 64, (9, 10, 16)),     # voxel count not a multiple of the 128-voxel tile
    (1, 32, 64, (64, 64, 64)),    # 2048 tiles: g tiles and ring stages reused many times
    (1, 16, 48, (3, 4, 8)),       # a single tile
]


@pytest.mark.parametrize("n,c,hc,spatial", GELU_BWD_SHAPES)
def test_fused_gelu_backward_matches_separate_kernels(n, c, hc, spatial):
    from mednext_accel_b200.pointwise import pw_gelu_bwd

    dy = rand((n, c, *spatial), 31).cuda()
    u = (rand((n, hc, *spatial), 32).double() * 1.5).to(torch.bfloat16).cuda()
    w = rand((c, hc), 33, scale=1 / np.sqrt(hc)).cuda()   # project weight [c, h]
    wpt = w.t().contiguous()
    out = pw_gelu_bwd(dy, wpt, u)
    assert out is not None
    du, dw, db = out
    du_ref, _ = pw_gemm(dy, wpt, hc, aux=u, gelu_grad=True)
    dw_ref, db_ref = pw_wgrad(dy, u, prologue=nat.PRO_GELU)
    torch.cuda.synchronize()
    assert torch.equal(du, du_ref)  # same input-grad arithmetic
    assert orc.rel_l2(h(dw), h(dw_ref)) <= 2e-3
    assert orc.rel_l2(h(db), h(db_ref)) <= 1e-5
    # and against the oracle: dW = dy . GELU(u)^T on the same bf16 inputs
    g = orc.round_bf16(orc.gelu(h(u)))
    want_dw = np.einsum("ncv,nhv->ch", h(dy).reshape(n, c, -1), g.reshape(n, hc, -1))
    assert orc.rel_l2(h(dw), want_dw) <= 4e-3
    assert orc.rel_l2(h(db), h(dy).reshape(n, c, -1).sum(axis=(0, 2))) <= 1e-5


GN_BWD_SHAPES = [
    # (n, h = du channels, c = dz / t channels, spatial)
    (1, 64, 32, (16, 16, 16)),
    (2, 64, 64, (8, 8, 8)),
    (2, 48, 112, (9, 10, 16)),
    (1, 64, 32, (64, 64, 64)),
]


@pytest.mark.parametrize("n,hc,c,spatial", GN_BWD_SHAPES)
def test_fused_groupnorm_backward_matches_separate_kernels(n, hc, c, spatial):
    from mednext_accel_b200.pointwise import gn_backward_from_partials, pw_gn_bwd_fused

    du = rand((n, hc, *spatial), 51).cuda()
    t = (rand((n, c, *spatial), 52).double() * 2 + 0.5).to(torch.bfloat16).cuda()
    w = rand((hc, c), 53, scale=1 / np.sqrt(c)).cuda()   # expand weight [h, c]
    wt = w.t().contiguous()
    gamma = (1 + 0.2 * rand((c,), 54, torch.float64)).float().cuda()
    beta = (0.2 * rand((c,), 55, torch.float64)).float().cuda()
    stats = gn_stats(t, 1e-5)
    out = pw_gn_bwd_fused(du, wt, t, stats, gamma, beta)
    assert out is not None
    dz, part, dw, db = out
    dz_ref, part_ref = pw_gemm(du, wt, c, aux=t, gn_bwd_stats=stats)
    dw_ref, db_ref = pw_wgrad(du, t, prologue=nat.PRO_GROUPNORM, pro_stats=stats, pro_gamma=gamma, pro_beta=beta)
    torch.cuda.synchronize()
    assert torch.equal(dz, dz_ref)  # same input-grad arithmetic
    got = gn_backward_from_partials(dz, t, stats, gamma, part)
    want = gn_backward_from_partials(dz_ref, t, stats, gamma, part_ref)
    for a, b in zip(got, want, strict=True):
        assert torch.equal(a, b)  # the same GroupNorm-backward partial sums
    assert orc.rel_l2(h(dw), h(dw_ref)) <= 1e-5  # same GroupNorm(t) values, another summation order
    assert orc.rel_l2(h(db), h(db_ref)) <= 1e-5


MLP_SHAPES = [
    # (n, c, h, c2, spatial, residual)
    (1, 32, 64, 32, (16, 16, 16), True),
    (2, 32, 64, 64, (8, 8, 8), False),
    (1, 64, 128, 32, (15, 15, 16), True),   # the up block's level-0 shapes
    (2, 16, 48, 16, (9, 10, 16), True),     # voxel count not a multiple of 128
    (1, 32, 64, 32, (64, 64, 64), True),    # 2048 tiles: rings and g tiles wrap many times
]


@pytest.mark.parametrize("n,c,hc,c2,spatial,with_res", MLP_SHAPES)
def test_fused_expansion_matches_separate_kernels(n, c, hc, c2, spatial, with_res):
    """u and y bit for bit against the two separate GEMMs (same roundings, same MMAs)."""
    from mednext_accel_b200.pointwise import pw_mlp_fwd

    t = (rand((n, c, *spatial), 61).double() * 2 + 0.5).to(torch.bfloat16).cuda()
    gamma = (1 + 0.2 * rand((c,), 62, torch.float64)).float().cuda()
    beta = (0.2 * rand((c,), 63, torch.float64)).float().cuda()
    we = rand((hc, c), 64, scale=1 / np.sqrt(c)).cuda()
    be = rand((hc,), 65, torch.float32).cuda()
    wp = rand((c2, hc), 66, scale=1 / np.sqrt(hc)).cuda()
    bp = rand((c2,), 67, torch.float32).cuda()
    res = rand((n, c2, *spatial), 68).cuda() if with_res else None
    stats = gn_stats(t, 1e-5)
    out = pw_mlp_fwd(t, stats, gamma, beta, we, be, wp, bp, res)
    assert out is not None
    u, y = out
    u_ref, _ = pw_gemm(t, we, hc, prologue=nat.PRO_GROUPNORM, pro_stats=stats, pro_gamma=gamma, pro_beta=beta,
                       bias=be)
    y_ref, _ = pw_gemm(u_ref, wp, c2, prologue=nat.PRO_GELU, bias=bp, residual=res)
    torch.cuda.synchronize()
    assert torch.equal(u, u_ref)
    assert torch.equal(y, y_ref)


def test_fused_gelu_backward_declines_uncovered_shapes():
    from mednext_accel_b200.pointwise import pw_gelu_bwd

    dy = rand((1, 32, 8, 8, 8), 34).cuda()
    for hh, cc in ((128, 32), (64, 96)):
        d = rand((1, cc, 8, 8, 8), 35).cuda()
        u = rand((1, hh, 8, 8, 8), 36).cuda()
        assert pw_gelu_bwd(d, torch.zeros((hh, cc), dtype=torch.bfloat16, device="cuda"), u) is None
    assert dy is not None


def test_no_device_error_recorded():
    assert nat.device_error() == 0


# Deep, narrow levels: few 128-voxel tiles and K up to 2048 (long K loops through the
# ring, two samples, ragged voxel counts).
SPLITK_SHAPES = [
    (1, 1024, 256, (16, 16, 16)),   # level 3 compress: 32 tiles x 16 K stages
    (1, 2048, 512, (8, 8, 8)),      # level 4 compress: 8 tiles x 32 K stages
    (2, 1024, 256, (8, 8, 9)),      # two samples, ragged voxel count
]


@pytest.mark.parametrize("n,cin,cout,spatial", SPLITK_SHAPES)
def test_split_k_gelu_prologue_bias_residual(n, cin, cout, spatial):
    u = rand((n, cin, *spatial), 41)
    w = rand((cout, cin), 42, scale=1 / np.sqrt(cin))
    b = rand((cout,), 43, torch.float32)
    res = rand((n, cout, *spatial), 44)
    y, _ = pw_gemm(u.cuda(), w.cuda(), cout, prologue=nat.PRO_GELU, bias=b.cuda(), residual=res.cuda())
    want = orc.pointwise_fwd(orc.round_bf16(orc.gelu(h(u))), h(w), h(b))
    want = orc.round_bf16(want) + h(res)
    assert_close_bf16(y, want, "y")


@pytest.mark.parametrize("n,cin,cout,spatial", SPLITK_SHAPES[:2])
def test_split_k_dgrad_epilogues(n, cin, cout, spatial):
    from mednext_accel_b200.pointwise import gn_backward_from_partials

    du = rand((n, cin, *spatial), 45)
    wt = rand((cout, cin), 46, scale=1 / np.sqrt(cin))
    t = rand((n, cout, *spatial), 47)
    stats = gn_stats(t.cuda(), 1e-5)
    dz, part = pw_gemm(du.cuda(), wt.cuda(), cout, aux=t.cuda(), gn_bwd_stats=stats)
    gamma = (1 + 0.1 * rand((cout,), 48, torch.float64)).float().cuda()
    dt, dg, db = gn_backward_from_partials(dz, t.cuda(), stats, gamma, part)
    assert_close_bf16(dz, orc.round_bf16(orc.pointwise_fwd(h(du), h(wt), None)), "dz")
    mean, rstd = h(stats)[:, 0], h(stats)[:, 1]
    want_dt, want_dg, want_db = orc.groupnorm_bwd(h(dz), h(t), mean, rstd, h(gamma))
    assert_close_bf16(dt, want_dt, "dt")
    np.testing.assert_allclose(h(dg), want_dg, rtol=2e-4, atol=2e-3)
    np.testing.assert_allclose(h(db), want_db, rtol=2e-4, atol=2e-3)
    u = rand((n, cout, *spatial), 49)
    dv, _ = pw_gemm(du.cuda(), wt.cuda(), cout, aux=u.cuda(), gelu_grad=True)
    want = orc.round_bf16(orc.pointwise_fwd(h(du), h(wt), None)) * orc.gelu_grad(h(u))
    assert_close_bf16(dv, want, "dv")


def test_split_k_results_are_bitwise_reproducible():
    """Repeated launches (as in a replayed CUDA graph) give identical bits."""
    n, cin, cout, spatial = SPLITK_SHAPES[0]
    u = rand((n, cin, *spatial), 51).cuda()
    w = rand((cout, cin), 52, scale=1 / np.sqrt(cin)).cuda()
    b = rand((cout,), 53, torch.float32).cuda()
    first, _ = pw_gemm(u, w, cout, prologue=nat.PRO_GELU, bias=b)
    for _ in range(3):
        again, _ = pw_gemm(u, w, cout, prologue=nat.PRO_GELU, bias=b)
        assert torch.equal(first, again)
    assert nat.device_error() == 0


GELU_OUT_SHAPES = [
    (1, 32, 64, (16, 16, 16)),     # level 0: GroupNorm prologue, 12 epilogue warps
    (2, 64, 192, (8, 8, 8)),       # level 1 widths, two samples
    (1, 96, 64, (8, 8, 16)),       # K not a multiple of 64
    (1, 256, 1024, (8, 8, 8)),     # deep level: narrow N tiles
]


@pytest.mark.parametrize("n,cin,cout,spatial", GELU_OUT_SHAPES)
def test_gelu_output_matches_the_gelu_prologue_path_bit_for_bit(n, cin, cout, spatial):
    """(u, g) from the expand GEMM's GELU-output epilogue: u equals the plain expand
    GEMM, g equals GELU(u) as the compress GEMM's prologue computes it (its prologue
    output), and the compress GEMM on g equals the compress GEMM with the GELU prologue."""
    from mednext_accel_b200.pointwise import pw_gemm_gelu_out

    t = (rand((n, cin, *spatial), 61).double() * 2 + 0.3).to(torch.bfloat16).cuda()
    gamma = (1 + 0.2 * rand((cin,), 62, torch.float64)).float().cuda()
    beta = (0.2 * rand((cin,), 63, torch.float64)).float().cuda()
    we = rand((cout, cin), 64, scale=1 / np.sqrt(cin)).cuda()
    be = rand((cout,), 65, torch.float32).cuda()
    stats = gn_stats(t, 1e-5)
    gn = dict(prologue=nat.PRO_GROUPNORM, pro_stats=stats, pro_gamma=gamma, pro_beta=beta, bias=be)
    out = pw_gemm_gelu_out(t, we, cout, **gn)
    assert out is not None
    u, g = out
    u_ref, _ = pw_gemm(t, we, cout, **gn)
    assert torch.equal(u, u_ref)
    wp = rand((cin, cout), 66, scale=1 / np.sqrt(cout)).cuda()
    bp = rand((cin,), 67, torch.float32).cuda()
    g_ref = torch.empty_like(u)
    y_ref, _ = pw_gemm(u, wp, cin, prologue=nat.PRO_GELU, bias=bp, pro_out=g_ref)
    assert torch.equal(g, g_ref)
    y, _ = pw_gemm(g, wp, cin, bias=bp)
    assert torch.equal(y, y_ref)
    want_g = orc.round_bf16(orc.gelu(h(u)))
    assert_close_bf16(g, want_g, "g")


def test_gelu_output_declines_unaligned_rows():
    from mednext_accel_b200.pointwise import pw_gemm_gelu_out

    t = rand((1, 32, 5, 5, 5), 68).cuda()  # 125 voxels: rows not 16-byte aligned
    we = rand((64, 32), 69, scale=0.2).cuda()
    assert pw_gemm_gelu_out(t, we, 64) is None

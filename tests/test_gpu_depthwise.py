"""Depthwise Conv3d kernels on the GPU against the CPU oracle and the golden
vectors of the reference (stride 1, stride 2 and transposed; every dtype)."""

from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch
from torch.nn import functional as F

from mednext_accel_b200 import _native as nat
from mednext_accel_b200 import depthwise as dwk
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

# fp32 parity bar of the north star: max relative error <= 1e-5; 16-bit outputs
# are compared with the oracle evaluated on the same rounded inputs.
TOL = {
    torch.float64: dict(max_rel=1e-12),
    torch.float32: dict(max_rel=1e-5),
    torch.bfloat16: dict(max_rel=1.6e-2, rel_l2=4e-3),
    torch.float16: dict(max_rel=2e-3, rel_l2=1e-3),
}


def check(got: torch.Tensor, want: np.ndarray, dtype: torch.dtype, what: str, scale: float = 1.0) -> None:
    g = got.detach().double().cpu().numpy()
    tol = TOL[dtype]
    mr = orc.max_rel(g, want)
    assert mr <= tol["max_rel"] * scale, f"{what}: max_rel {mr:.3e}"
    if "rel_l2" in tol:
        rl = orc.rel_l2(g, want)
        assert rl <= tol["rel_l2"] * scale, f"{what}: rel_l2 {rl:.3e}"


def seed_of(*key) -> int:
    return zlib.crc32(repr(key).encode()) % 100_000


def rand(shape, dtype, seed, scale=1.0):
    gen = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=gen, dtype=torch.float64) * scale).to(dtype)


def host(t: torch.Tensor) -> np.ndarray:
    return t.double().numpy()


SHAPES = [(2, 3, 5, 6, 7), (1, 4, 8, 16, 16), (1, 2, 9, 10, 24), (2, 5, 6, 3, 33), (1, 3, 12, 12, 130)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16, torch.float64])
@pytest.mark.parametrize("k", [1, 3, 5, 7])
@pytest.mark.parametrize("shape", SHAPES)
def test_stride1_forward_dgrad_wgrad(dtype, k, shape):
    seed = seed_of(str(dtype), k, shape)
    x = rand(shape, dtype, seed)
    w = rand((shape[1], 1, k, k, k), dtype, seed + 1, scale=1 / np.sqrt(k**3))
    b = rand((shape[1],), dtype, seed + 2)
    dy = rand(shape, dtype, seed + 3)
    xg, wg, bg, dyg = (t.cuda() for t in (x, w, b, dy))
    y = dwk.dw_forward(xg, wg, bg, k)
    dx = dwk.dw_dgrad(dyg, wg, k)
    dw, db = dwk.dw_wgrad(xg, dyg, k)
    torch.cuda.synchronize()
    check(y, orc.dw_fwd(host(x), host(w), host(b), k), dtype, "y")
    check(dx, orc.dw_dgrad(host(dy), host(w), k), dtype, "dx")
    want_dw, want_db = orc.dw_wgrad(host(x), host(dy), k)
    # weight grads reduce thousands of products: bf16/fp16 output rounding only
    check(dw, want_dw, dtype, "dw", scale=2.0)
    check(db, want_db, dtype, "db", scale=2.0)


@pytest.mark.parametrize("k", [1, 3, 5])
def test_stride1_against_reference_golden_fp64(golden, k):
    g = golden("depthwise.npz")
    t = f"s1_k{k}/"
    cu = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    y = dwk.dw_forward(cu(g[t + "x"]), cu(g[t + "w"]), cu(g[t + "b"]), k)
    dx = dwk.depthwise_input_grad(cu(g[t + "dy"]), cu(g[t + "w"]), block=128)
    dw = dwk.depthwise_weight_grad(cu(g[t + "x"]), cu(g[t + "dy"]), splits=4, block=128, kernel_size=k)
    # reference tolerances, tests/ops/test_depthwise.py:61-62
    torch.testing.assert_close(y.cpu(), torch.from_numpy(g[t + "y"]), rtol=2e-12, atol=2e-12)
    torch.testing.assert_close(dx.cpu(), torch.from_numpy(g[t + "dx"]), rtol=2e-12, atol=2e-12)
    torch.testing.assert_close(dw.cpu(), torch.from_numpy(g[t + "dw"]), rtol=2e-5, atol=2e-5)


def test_stride2_and_transpose_against_reference_golden_fp64(golden):
    g = golden("depthwise.npz")
    cu = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    for k in (3, 5):
        t = f"s2_k{k}/"
        x = g[t + "x"]
        y = dwk.s2_forward(cu(x), cu(g[t + "w"]), cu(g[t + "b"]), k)
        dx = dwk.depthwise_stride2_input_grad(cu(g[t + "dy"]), cu(g[t + "w"]), x.shape[2:], block=128)
        dw, db = dwk.s2_wgrad(cu(x), cu(g[t + "dy"]), k)
        for got, key in ((y, "y"), (dx, "dx"), (dw, "dw"), (db, "db")):
            torch.testing.assert_close(got.cpu(), torch.from_numpy(g[t + key]), rtol=2e-12, atol=2e-12)
        t = f"t_k{k}/"
        y = dwk.t_forward(cu(g[t + "x"]), cu(g[t + "w"]), cu(g[t + "b"]), k)
        dx = dwk.t_dgrad(cu(g[t + "dy"]), cu(g[t + "w"]), k)
        dw = dwk.depthwise_transpose_weight_grad(cu(g[t + "x"]), cu(g[t + "dy"]), splits=4, block=128, kernel_size=k)
        _, db = dwk.t_wgrad(cu(g[t + "x"]), cu(g[t + "dy"]), k)
        for got, key in ((y, "y"), (dx, "dx"), (dw, "dw"), (db, "db")):
            torch.testing.assert_close(got.cpu(), torch.from_numpy(g[t + key]), rtol=2e-12, atol=2e-12)


S2_SHAPES = [(2, 3, 5, 6, 7), (1, 4, 16, 16, 16), (1, 2, 9, 12, 17)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("k", [1, 3, 5, 7])
@pytest.mark.parametrize("shape", S2_SHAPES)
def test_stride2_and_transpose(dtype, k, shape):
    seed = seed_of("s2", str(dtype), k, shape)
    n, c = shape[:2]
    w = rand((c, 1, k, k, k), dtype, seed + 1, scale=1 / np.sqrt(k**3))
    b = rand((c,), dtype, seed + 2)
    # down block: big -> small
    x = rand(shape, dtype, seed)
    y = dwk.s2_forward(x.cuda(), w.cuda(), b.cuda(), k)
    dy = rand(tuple(y.shape), dtype, seed + 3)
    dx = dwk.s2_dgrad(dy.cuda(), w.cuda(), shape[2:], k)
    dw, db = dwk.s2_wgrad(x.cuda(), dy.cuda(), k)
    check(y, orc.s2_fwd(host(x), host(w), host(b), k), dtype, "s2 y")
    check(dx, orc.s2_dgrad(host(dy), host(w), shape[2:], k), dtype, "s2 dx")
    want_dw, want_db = orc.s2_wgrad(host(x), host(dy), k)
    check(dw, want_dw, dtype, "s2 dw", scale=2.0)
    check(db, want_db, dtype, "s2 db", scale=2.0)
    # up block: small -> big (2S-1)
    xs = rand(shape, dtype, seed + 4)
    yt = dwk.t_forward(xs.cuda(), w.cuda(), b.cuda(), k)
    dyt = rand(tuple(yt.shape), dtype, seed + 5)
    dxt = dwk.t_dgrad(dyt.cuda(), w.cuda(), k)
    dwt, dbt = dwk.t_wgrad(xs.cuda(), dyt.cuda(), k)
    check(yt, orc.t_fwd(host(xs), host(w), host(b), k), dtype, "t y")
    check(dxt, orc.t_dgrad(host(dyt), host(w), k), dtype, "t dx")
    want_dw, want_db = orc.t_wgrad(host(xs), host(dyt), k)
    check(dwt, want_dw, dtype, "t dw", scale=2.0)
    check(dbt, want_db, dtype, "t db", scale=2.0)


def test_config1_fp32_full_size():
    """The single depthwise-conv workload: N=1, C=32, 64^3, k=3, fp32, bias; weights ~N(0,1)/sqrt(27),
    seed 0; y, grad_input, grad_weight against F.conv3d autograd on CPU."""
    torch.manual_seed(0)
    x = torch.randn(1, 32, 64, 64, 64)
    dy = torch.randn(1, 32, 64, 64, 64)
    w = torch.randn(32, 1, 3, 3, 3) / np.sqrt(27)
    b = torch.randn(32)
    xr = x.double().requires_grad_()
    wr = w.double().requires_grad_()
    br = b.double().requires_grad_()
    yr = F.conv3d(xr, wr, br, padding=1, groups=32)
    dxr, dwr, dbr = torch.autograd.grad(yr, (xr, wr, br), dy.double())
    op = dwk.depthwise_conv3d_regular
    xg = x.cuda().requires_grad_()
    wg = w.cuda().requires_grad_()
    bg = b.cuda().requires_grad_()
    yg = op(xg, wg, bg, 3, 32, 64, 8, 512, 128, True, True)
    dxg, dwg, dbg = torch.autograd.grad(yg, (xg, wg, bg), dy.cuda())
    for got, want, name in ((yg, yr, "y"), (dxg, dxr, "dx"), (dwg, dwr, "dw"), (dbg, dbr, "db")):
        mr = orc.max_rel(got.detach().double().cpu().numpy(), want.detach().numpy())
        assert mr <= 1e-5, f"{name}: {mr:.3e}"


def test_weight_grad_is_deterministic():
    x = rand((2, 8, 32, 32, 32), torch.bfloat16, 5).cuda()
    dy = rand((2, 8, 32, 32, 32), torch.bfloat16, 6).cuda()
    a = dwk.dw_wgrad(x, dy, 3)
    b = dwk.dw_wgrad(x, dy, 3)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    a = dwk.t_wgrad(x, rand((2, 8, 63, 63, 63), torch.bfloat16, 7).cuda(), 3)
    assert torch.isfinite(a[0].float()).all()


PACKED_SHAPES = [
    (1, 3, 6, 40, 256),      # 8 column groups per row (permuted lanes), two W tiles, ragged H tile
    (2, 2, 5, 9, 64),        # 4 column groups per row
    (1, 2, 11, 70, 128),     # three H tiles, the last one ragged
    (1, 2, 7, 8, 16),        # one column group per row
    (1, 32, 128, 128, 128),  # the benchmark's level-0 shape
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", PACKED_SHAPES)
def test_packed_k3_kernel_is_bit_exact_with_fp32_kernel(dtype, shape):
    """k = 3 on 16-bit tensors runs the packed-FMA kernel, which sums each output in
    the fp32 kernel's order: its outputs are the fp32 kernel's outputs on the same
    inputs, rounded once (forward with bias, input grad with addend)."""
    seed = seed_of("packed", str(dtype), shape)
    x = rand(shape, dtype, seed).cuda()
    w = rand((shape[1], 1, 3, 3, 3), dtype, seed + 1, scale=0.2).cuda()
    b = rand((shape[1],), dtype, seed + 2).cuda()
    a = rand(shape, dtype, seed + 3).cuda()
    y, stats = dwk.dw_forward(x, w, b, 3, gn_eps=1e-5)
    assert torch.equal(y, dwk.dw_forward(x.float(), w.float(), b.float(), 3).to(dtype))
    dx = dwk.dw_dgrad(x, w, 3, addend=a)
    assert torch.equal(dx, dwk.dw_dgrad(x.float(), w.float(), 3, addend=a.float()).to(dtype))
    yf = y.double().reshape(shape[0] * shape[1], -1)
    torch.testing.assert_close(stats[:, 0].double(), yf.mean(1), rtol=1e-5, atol=1e-6)
    rstd = 1 / torch.sqrt(yf.var(1, unbiased=False) + 1e-5)
    torch.testing.assert_close(stats[:, 1].double(), rstd, rtol=1e-5, atol=1e-6)


WGRAD_SHAPES = [
    (1, 3, 6, 40, 256),      # two W tiles, ragged H tile
    (2, 2, 5, 9, 64),
    (1, 2, 11, 70, 128),     # three H tiles, the last one ragged
    (1, 2, 7, 8, 16),
    (2, 8, 32, 32, 32),
    (1, 32, 128, 128, 128),  # the benchmark's level-0 shape
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("k", [3, 5, 7])
@pytest.mark.parametrize("shape", WGRAD_SHAPES)
def test_weight_grad_16bit_is_bit_exact_with_fp32_kernel(dtype, k, shape):
    """The stride-1 weight grads on 16-bit tensors (k = 3, and the grouped k = 5 / 7
    kernel) multiply the packed elements with mixed-precision FMAs (16-bit operands,
    fp32 sums) in the fp32 kernel's order on the same tiling; a product of two
    16-bit floats is exact in fp32, so the weight and bias grads are the fp32
    kernel's on the widened inputs, rounded once."""
    seed = seed_of("wgrad16", str(dtype), k, shape)
    x = rand(shape, dtype, seed).cuda()
    dy = rand(shape, dtype, seed + 1).cuda()
    dw, db = dwk.dw_wgrad(x, dy, k)
    dw32, db32 = dwk.dw_wgrad(x.float(), dy.float(), k)
    assert torch.equal(dw, dw32.to(dtype)) and torch.equal(db, db32.to(dtype))
    assert nat.device_error() == 0


TC_SHAPES = [
    (1, 32, 64, 128, 128),   # level-0 planes (64-column tiles, 32-row tiles)
    (1, 64, 64, 64, 64),     # level 1
    (1, 128, 32, 32, 32),    # level 2 (32-column tiles)
    (1, 256, 16, 16, 16),    # level 3 (16-column tiles, one 16-row tile)
    (1, 3, 6, 40, 256),      # four W tiles, a ragged second H tile
    (2, 2, 5, 9, 64),        # short planes and depth
    (2, 5, 17, 33, 48),      # 16-column tiles, 33 rows: a one-row last H tile
]


def _assert_one_rounding(got: torch.Tensor, want32: torch.Tensor, what: str) -> None:
    """got (16-bit) is want32 (fp32) rounded once, up to the few fp32 ulps by which the
    tensor-core sum may differ from the FMA sum: every element within one 16-bit ulp
    (plus an fp32-level allowance where the taps cancel), and all but a few (values
    within a few fp32 ulps of a rounding boundary: at most 1 %, measured about 0.3 %
    for fp16 at k = 5) exactly the rounded fp32 value."""
    dt = got.dtype
    ulp = torch.finfo(dt).eps
    diff = (got.float() - want32).abs()
    bound = ulp * want32.abs() + 2.0**-18 * want32.abs().max()
    assert bool((diff <= bound).all()), f"{what}: {(diff / bound).max().item():.3f} x the bound"
    mismatch = (got != want32.to(dt)).sum().item()
    assert mismatch <= max(4, got.numel() // 100), f"{what}: {mismatch} of {got.numel()} not the rounded fp32 value"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("k", [5, 7])
@pytest.mark.parametrize("shape", TC_SHAPES)
def test_tensor_core_k5_k7_kernels_match_fp32_kernel(dtype, k, shape):
    """k = 5 and 7 on 16-bit tensors with W a multiple of 16 run on the tensor cores
    (band matrices along W, one MMA per (kd, kh) tap pair, fp32 accumulation in TMEM):
    the forward with bias and GroupNorm statistics and the input grad with the
    residual addend are the fp32 kernel's results rounded once, to within the tensor
    core's own fp32 summation order; the statistics are those of the stored output."""
    seed = seed_of("tc", str(dtype), k, shape)
    x = rand(shape, dtype, seed).cuda()
    w = rand((shape[1], 1, k, k, k), dtype, seed + 1, scale=1 / np.sqrt(k**3)).cuda()
    b = rand((shape[1],), dtype, seed + 2).cuda()
    a = rand(shape, dtype, seed + 3).cuda()
    y, stats = dwk.dw_forward(x, w, b, k, gn_eps=1e-5)
    _assert_one_rounding(y, dwk.dw_forward(x.float(), w.float(), b.float(), k), "y")
    dx = dwk.dw_dgrad(x, w, k, addend=a)
    _assert_one_rounding(dx, dwk.dw_dgrad(x.float(), w.float(), k, addend=a.float()), "dx")
    y0 = dwk.dw_forward(x, w, None, k)
    _assert_one_rounding(y0, dwk.dw_forward(x.float(), w.float(), None, k), "y without bias")
    yf = y.double().reshape(shape[0] * shape[1], -1)
    torch.testing.assert_close(stats[:, 0].double(), yf.mean(1), rtol=1e-5, atol=1e-6)
    rstd = 1 / torch.sqrt(yf.var(1, unbiased=False) + 1e-5)
    torch.testing.assert_close(stats[:, 1].double(), rstd, rtol=1e-5, atol=1e-6)
    assert nat.device_error() == 0


DOWN_SHAPES = [
    (1, 32, 128, 128, 128),  # the benchmark's first down block
    (2, 3, 16, 20, 32),      # ragged last row tile of the small grid
    (1, 2, 9, 6, 16),        # odd depth: the last input plane is padding
    (1, 4, 8, 40, 256),      # two 64-wide tiles along W
    (1, 2, 4, 4, 16),        # a single output plane pair
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", DOWN_SHAPES)
def test_stride2_forward_tma_kernel_is_bit_exact_with_fp32_kernel(dtype, shape):
    """The down block's forward (k = 3, 16-bit) runs on the TMA plane ring with
    packed FMAs and sums bias, then taps in (kd, kh, kw) order, as the fp32 gather
    does: its outputs are the fp32 kernel's outputs on the same inputs, rounded once."""
    seed = seed_of("down", str(dtype), shape)
    x = rand(shape, dtype, seed).cuda()
    w = rand((shape[1], 1, 3, 3, 3), dtype, seed + 1, scale=0.2).cuda()
    b = rand((shape[1],), dtype, seed + 2).cuda()
    y = dwk.s2_forward(x, w, b, 3)
    assert torch.equal(y, dwk.s2_forward(x.float(), w.float(), b.float(), 3).to(dtype))
    assert nat.device_error() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", DOWN_SHAPES)
def test_stride2_weight_grad_tma_kernel_matches_fp32_kernel(dtype, shape):
    """The down block's weight grad (k = 3, 16-bit) runs on the TMA plane ring with
    packed FMAs; it sums in its own fixed order, so it matches the fp32 kernel on
    the same inputs to the output's rounding (one 16-bit ulp), and repeats exactly."""
    seed = seed_of("down-wgrad", str(dtype), shape)
    x = rand(shape, dtype, seed).cuda()
    small = (shape[0], shape[1], *((s + 1) // 2 for s in shape[2:]))
    dy = rand(small, dtype, seed + 1).cuda()
    dw, db = dwk.s2_wgrad(x, dy, 3)
    dw32, db32 = dwk.s2_wgrad(x.float(), dy.float(), 3)
    for got, want in ((dw, dw32), (db, db32)):
        scale = want.abs().max().item()
        torch.testing.assert_close(got.float(), want, rtol=2.0**-7, atol=1e-4 * scale)
    dw2, db2 = dwk.s2_wgrad(x, dy, 3)
    assert torch.equal(dw, dw2) and torch.equal(db, db2)
    assert nat.device_error() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", DOWN_SHAPES)
def test_stride2_input_grad_tma_kernel_is_bit_exact_with_fp32_kernel(dtype, shape):
    """The down block's input grad (k = 3, 16-bit) scatters small-grid planes from the
    TMA ring with packed FMAs, summing bias, taps in (a_d, a_h, a_w) order and the
    even-position addend last, as the fp32 scatter does: equal after one rounding."""
    seed = seed_of("down-dgrad", str(dtype), shape)
    small = (shape[0], shape[1], *((s + 1) // 2 for s in shape[2:]))
    dy = rand(small, dtype, seed).cuda()
    w = rand((shape[1], 1, 3, 3, 3), dtype, seed + 1, scale=0.2).cuda()
    a = rand(small, dtype, seed + 2).cuda()
    spatial = tuple(shape[2:])
    for addend in (None, a):
        dx = dwk.s2_dgrad(dy, w, spatial, 3, addend_even=addend)
        want = dwk.s2_dgrad(dy.float(), w.float(), spatial, 3,
                            addend_even=None if addend is None else addend.float())
        assert torch.equal(dx, want.to(dtype))
    assert nat.device_error() == 0


# Up-block grids: small (d, h, w) inputs of the transposed conv; the fused up
# block stores its (2d-1, 2h-1, 2w-1) tensors with W-rows padded to a multiple of 8.
UP_SHAPES = [
    (1, 64, 64, 64, 64),     # the benchmark's level-0 up block (C64 64^3 -> 127^3)
    (2, 3, 8, 10, 16),       # ragged row tile, two samples
    (1, 4, 5, 7, 8),         # odd small depth and height
    (1, 2, 4, 4, 128),       # two 64-wide tiles along W
    (1, 3, 6, 6, 12),        # small W not a multiple of 8: packed-FMA path declines
]


def _pitched(t: torch.Tensor, pitch: int, fill: float) -> torch.Tensor:
    """t [n, c, D, H, W] copied into [n, c, D, H, pitch] with `fill` in the pad columns."""
    out = torch.full((*t.shape[:4], pitch), fill, dtype=t.dtype, device=t.device)
    out[..., : t.shape[4]] = t
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", UP_SHAPES)
def test_up_block_row_pitched_kernels_match_the_packed_fp32_kernels(dtype, shape):
    """The transposed conv on the row-pitched layout of the fused up block: forward
    and input grad (k = 3, 16-bit, TMA plane ring with packed FMAs where the rows are
    2w elements apart) give the fp32 kernels' results on packed grids rounded once;
    the forward writes zeros into the pad columns; input and weight grads ignore
    whatever the pad columns of dy hold; the weight grad matches the fp32 kernel to
    the output's rounding and repeats exactly."""
    seed = seed_of("up-rows", str(dtype), shape)
    n, c, d, h, w = shape
    big = (n, c, 2 * d - 1, 2 * h - 1, 2 * w - 1)
    pitch = (2 * w - 1 + 7) // 8 * 8
    xs = rand(shape, dtype, seed).cuda()
    wt = rand((c, 1, 3, 3, 3), dtype, seed + 1, scale=0.2).cuda()
    b = rand((c,), dtype, seed + 2).cuda()
    y = dwk.t_forward(xs, wt, b, 3, row_pitch=pitch)
    assert tuple(y.shape) == (*big[:4], pitch)
    want = dwk.t_forward(xs.float(), wt.float(), b.float(), 3).to(dtype)
    assert torch.equal(dwk.pitched_view(y, big[2:]), want)
    assert torch.all(y[..., big[4]:] == 0)
    # with the GroupNorm statistics of the output (fused into the packed kernel)
    from mednext_accel_b200.pointwise import gn_stats

    y2, st = dwk.t_forward_stats(xs, wt, b, 3, 1e-5, row_pitch=pitch)
    assert torch.equal(y2, y)
    torch.testing.assert_close(st, gn_stats(y, 1e-5, row_len=big[4]), rtol=1e-5, atol=1e-6)
    dy = rand(big, dtype, seed + 3).cuda()
    dyp = _pitched(dy, pitch, 1000.0)
    add = rand(shape, dtype, seed + 4).cuda()
    for addend in (None, add):
        dx = dwk.t_dgrad(dyp, wt, 3, small=(d, h, w), addend=addend)
        want = dwk.t_dgrad(dy.float(), wt.float(), 3, addend=None if addend is None else addend.float())
        assert torch.equal(dx, want.to(dtype))
    dw, db = dwk.t_wgrad(xs, dyp, 3)
    dw32, db32 = dwk.t_wgrad(xs.float(), dy.float(), 3)
    for got, want in ((dw, dw32), (db, db32)):
        scale = want.abs().max().item()
        torch.testing.assert_close(got.float(), want, rtol=2.0**-7, atol=1e-4 * scale)
    dw2, db2 = dwk.t_wgrad(xs, dyp, 3)
    assert torch.equal(dw, dw2) and torch.equal(db, db2)
    assert nat.device_error() == 0


@pytest.mark.parametrize("shape,pitch", [((1, 64, 127, 127, 127), 128), ((2, 3, 15, 19, 31), 32),
                                         ((1, 5, 7, 9, 11), 16)])
def test_groupnorm_statistics_of_row_pitched_grid(shape, pitch):
    """gn_stats over the valid columns of a row-pitched grid whose pad columns hold
    large values: the statistics of the packed grid (fp64 reference, 1e-5)."""
    from mednext_accel_b200.pointwise import gn_stats

    seed = seed_of("gn-rows", shape)
    t = (rand(shape, torch.float32, seed) * 3 + 0.5).to(torch.bfloat16).cuda()
    st = gn_stats(_pitched(t, pitch, 500.0), 1e-5, row_len=shape[4]).cpu().double()
    flat = t.double().reshape(shape[0] * shape[1], -1)
    mean = flat.mean(dim=1).cpu()
    rstd = (1.0 / torch.sqrt(flat.var(dim=1, unbiased=False) + 1e-5)).cpu()
    torch.testing.assert_close(st[:, 0], mean, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(st[:, 1], rstd, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_weight_grads_with_fp32_output_equal_the_cast_of_the_16bit_ones(dtype):
    """The _f32out weight-grad entry points write what casting the 16-bit result to fp32
    gives (stride 1, stride 2 on aligned and unaligned grids, transposed)."""
    gen_seed = seed_of("f32out", str(dtype))
    for shape in ((1, 4, 8, 16, 16), (2, 3, 5, 6, 7), (1, 32, 32, 32, 32)):
        x = rand(shape, dtype, gen_seed).cuda()
        dy = rand(shape, dtype, gen_seed + 1).cuda()
        small = (shape[0], shape[1], *((s + 1) // 2 for s in shape[2:]))
        dys = rand(small, dtype, gen_seed + 2).cuda()
        big_t = (shape[0], shape[1], *(2 * s - 1 for s in small[2:]))
        dyt = rand(big_t, dtype, gen_seed + 3).cuda()
        xs = rand(small, dtype, gen_seed + 4).cuda()
        cases = (
            (dwk.dw_wgrad, (x, dy, 3)),
            (dwk.s2_wgrad, (x, dys, 3)),
            (dwk.t_wgrad, (xs, dyt, 3)),
        )
        for fn, args in cases:
            dw16, db16 = fn(*args)
            dw32, db32 = fn(*args, out_dtype=torch.float32)
            assert dw32.dtype == torch.float32 and db32.dtype == torch.float32
            assert torch.equal(dw32, dw16.float()), fn.__name__
            assert torch.equal(db32, db16.float()), fn.__name__
    assert nat.device_error() == 0


def test_dgrad_with_addend_adds_residual():
    x = rand((1, 4, 8, 16, 16), torch.bfloat16, 8).cuda()
    w = rand((4, 1, 3, 3, 3), torch.bfloat16, 9).cuda()
    r = rand((1, 4, 8, 16, 16), torch.bfloat16, 10).cuda()
    plain = dwk.dw_dgrad(x, w, 3).float()
    fused = dwk.dw_dgrad(x, w, 3, addend=r).float()
    torch.testing.assert_close(fused, plain + r.float(), rtol=1e-2, atol=2e-2)


def test_gn_statistics_fused_into_forward():
    x = rand((2, 4, 16, 16, 16), torch.bfloat16, 11).cuda()
    w = rand((4, 1, 3, 3, 3), torch.bfloat16, 12).cuda()
    y, stats = dwk.dw_forward(x, w, None, 3, gn_eps=1e-5)
    yf = y.double().reshape(8, -1)
    mean = yf.mean(1)
    rstd = 1 / torch.sqrt(yf.var(1, unbiased=False) + 1e-5)
    torch.testing.assert_close(stats[:, 0].double(), mean, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(stats[:, 1].double(), rstd, rtol=1e-5, atol=1e-6)


def test_low_level_errors_match_reference():
    x = torch.randn(1, 2, 4, 4, 4)
    w = torch.randn(2, 1, 3, 3, 3)
    with pytest.raises(ValueError, match="CUDA"):
        dwk.depthwise_input_grad(x, w)
    with pytest.raises(ValueError, match="power of two"):
        dwk.depthwise_input_grad(x.cuda(), w.cuda(), block=100)
    with pytest.raises(ValueError, match="odd"):
        dwk.depthwise_weight_grad(x.cuda(), x.cuda(), kernel_size=4)
    with pytest.raises(ValueError, match="contiguous"):
        dwk.depthwise_input_grad(x.cuda().transpose(2, 3), w.cuda())


def test_no_device_error_recorded():
    assert nat.device_error() == 0

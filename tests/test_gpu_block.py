"""Fused MedNeXt block and full model on the GPU against the CPU oracle / the
reference's pure-PyTorch path.  bf16 autocast bar: relative L2 <= 2e-2."""

from __future__ import annotations

import copy
import zlib

import numpy as np
import pytest
import torch
from torch.nn import functional as F
from torch.utils._python_dispatch import TorchDispatchMode

import mednext_accel_b200 as mx
from mednext_accel_b200 import _native as nat
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
BAR = 2e-2


class OpSpy(TorchDispatchMode):
    def __init__(self):
        super().__init__()
        self.ops = []

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        self.ops.append(func._schema.name)
        return func(*args, **(kwargs or {}))


def _seed(*key):
    return zlib.crc32(repr(key).encode()) % 100_000


def make_block(kind, cin, cout, ratio, k, seed, checkpoint_expansion=False):
    torch.manual_seed(seed)
    cls = {"regular": mx.MedNeXtBlock, "down": mx.MedNeXtDownBlock, "up": mx.MedNeXtUpBlock}[kind]
    block = cls(spatial_dims=3, in_channels=cin, out_channels=cout, expansion_ratio=ratio, kernel_size=k,
                checkpoint_expansion=checkpoint_expansion)
    with torch.no_grad():
        block.norm.weight.copy_(1.0 + 0.1 * torch.randn_like(block.norm.weight))
        block.norm.bias.copy_(0.1 * torch.randn_like(block.norm.bias))
    return block


def install(module):
    from mednext_accel_b200.adaptive import ModelOptimizationContext

    mx.install_adaptive_operators(module, resolver=mx.PolicyResolver(),
                                  model_context=ModelOptimizationContext("mednext_v1", "base", "none"))
    return module


def run_fused(block, x, dy):
    block = install(copy.deepcopy(block)).cuda().train()
    xg = x.cuda().requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16), OpSpy() as spy:
        y = block(xg)
    grads = torch.autograd.grad(y, (xg, *block.parameters()), dy.cuda().to(y.dtype))
    assert "mednext_accel_b200::mednext_block" in spy.ops
    names = [n for n, _ in block.named_parameters()]
    return y, dict(zip(["dx", *names], grads, strict=True))


def oracle_block(block, x, dy, kind):
    state = {k: v.detach().double().numpy() for k, v in block.state_dict().items()}
    p = orc.BlockParams.from_state(state)
    xn = x.double().numpy()
    addend = None
    if kind == "down":
        xb = orc.round_bf16(xn)
        addend = orc.round_bf16(orc.pointwise_fwd(xb[:, :, ::2, ::2, ::2], orc.round_bf16(state["residual.weight"]),
                                                  orc.round_bf16(state["residual.bias"])))
    elif kind == "up":
        xb = orc.round_bf16(xn)
        n, c, d, h, w = xn.shape
        up = np.zeros((n, c, 2 * d - 1, 2 * h - 1, 2 * w - 1))
        up[:, :, ::2, ::2, ::2] = xb
        rw = orc.round_bf16(state["residual.weight"])
        addend = orc.round_bf16(orc.pointwise_fwd(up, np.transpose(rw, (1, 0, 2, 3, 4)), None)
                                + orc.round_bf16(state["residual.bias"]).reshape(1, -1, 1, 1, 1))
    dyn = dy.double().numpy()
    if kind == "up":
        dyn = dyn[:, :, 1:, 1:, 1:]
    return orc.block_reference(xn, dyn, p, kind, addend=addend, residual_is_input=(kind == "regular"))


CASES = [
    ("regular", 32, 32, 2, 3, (2, 32, 16, 16, 16)),
    ("regular", 16, 16, 4, 5, (1, 16, 12, 12, 12)),
    ("regular", 64, 64, 3, 3, (1, 64, 8, 8, 8)),
    ("regular", 8, 8, 2, 7, (1, 8, 9, 10, 11)),
    ("down", 16, 32, 3, 3, (1, 16, 16, 16, 16)),
    ("up", 32, 16, 2, 3, (1, 32, 8, 8, 8)),
]


@pytest.mark.parametrize("kind,cin,cout,ratio,k,shape", CASES)
def test_fused_block_matches_oracle(kind, cin, cout, ratio, k, shape):
    seed = _seed(kind, cin, k, shape)
    block = make_block(kind, cin, cout, ratio, k, seed)
    gen = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(shape, generator=gen).to(torch.bfloat16)
    ref = block.train()
    out_shape = ref(x.float()).shape if kind != "up" else None
    if kind == "up":
        out_shape = (shape[0], cout, *(2 * s for s in shape[2:]))
    dy = torch.randn(out_shape, generator=gen).to(torch.bfloat16)
    y, grads = run_fused(block, x, dy)
    want_y, want = oracle_block(block, x, dy, kind)
    got_y = y.detach().double().cpu().numpy()
    if kind == "up":
        assert torch.count_nonzero(y[:, :, 0]) == 0
        got_y = got_y[:, :, 1:, 1:, 1:]
    assert orc.rel_l2(got_y, want_y) <= BAR, orc.rel_l2(got_y, want_y)
    if kind == "regular":
        assert orc.rel_l2(grads["dx"].double().cpu().numpy(), want["dx"]) <= BAR
    for name in ("depthwise.weight", "norm.weight", "norm.bias", "expand.weight", "expand.bias",
                 "project.weight", "project.bias"):
        got = grads[name].double().cpu().numpy()
        err = orc.rel_l2(got, want[name])
        assert err <= BAR, f"{name}: {err:.3e}"
    # the depthwise bias grad is sum(dt), analytically zero under GroupNorm(C, C)
    got = grads["depthwise.bias"].double().cpu().numpy()
    assert np.all(np.abs(got - want["depthwise.bias"]) <= BAR * want["depthwise.bias_scale"])
    if kind in ("down", "up"):
        # the strided 1x1 residual convolution runs inside the fused operator
        xb = orc.round_bf16(x.double().numpy())
        dyn = dy.double().numpy()
        if kind == "down":
            # out[m] = W x[2m] + b: dW = sum dy (x) x_even, db = sum dy
            _, want_rw, want_rb = orc.pointwise_bwd(dyn, np.ascontiguousarray(xb[:, :, ::2, ::2, ::2]),
                                                    block.residual.weight.detach().double().numpy()[:, :, 0, 0, 0])
        else:
            # out[2m] = W^T x[m] + b on the (2S-1)^3 interior of the left-padded output
            inner = dyn[:, :, 1:, 1:, 1:]
            want_rw = np.einsum("ncdhw,nkdhw->ck", xb, inner[:, :, ::2, ::2, ::2])
            want_rb = inner.sum(axis=(0, 2, 3, 4))
        got_rw = grads["residual.weight"].double().cpu().numpy().reshape(want_rw.shape)
        assert orc.rel_l2(got_rw, want_rw) <= BAR, orc.rel_l2(got_rw, want_rw)
        assert orc.rel_l2(grads["residual.bias"].double().cpu().numpy(), want_rb) <= BAR


def test_checkpointed_expansion_matches_stored():
    block = make_block("regular", 32, 32, 4, 3, 7)
    gen = torch.Generator().manual_seed(8)
    x = torch.randn((1, 32, 16, 16, 16), generator=gen).to(torch.bfloat16)
    dy = torch.randn((1, 32, 16, 16, 16), generator=gen).to(torch.bfloat16)
    y1, g1 = run_fused(block, x, dy)
    block_ck = copy.deepcopy(block)
    block_ck.checkpoint_expansion = True
    y2, g2 = run_fused(block_ck, x, dy)
    torch.testing.assert_close(y1, y2, rtol=0, atol=0)
    for k in g1:
        torch.testing.assert_close(g1[k], g2[k], rtol=0, atol=0)


def test_config2_block_full_size_against_reference_path():
    """The standalone-block workload: MedNeXtBlock N=2, C=64, 64^3, R=4, k=5 under bf16
    autocast, PyTorch default init from seed 0, input and upstream grad ~N(0,1).
    Compared with the same block run through the reference's pure-PyTorch path
    (native modules) in fp32 on the same GPU."""
    torch.manual_seed(0)
    block = mx.MedNeXtBlock(spatial_dims=3, in_channels=64, out_channels=64, expansion_ratio=4, kernel_size=5)
    x = torch.randn(2, 64, 64, 64, 64)
    dy = torch.randn(2, 64, 64, 64, 64)
    ref = copy.deepcopy(block).cuda().train()
    xr = x.cuda().requires_grad_()
    yr = ref(xr)
    gr = torch.autograd.grad(yr, (xr, *ref.parameters()), dy.cuda())
    y, grads = run_fused(block, x, dy)
    assert y.dtype == torch.float32  # residual add promotes to the fp32 input, as in the reference
    assert orc.rel_l2(y.detach().double().cpu().numpy(), yr.detach().double().cpu().numpy()) <= BAR
    names = ["dx", *[n for n, _ in block.named_parameters()]]
    for name, want in zip(names, gr, strict=True):
        if name == "depthwise.bias":
            # analytically zero under GroupNorm(C, C): both sides are rounding noise
            # summed over 2*64^3 voxels; the small-block tests check it against the
            # oracle at the scale sum|dt|
            continue
        err = orc.rel_l2(grads[name].double().cpu().numpy(), want.double().cpu().numpy())
        assert err <= BAR, f"{name}: {err:.3e}"


def _loss(heads, target):
    if isinstance(heads, torch.Tensor):
        heads = (heads,)
    total = 0
    for hd in heads:
        t = target if hd.shape[2:] == target.shape[1:] else F.interpolate(
            target[:, None].float(), size=hd.shape[2:], mode="nearest")[:, 0].long()
        total = total + F.cross_entropy(hd.float(), t)
    return total / len(heads)


def test_small_model_step_matches_native_path():
    torch.manual_seed(0)
    fused = mx.mednext_small(in_channels=1, out_channels=3, base_channels=16, deep_supervision=True).cuda().train()
    native = mx.mednext_small(in_channels=1, out_channels=3, base_channels=16, deep_supervision=True,
                              optimization="reference").cuda().train()
    native.load_state_dict(fused.state_dict())
    gen = torch.Generator().manual_seed(1)
    x = torch.randn((2, 1, 64, 64, 64), generator=gen).cuda()
    target = torch.randint(0, 3, (2, 64, 64, 64), generator=gen).cuda()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        lf = _loss(fused(x), target)
        ln = _loss(native(x), target)
    lf.backward()
    ln.backward()
    assert abs(lf.item() - ln.item()) <= 1e-2 * abs(ln.item())
    worst = 0.0
    for (name, pf), (_, pn) in zip(fused.named_parameters(), native.named_parameters(), strict=True):
        if name.endswith("depthwise.bias") and "residual" not in name:
            continue  # analytically zero under GroupNorm(C, C)
        err = orc.rel_l2(pf.grad.double().cpu().numpy(), pn.grad.double().cpu().numpy())
        worst = max(worst, err)
        assert err <= 5e-2, f"{name}: {err:.3e}"


def test_loss_curve_matches_native_path_over_adamw_steps():
    """Per-step loss within 1% of the reference's pure-PyTorch path over AdamW steps."""
    torch.manual_seed(0)
    fused = mx.mednext_small(in_channels=1, out_channels=3, base_channels=8, deep_supervision=True).cuda().train()
    native = mx.mednext_small(in_channels=1, out_channels=3, base_channels=8, deep_supervision=True,
                              optimization="reference").cuda().train()
    native.load_state_dict(fused.state_dict())
    opt_f = torch.optim.AdamW(fused.parameters(), lr=1e-4)
    opt_n = torch.optim.AdamW(native.parameters(), lr=1e-4)
    gen = torch.Generator().manual_seed(2)
    x = torch.randn((1, 1, 64, 64, 64), generator=gen).cuda()
    target = torch.randint(0, 3, (1, 64, 64, 64), generator=gen).cuda()
    for _ in range(50):
        losses = []
        for model, opt in ((fused, opt_f), (native, opt_n)):
            opt.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = _loss(model(x), target)
            loss.backward()
            opt.step()
            losses.append(loss.item())
        assert abs(losses[0] - losses[1]) <= 1e-2 * abs(losses[1]), losses


@pytest.mark.parametrize("spatial,pitch", [((7, 9, 11), 0), ((7, 9, 11), 16), ((15, 15, 15), 16),
                                           ((127, 127, 127), 128), ((63, 63, 63), 64)])
@pytest.mark.parametrize("with_addend", [False, True])
def test_pad_front_and_unpad_match_torch(spatial, pitch, with_addend):
    """pad_front_add / unpad_front on packed and row-pitched grids (the 16-byte
    shifted-copy path when the pitch is the padded row length) equal torch's pad,
    add and slice exactly; unpad writes zeros into the pad columns."""
    from mednext_accel_b200 import depthwise as dwk

    n, c = 2, 3
    rp = pitch or spatial[2]
    gen = torch.Generator().manual_seed(_seed("pad", spatial, pitch))
    v = torch.randn((n, c, spatial[0], spatial[1], rp), generator=gen).to(torch.bfloat16).cuda()
    padded_shape = (n, c, *(s + 1 for s in spatial))
    addend = torch.randn(padded_shape, generator=gen).to(torch.bfloat16).cuda() if with_addend else None
    got = dwk.pad_front_add(v, spatial, addend)
    want = F.pad(dwk.pitched_view(v, spatial), (1, 0) * 3)
    if addend is not None:
        want = want + addend
    assert torch.equal(got, want)
    back = dwk.unpad_front(got if addend is None else want, pitch)
    want_back = torch.zeros_like(v)
    dwk.pitched_view(want_back, spatial).copy_((want)[:, :, 1:, 1:, 1:])
    assert torch.equal(back, want_back)


@pytest.mark.parametrize("small,pitch", [((8, 8, 8), 16), ((64, 64, 64), 128), ((3, 5, 6), 0), ((4, 4, 12), 24)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_upsample2_fill_matches_torch(small, pitch, with_bias):
    """upsample2_fill: small[m] at the all-even big positions 2m, the bias elsewhere, zeros
    in the pad columns, on packed and row-pitched big grids (the 16-byte path where the
    pitch is 2w)."""
    from mednext_accel_b200 import depthwise as dwk

    n, c = 2, 3
    gen = torch.Generator().manual_seed(_seed("upsample", small, pitch))
    s = torch.randn((n, c, *small), generator=gen).to(torch.bfloat16).cuda()
    b = torch.randn((c,), generator=gen).cuda() if with_bias else None
    got = dwk.upsample2_fill(s, b, pitch)
    big = tuple(2 * v - 1 for v in small)
    fill = b.to(torch.bfloat16) if b is not None else torch.zeros(c, dtype=torch.bfloat16, device="cuda")
    want = fill.view(1, c, 1, 1, 1).expand(n, c, *big).clone()
    want[:, :, ::2, ::2, ::2] = s
    assert torch.equal(dwk.pitched_view(got, big), want)
    assert torch.all(got[..., big[2]:] == 0)


def test_up_block_skip_addend_is_fused_exactly():
    """block(x, addend=skip) == block(x) + skip, and the skip's grad is dy."""
    block = make_block("up", 32, 16, 2, 3, 7)
    gen = torch.Generator().manual_seed(8)
    x = torch.randn((1, 32, 8, 8, 8), generator=gen).to(torch.bfloat16)
    skip = torch.randn((1, 16, 16, 16, 16), generator=gen).to(torch.bfloat16).cuda()
    dy = torch.randn((1, 16, 16, 16, 16), generator=gen).to(torch.bfloat16).cuda()
    blk = install(copy.deepcopy(block)).cuda().train()
    xg = x.cuda().requires_grad_()
    sg = skip.clone().requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16), OpSpy() as spy:
        y1 = blk(xg, sg)
        y0 = blk(xg)
    assert spy.ops.count("mednext_accel_b200::mednext_block") == 2
    assert torch.equal(y1, y0 + skip)
    g1 = torch.autograd.grad(y1, (xg, sg, *blk.parameters()), dy)
    g0 = torch.autograd.grad(y0, (xg, *blk.parameters()), dy)
    assert torch.equal(g1[1], dy)
    for a, b in zip((g1[0], *g1[2:]), g0, strict=True):
        assert torch.equal(a, b)


@pytest.mark.parametrize("c,rc,cout", [(32, 64, 32), (17, 51, 33), (512, 2048, 512)])
def test_parameter_casts_are_exact(c, rc, cout):
    """One mednext_cast_params launch gives exactly torch's casts, plain and transposed."""
    from mednext_accel_b200.block import _block_params

    gen = torch.Generator().manual_seed(_seed("cast", c, rc))
    dw_w = torch.randn((c, 1, 3, 3, 3), generator=gen).cuda()
    dw_b = torch.randn((c,), generator=gen).cuda()
    e_w = torch.randn((rc, c, 1, 1, 1), generator=gen).cuda()
    e_b = torch.randn((rc,), generator=gen).cuda()
    p_w = torch.randn((cout, rc, 1, 1, 1), generator=gen).cuda()
    p_b = torch.randn((cout,), generator=gen).cuda()
    bf = torch.bfloat16
    prm = _block_params(dw_w, dw_b, e_w, e_b, p_w, p_b, bf, transposed=True)
    torch.cuda.synchronize()
    assert torch.equal(prm.wdw, dw_w.to(bf))
    assert torch.equal(prm.bdw.reshape(-1), dw_b.to(bf))
    assert torch.equal(prm.ew, e_w.reshape(rc, c).to(bf))
    assert torch.equal(prm.pw, p_w.reshape(cout, rc).to(bf))
    assert torch.equal(prm.ewt, e_w.reshape(rc, c).t().contiguous().to(bf))
    assert torch.equal(prm.pwt, p_w.reshape(cout, rc).t().contiguous().to(bf))
    assert torch.equal(prm.eb, e_b.to(bf).float())
    assert torch.equal(prm.pb, p_b.to(bf).float())


def test_no_device_error_recorded():
    assert nat.device_error() == 0

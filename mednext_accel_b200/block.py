"""Fused MedNeXt block: one autograd node per block on sm_100a.

Computes, for ``kind`` in {regular, down, up} (reference models/blocks.py:47-182):

    t = depthwise(x)                      regular: stride 1; down: stride 2; up: transposed stride 2
    z = GroupNorm(C, C)(t)                never materialised: applied while staging the expand GEMM
    u = expand(z)                         tcgen05 GEMM, bias in the epilogue
    y = project(gelu(u)) + addend         tcgen05 GEMM, GELU in the prologue, bias + residual in the epilogue

Backward recomputes nothing but ``u`` when expansion checkpointing is on, and
never materialises gelu(u), z or the GroupNorm-input gradient's intermediates:

    du   = (dy Wp) * gelu'(u)             dgrad GEMM with the GELU derivative in the epilogue
    dWp  = sum dy (x) gelu(u)             wgrad GEMM, GELU in the prologue
    dWe  = sum du (x) z                   wgrad GEMM, GroupNorm in the prologue
    dz   = du We                          dgrad GEMM + per-tile GroupNorm-backward sums in the epilogue
    dt   = GroupNorm backward(dz)         one elementwise pass
    dx   = depthwise dgrad(dt) (+ dy)     residual added in the same kernel
    dWdw = depthwise wgrad(x, dt)         bias grad in the same pass

Precision follows the reference under CUDA autocast: the depthwise conv and both
GEMMs take bfloat16 (or float16) operands with fp32 accumulation, GroupNorm
statistics and normalisation are fp32, outputs of each stage are rounded to the
compute dtype where the reference stores them in that dtype.
"""

from __future__ import annotations

import torch
from torch import Tensor
from torch.library import custom_op
from torch.nn import functional as F

from . import _native as nat
from . import depthwise as dwk
from .pointwise import (gelu_bwd_fused_covers, gn_backward_from_partials, gn_stats, pw_gelu_bwd, pw_gemm,
                        pw_gemm_gelu_out, pw_gn_bwd_fused, pw_wgrad)

_NS = "mednext_accel_b200"
KIND_REGULAR, KIND_DOWN, KIND_UP = 0, 1, 2
_CODES = {0: torch.float32, 1: torch.bfloat16, 2: torch.float16}


class _Params:
    """Compute-dtype copies of one block's parameters: depthwise weight and bias,
    expand / project GEMM weights ([out, in]) and their biases rounded to the
    compute dtype but kept fp32 for the epilogue, plus, for the backward, the
    transposed GEMM weights of the input-grad GEMMs."""

    __slots__ = ("wdw", "bdw", "ew", "eb", "pw", "pb", "ewt", "pwt", "rw", "rb")


def _block_params(dw_w: Tensor, dw_b: Tensor | None, e_w: Tensor, e_b: Tensor, p_w: Tensor, p_b: Tensor | None,
                  cdt, *, transposed: bool, res: tuple[Tensor, bool] | None = None,
                  res_b: Tensor | None = None) -> _Params:
    """All casts of a block in one ``mednext_cast_params`` launch (fp32 parameters),
    else per-tensor casts.  Every GEMM weight starts on a 128-byte boundary, as the
    TMA paths require.  ``dw_b`` / ``p_b`` may be None (the backward needs neither).
    ``res`` = (residual conv weight, transpose): its [rows, cols] matrix is cast to
    ``rw`` as is or transposed; ``res_b`` becomes ``rb`` (rounded, fp32)."""
    rc, c = int(e_w.shape[0]), int(e_w.shape[1])
    cout = int(p_w.shape[0])
    out = _Params()
    out.rw = out.rb = None
    params = [t for t in (dw_w, dw_b, e_w, e_b, p_w, p_b, res_b, res[0] if res else None) if t is not None]
    if not all(t.dtype == torch.float32 and t.is_contiguous() for t in params) or cdt == torch.float32:
        if res is not None:
            r2 = res[0].reshape(res[0].shape[0], res[0].shape[1])
            out.rw = (r2.t() if res[1] else r2).to(cdt).contiguous()
        if res_b is not None:
            out.rb = res_b.to(cdt).float()
        out.wdw = dw_w.to(cdt).contiguous()
        out.bdw = dw_b.to(cdt) if dw_b is not None else None
        out.ew, out.eb = e_w.reshape(rc, c).to(cdt).contiguous(), e_b.to(cdt).float()
        out.pw = p_w.reshape(cout, rc).to(cdt).contiguous()
        out.pb = p_b.to(cdt).float() if p_b is not None else None
        out.ewt = out.ew.t().contiguous() if transposed else None
        out.pwt = out.pw.t().contiguous() if transposed else None
        return out
    code = nat.dtype_code(cdt)
    f32 = nat.dtype_code(torch.float32)
    # (name, src, rows, cols, transpose) in the compute dtype; offsets on 64-element boundaries
    half = [("wdw", dw_w, c, dw_w[0].numel(), 0), ("ew", e_w, rc, c, 0), ("pw", p_w, cout, rc, 0)]
    if res is not None:
        half.append(("rw", res[0], int(res[0].shape[0]), int(res[0].shape[1]), int(res[1])))
    if dw_b is not None:
        half.append(("bdw", dw_b, 1, c, 0))
    if transposed:
        half += [("ewt", e_w, rc, c, 1), ("pwt", p_w, cout, rc, 1)]
    offs, total = [], 0
    for _, _, r, k, _ in half:
        offs.append(total)
        total += (r * k + 63) // 64 * 64
    buf = torch.empty(total, dtype=cdt, device=dw_w.device)
    nrb = int(res_b.numel()) if res_b is not None else 0
    fbuf = torch.empty(rc + cout + nrb, dtype=torch.float32, device=dw_w.device)
    out.bdw = out.pb = None
    entries = []
    for (name, src, r, k, tr), off in zip(half, offs, strict=True):
        view = buf[off : off + r * k]
        setattr(out, name, view)
        entries.append(nat.CastEntry(src.data_ptr(), view.data_ptr(), r, k, code, f32, tr))
    out.eb = fbuf[:rc]
    entries.append(nat.CastEntry(e_b.data_ptr(), out.eb.data_ptr(), 1, rc, f32, code, 0))
    if p_b is not None:
        out.pb = fbuf[rc : rc + cout]
        entries.append(nat.CastEntry(p_b.data_ptr(), out.pb.data_ptr(), 1, cout, f32, code, 0))
    if res_b is not None:
        out.rb = fbuf[rc + cout :]
        entries.append(nat.CastEntry(res_b.data_ptr(), out.rb.data_ptr(), 1, nrb, f32, code, 0))
    table = (nat.CastEntry * len(entries))(*entries)
    nat.check(nat.load().mednext_cast_params(table, len(entries), nat.stream()), "mednext_cast_params")
    out.wdw = out.wdw.view(dw_w.shape)
    out.ew, out.pw = out.ew.view(rc, c), out.pw.view(cout, rc)
    if res is not None:
        r0, r1 = int(res[0].shape[0]), int(res[0].shape[1])
        out.rw = out.rw.view((r1, r0) if res[1] else (r0, r1))
    if transposed:
        out.ewt, out.pwt = out.ewt.view(c, rc), out.pwt.view(rc, cout)
    else:
        out.ewt = out.pwt = None
    return out


# The block backward runs its weight grads on a side stream beside the input-grad
# chain (both orders give the same bits).  The deep levels gain most, where each
# kernel leaves most SMs idle; at every level it measured no slower (Base k3 step:
# 15.16 ms without, 14.62 ms at 32^3 and below, 14.55 ms at every level).
_SIDE_STREAMS: dict[int, torch.cuda.Stream] = {}


class _Branch:
    """Launches on a side stream forked from the current one (when ``on``): each
    ``run`` waits for everything queued so far on the current stream, ``join``
    makes the current stream wait for the side stream and marks the side stream's
    outputs as used by the current stream (for the caching allocator).  The side
    stream is per device and lives as long as the process; CUDA-graph capture
    records the fork and the join."""

    def __init__(self, device: torch.device, on: bool) -> None:
        self.on = on
        if on:
            idx = device.index if device.index is not None else torch.cuda.current_device()
            self.main = torch.cuda.current_stream(device)
            side = _SIDE_STREAMS.get(idx)
            if side is None:
                side = _SIDE_STREAMS[idx] = torch.cuda.Stream(device=device)
            self.side = side

    def run(self, fn):
        if not self.on:
            return fn()
        self.side.wait_stream(self.main)
        with torch.cuda.stream(self.side):
            return fn()

    def join(self, *outs: Tensor | None) -> None:
        if not self.on:
            return
        self.main.wait_stream(self.side)
        for t in outs:
            if t is not None:
                t.record_stream(self.main)


def _even(x: Tensor) -> Tensor:
    """x at the all-even positions, contiguous: the input of a 1x1x1 stride-2 conv."""
    return x[:, :, ::2, ::2, ::2].contiguous()


def _row_pitch(spatial: tuple[int, ...]) -> tuple[int, int]:
    """(valid voxels, W-row pitch rounded up to 8 elements = 16 bytes of bf16) of the
    up block's (2S-1)^3 grid."""
    vox = 1
    for s in spatial:
        vox *= int(s)
    return vox, (int(spatial[-1]) + 7) // 8 * 8


def _depthwise_forward(xb: Tensor, w: Tensor, b: Tensor | None, kind: int, k: int, eps: float) -> tuple[Tensor, Tensor]:
    if kind == KIND_REGULAR:
        return dwk.dw_forward(xb, w, b, k, gn_eps=eps)
    t = dwk.s2_forward(xb, w, b, k) if kind == KIND_DOWN else dwk.t_forward(xb, w, b, k)
    return t, gn_stats(t, eps)


def _expansion(t: Tensor, stats: Tensor, gn_w: Tensor, gn_b: Tensor, prm: _Params, cdt, cout: int,
               res: Tensor | None) -> tuple[Tensor, Tensor, Tensor]:
    """(u, g, y): u = expand(GroupNorm(t)), y = project(GELU(u)) (+ res), and g =
    GELU(u) where the backward wants it stored (else an empty tensor).

    Where the backward's fused project kernel (``pw_gelu_bwd``) covers the block it
    recomputes GELU(u) from u on the fly, so the project GEMM applies GELU as its
    prologue and nothing more is stored.  Elsewhere the expand GEMM's epilogue
    writes g beside u: the project GEMM runs without a prologue (and, at the deep
    levels, on narrower N tiles) and the backward's project weight grad reads g.
    Both forms give the same bits.  (The one-kernel form, ``pointwise.pw_mlp_fwd``,
    gives the same bits too but measured slower at level 0: its two epilogue groups
    wait on the GELU pass between the GEMMs.)"""
    ydt = res.dtype if res is not None else cdt
    resc = res.contiguous() if res is not None else None
    ug = None
    if _stores_gelu(int(t.shape[0]), int(prm.pw.shape[0]), int(prm.ew.shape[0]), int(t[0, 0].numel()), cdt):
        ug = _expand_gelu(t, stats, gn_w, gn_b, prm)
    if ug is not None:
        u, g = ug
        y, _ = pw_gemm(g, prm.pw, cout, out_dtype=ydt, bias=prm.pb, residual=resc)
        return u, g, y
    u = _expand(t, stats, gn_w, gn_b, prm, cdt)
    y, _ = pw_gemm(u, prm.pw, cout, out_dtype=ydt, prologue=nat.PRO_GELU, bias=prm.pb, residual=resc)
    return u, u.new_empty((0,)), y


def _stores_gelu(n: int, cout: int, rc: int, vox: int, cdt) -> bool:
    """Whether a block stores g = GELU(u): where the fused project backward does not
    cover it and the GELU-output GEMM can produce g (bf16, 16-byte aligned rows)."""
    return cdt == torch.bfloat16 and vox % 8 == 0 and not gelu_bwd_fused_covers(n, cout, rc, vox, cdt)


def _expand_gelu(t: Tensor, stats: Tensor, gn_w: Tensor, gn_b: Tensor, prm: _Params) -> tuple[Tensor, Tensor] | None:
    rc = int(prm.ew.shape[0])
    return pw_gemm_gelu_out(t, prm.ew, rc, prologue=nat.PRO_GROUPNORM, pro_stats=stats,
                            pro_gamma=gn_w.float().contiguous(), pro_beta=gn_b.float().contiguous(), bias=prm.eb)


def _expand(t: Tensor, stats: Tensor, gn_w: Tensor, gn_b: Tensor, prm: _Params, cdt) -> Tensor:
    rc = int(prm.ew.shape[0])
    u, _ = pw_gemm(
        t, prm.ew, rc, out_dtype=cdt, prologue=nat.PRO_GROUPNORM, pro_stats=stats,
        pro_gamma=gn_w.float().contiguous(), pro_beta=gn_b.float().contiguous(), bias=prm.eb,
    )
    return u


@custom_op(f"{_NS}::mednext_block", mutates_args=())
def mednext_block(
    x: Tensor,
    addend: Tensor | None,
    dw_w: Tensor,
    dw_b: Tensor,
    gn_w: Tensor,
    gn_b: Tensor,
    e_w: Tensor,
    e_b: Tensor,
    p_w: Tensor,
    p_b: Tensor,
    res_w: Tensor | None,
    res_b: Tensor | None,
    kind: int,
    kernel_size: int,
    eps: float,
    residual_is_input: bool,
    keep_expansion: bool,
    compute_dtype: int,
) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Returns (y, t, u, g, stats); t, u and g = GELU(u) (both empty when not kept)
    and stats are saved for backward and carry no gradient.

    For the up block (kind 2) y is the final, left-padded (2S)^3 output of the
    reference's ``F.pad(block(x) + residual(x))`` and t, u are row-pitched
    [n, c, 2S-1, 2S-1, pitch] buffers whose W-rows hold 2S-1 voxels and pad
    columns up to a multiple of 8, so that every depthwise and GEMM operand has
    16-byte aligned rows for TMA (the GEMMs run over the pad columns too).  Its
    ``addend`` (the decoder's skip, models/mednext_v1.py:205) has the padded
    shape and is added after the pad, in the same pass.

    ``res_w`` / ``res_b`` (down and up blocks, instead of ``addend``): the 1x1x1
    stride-2 residual convolution (models/blocks.py:128-136, 173-182) computed here
    on the pointwise GEMM: the down block's reads x at the even positions, the up
    block's product on the small grid is expanded onto the big grid with the bias
    at the odd positions."""
    cdt = _CODES[compute_dtype]
    xb = x.to(cdt).contiguous()
    # the down block's residual weight is [cout, cin]; the transposed up block's is [cin, cout]
    rmode = (res_w, kind == KIND_UP) if res_w is not None else None
    prm = _block_params(dw_w, dw_b, e_w, e_b, p_w, p_b, cdt, transposed=False, res=rmode, res_b=res_b)
    wdw, bdw = prm.wdw, prm.bdw
    cout = int(p_w.shape[0])
    res = x if residual_is_input else addend
    if kind == KIND_UP:
        big = tuple(2 * int(s) - 1 for s in x.shape[2:])
        _, pitch = _row_pitch(big)
        t, stats = dwk.t_forward_stats(xb, wdw, bdw, kernel_size, eps, row_pitch=pitch)
        res_p = None
        if res_w is not None:
            rs, _ = pw_gemm(xb, prm.rw, cout, out_dtype=cdt, bias=prm.rb)
            res_p = dwk.upsample2_fill(rs, prm.rb, pitch)
        u, g, y_p = _expansion(t, stats, gn_w, gn_b, prm, cdt, cout, res_p)
        if addend is not None and addend.dtype != cdt:
            y = F.pad(dwk.pitched_view(y_p, big), (1, 0) * 3) + addend
        else:
            y = dwk.pad_front_add(y_p, big, addend)
        if not keep_expansion:
            u, g = u.new_empty((0,)), u.new_empty((0,))
        return y, t, u, g, stats
    t, stats = _depthwise_forward(xb, wdw, bdw, kind, kernel_size, eps)
    if res_w is not None and kind == KIND_DOWN:
        res, _ = pw_gemm(_even(xb), prm.rw, cout, out_dtype=cdt, bias=prm.rb)
    u, g, y = _expansion(t, stats, gn_w, gn_b, prm, cdt, cout, res)
    if not keep_expansion:
        u, g = u.new_empty((0,)), u.new_empty((0,))
    return y, t, u, g, stats


@mednext_block.register_fake
def _(x, addend, dw_w, dw_b, gn_w, gn_b, e_w, e_b, p_w, p_b, res_w, res_b, kind, kernel_size, eps, residual_is_input,
      keep_expansion, compute_dtype):
    cdt = _CODES[compute_dtype]
    n, c = x.shape[0], x.shape[1]
    sp = tuple(x.shape[2:])
    res = x if residual_is_input else addend
    ydt = res.dtype if res is not None and res_w is None else cdt
    if kind == KIND_UP:
        ydt = torch.promote_types(cdt, addend.dtype) if addend is not None else cdt
        big = tuple(2 * s - 1 for s in sp)
        _, pitch = _row_pitch(big)
        y = x.new_empty((n, p_w.shape[0], *(2 * s for s in sp)), dtype=ydt)
        t = x.new_empty((n, c, big[0], big[1], pitch), dtype=cdt)
        u = x.new_empty((n, e_w.shape[0], big[0], big[1], pitch), dtype=cdt) if keep_expansion \
            else x.new_empty((0,), dtype=cdt)
    else:
        if kind == KIND_DOWN:
            sp = tuple((s + 1) // 2 for s in sp)
        y = x.new_empty((n, p_w.shape[0], *sp), dtype=ydt)
        t = x.new_empty((n, c, *sp), dtype=cdt)
        u = x.new_empty((n, e_w.shape[0], *sp), dtype=cdt) if keep_expansion else x.new_empty((0,), dtype=cdt)
    stats = x.new_empty((n * c, 2), dtype=torch.float32)
    vox = int(t[0, 0].numel())
    g = torch.empty_like(u) if keep_expansion and _stores_gelu(n, int(p_w.shape[0]), int(e_w.shape[0]), vox, cdt) \
        else x.new_empty((0,), dtype=cdt)
    return y, t, u, g, stats


@custom_op(f"{_NS}::mednext_block_backward", mutates_args=())
def mednext_block_backward(
    dy: Tensor,
    x: Tensor,
    t: Tensor,
    u_saved: Tensor,
    g_saved: Tensor,
    stats: Tensor,
    dw_w: Tensor,
    gn_w: Tensor,
    gn_b: Tensor,
    e_w: Tensor,
    e_b: Tensor,
    p_w: Tensor,
    res_w: Tensor | None,
    kind: int,
    kernel_size: int,
    residual_is_input: bool,
    compute_dtype: int,
) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Returns (dx, dw_w, dw_b, dgamma, dbeta, de_w, de_b, dp_w, dp_b, dres_w, dres_b)
    in the parameters' dtypes (the last two empty without ``res_w``)."""
    cdt = _CODES[compute_dtype]
    rc, c = int(e_w.shape[0]), int(e_w.shape[1])
    cout = int(p_w.shape[0])
    vox = None
    if kind == KIND_UP:
        # dy is the grad of the padded (2S)^3 output; the pad voxels carry no
        # dependence on the block, so only the (2S-1)^3 interior flows back,
        # repacked into the row-pitched layout with zeros in the pad columns (so
        # the GEMMs' sums over voxels see nothing there)
        big = tuple(2 * int(s) - 1 for s in x.shape[2:])
        vox, pitch = _row_pitch(big)
        dyb = dwk.unpad_front(dy.to(cdt), pitch)
    else:
        dy = dy.contiguous()
        dyb = dy.to(cdt)
    xb = x.to(cdt).contiguous()
    # input grad of the residual GEMM: the down block needs W^T [cin, cout], the up block W [cin, cout]
    rmode = (res_w, kind == KIND_DOWN) if res_w is not None else None
    prm = _block_params(dw_w, None, e_w, e_b, p_w, None, cdt, transposed=True, res=rmode)
    if u_saved.numel() > 0:
        u, g = u_saved, (g_saved if g_saved.numel() > 0 else None)
    else:  # the expansion was not kept (activation checkpointing): recompute it
        ug = None
        if _stores_gelu(int(t.shape[0]), cout, rc, int(t[0, 0].numel()), cdt):
            ug = _expand_gelu(t, stats, gn_w, gn_b, prm)
        u, g = ug if ug is not None else (_expand(t, stats, gn_w, gn_b, prm, cdt), None)
    # project dgrad with the GELU derivative in the epilogue and, where the fused
    # kernel covers the shape, the project weight grad from the same pass
    # the weight grads run on a side stream beside the input-grad chain
    br = _Branch(x.device, True)
    fused = pw_gelu_bwd(dyb, prm.pwt, u)
    if fused is not None:
        du, dpw, dpb = fused
    else:
        # the project weight grad from the stored GELU(u) (else GELU applied on load)
        dpw, dpb = br.run(lambda: pw_wgrad(dyb, g) if g is not None else pw_wgrad(dyb, u, prologue=nat.PRO_GELU))
        du, _ = pw_gemm(dyb, prm.pwt, rc, out_dtype=cdt, aux=u, gelu_grad=True)
    # GroupNorm affine parameters in fp32 for the kernels
    g_w = gn_w.float().contiguous()
    g_b = gn_b.float().contiguous()
    # expand dgrad + GroupNorm-backward partial sums (+ the expand weight grad, fused where covered)
    fused = pw_gn_bwd_fused(du, prm.ewt, t, stats, g_w, g_b)
    if fused is not None:
        dz, part, dew, deb = fused
    else:
        dew, deb = br.run(lambda: pw_wgrad(du, t, prologue=nat.PRO_GROUPNORM, pro_stats=stats, pro_gamma=g_w,
                                           pro_beta=g_b))
        dz, part = pw_gemm(du, prm.ewt, c, out_dtype=cdt, aux=t, gn_bwd_stats=stats)
    dt, dgamma, dbeta = gn_backward_from_partials(dz, t, stats, g_w, part, vox=vox)
    wdw = prm.wdw
    drw = drb = dxr = None
    if res_w is not None:
        cin = int(x.shape[1])
        if kind == KIND_DOWN:
            # residual out[m] = W x[2m] + b: its grad is dy on the small grid
            drw, drb = br.run(lambda: pw_wgrad(dyb, _even(xb)))
            dxr, _ = pw_gemm(dyb, prm.rw, cin, out_dtype=cdt)  # added at the even positions of dx
        else:
            # residual out[2m] = W^T x[m] + b, out[odd] = b: the weight and input grads see dy at
            # the even interior positions (odd in the left-padded output); the bias grad is the
            # sum of dy over the whole interior, which the project GEMM's bias grad already is
            dye = dy[:, :, 1::2, 1::2, 1::2].to(cdt).contiguous()
            drw_t, _ = br.run(lambda: pw_wgrad(dye, xb, want_bias=False))  # [cout, cin]
            drw = drw_t.t()
            drb = None  # dpb, once the side stream has joined
            dxr, _ = pw_gemm(dye, prm.rw, cin, out_dtype=cdt)
    # the depthwise weight grad straight in the parameter's dtype where the kernels offer it
    # (fp32 parameters, 16-bit compute: the same values as a cast of the compute-dtype grad)
    wdt = dw_w.dtype if dw_w.dtype in (xb.dtype, torch.float32) else None
    if kind == KIND_REGULAR:
        dwdw, dbdw = br.run(lambda: dwk.dw_wgrad(xb, dt, kernel_size, out_dtype=wdt))
        dx = dwk.dw_dgrad(dt, wdw, kernel_size, addend=dyb if residual_is_input and dy.dtype == cdt else None)
    elif kind == KIND_DOWN:
        dwdw, dbdw = br.run(lambda: dwk.s2_wgrad(xb, dt, kernel_size, out_dtype=wdt))
        dx = dwk.s2_dgrad(dt, wdw, tuple(int(s) for s in x.shape[2:]), kernel_size, addend_even=dxr)
    else:
        dwdw, dbdw = br.run(lambda: dwk.t_wgrad(xb, dt, kernel_size, out_dtype=wdt))
        dx = dwk.t_dgrad(dt, wdw, kernel_size, small=tuple(int(s) for s in x.shape[2:]), addend=dxr)
    br.join(dpw, dpb, dew, deb, drw, drb, dwdw, dbdw)
    if res_w is not None and kind == KIND_UP:
        drb = dpb.clone()
    if dx.dtype != x.dtype:
        dx = dx.to(x.dtype)
        if residual_is_input:
            dx = dx + dy.to(x.dtype)
    elif residual_is_input and kind != KIND_REGULAR:
        dx = dx + dy
    pdt = dw_w.dtype
    return (
        dx,
        dwdw.to(pdt),
        dbdw.to(pdt),
        dgamma.to(gn_w.dtype),
        dbeta.to(gn_b.dtype),
        dew.reshape(e_w.shape).to(e_w.dtype),
        deb.to(e_b.dtype),
        dpw.reshape(p_w.shape).to(p_w.dtype),
        dpb.to(p_w.dtype),
        drw.reshape(res_w.shape).to(res_w.dtype) if drw is not None else dpw.new_empty((0,)),
        drb.to(res_w.dtype) if drb is not None else dpw.new_empty((0,)),
    )


@mednext_block_backward.register_fake
def _(dy, x, t, u_saved, g_saved, stats, dw_w, gn_w, gn_b, e_w, e_b, p_w, res_w, kind, kernel_size,
      residual_is_input, compute_dtype):
    nres = 0 if res_w is None else res_w.shape[1] if kind == KIND_UP else res_w.shape[0]
    return (
        torch.empty_like(x),
        torch.empty_like(dw_w),
        dw_w.new_empty((dw_w.shape[0],)),
        torch.empty_like(gn_w),
        torch.empty_like(gn_b),
        torch.empty_like(e_w),
        torch.empty_like(e_b),
        torch.empty_like(p_w),
        p_w.new_empty((p_w.shape[0],)),
        torch.empty_like(res_w) if res_w is not None else p_w.new_empty((0,)),
        p_w.new_empty((nres,)),
    )


def _setup(ctx, inputs, output):
    (x, addend, dw_w, dw_b, gn_w, gn_b, e_w, e_b, p_w, p_b, res_w, res_b, kind, k, eps, residual_is_input, keep,
     cdt) = inputs
    y, t, u, g, stats = output
    ctx.save_for_backward(x, t, u, g, stats, dw_w, gn_w, gn_b, e_w, e_b, p_w, res_w)
    ctx.mark_non_differentiable(t, u, g, stats)
    # t, u and stats never receive a gradient: without this, autograd would allocate
    # and zero-fill tensors of their (expanded, full-resolution) shapes every step
    ctx.set_materialize_grads(False)
    ctx.kind = kind
    ctx.k = k
    ctx.residual_is_input = residual_is_input
    ctx.cdt = cdt
    ctx.has_addend = addend is not None
    ctx.addend_dtype = addend.dtype if addend is not None else None


def _backward(ctx, dy, _dt, _du, _dg, _dstats):
    if dy is None:  # the block output does not reach the loss
        return (None,) * 18
    x, t, u, g, stats, dw_w, gn_w, gn_b, e_w, e_b, p_w, res_w = ctx.saved_tensors
    dx, dww, dwb, dgw, dgb, dew, deb, dpw, dpb, drw, drb = mednext_block_backward(
        dy, x, t, u, g, stats, dw_w, gn_w, gn_b, e_w, e_b, p_w, res_w, ctx.kind, ctx.k, ctx.residual_is_input,
        ctx.cdt
    )
    if res_w is None:
        drw = drb = None
    d_add = None
    if ctx.has_addend and ctx.needs_input_grad[1]:
        # the up block's addend is added after the pad: its grad is all of dy
        d_add = dy if dy.dtype == ctx.addend_dtype else dy.to(ctx.addend_dtype)
    return dx, d_add, dww, dwb, dgw, dgb, dew, deb, dpw, dpb, drw, drb, None, None, None, None, None, None


mednext_block.register_autograd(_backward, setup_context=_setup)


def dtype_code(dtype: torch.dtype) -> int:
    for code, dt in _CODES.items():
        if dt == dtype:
            return code
    raise ValueError(f"unsupported compute dtype {dtype}")

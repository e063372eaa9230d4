"""Tensor-core pointwise (1x1x1) convolution and GroupNorm operators.

``pointwise_conv3d`` is the sm_100a replacement of the reference's
``AdaptivePointwise3d._gemm`` (per-sample ``torch.addmm``, ops/adaptive.py:174-188)
and of the native ``F.conv3d`` it otherwise calls (ops/adaptive.py:200).
``group_norm`` covers ``nn.GroupNorm(C, C)`` (models/blocks.py:74) for the
per-operator path; the fused block applies GroupNorm inside its GEMM prologue.

The ``pw_*`` / ``gn_*`` helpers are the raw launches used by the custom ops here
and by :mod:`mednext_accel_b200.block`.
"""

from __future__ import annotations

import torch
from torch import Tensor
from torch.library import custom_op

from . import _native as nat

_NS = "mednext_accel_b200"


def _vox(t: Tensor) -> int:
    v = 1
    for s in t.shape[2:]:
        v *= int(s)
    return v


# --------------------------------------------------------------------------- raw launches
def pw_gemm(
    a: Tensor,
    wt: Tensor,
    cout: int,
    *,
    out_dtype: torch.dtype | None = None,
    prologue: int = nat.PRO_NONE,
    pro_stats: Tensor | None = None,
    pro_gamma: Tensor | None = None,
    pro_beta: Tensor | None = None,
    bias: Tensor | None = None,
    residual: Tensor | None = None,
    aux: Tensor | None = None,
    gelu_grad: bool = False,
    gn_bwd_stats: Tensor | None = None,
    out: Tensor | None = None,
    pro_out: Tensor | None = None,
) -> tuple[Tensor, Tensor | None]:
    """y[s, j, v] = epi(sum_k wt[j, k] * pro(a[s, k, v])) on the tensor cores.

    ``a``: [S, cin, *spatial]; ``wt``: [cout, cin] contiguous in a's dtype.
    ``pro_out`` (shape and dtype of ``a``): receives pro(a) as the GEMM consumed it.
    Returns (y, gn_partial_workspace or None)."""
    nat.require_device(a)
    lib = nat.load()
    n, cin = int(a.shape[0]), int(a.shape[1])
    vox = _vox(a)
    odt = out_dtype or (residual.dtype if residual is not None else a.dtype)
    y = out if out is not None else torch.empty((n, cout, *a.shape[2:]), dtype=odt, device=a.device)
    epi = 0
    if bias is not None:
        epi |= nat.EPI_BIAS
    if residual is not None:
        epi |= nat.EPI_RESIDUAL
    if gelu_grad:
        epi |= nat.EPI_GELU_GRAD
    if gn_bwd_stats is not None:
        epi |= nat.EPI_GN_BWD_STATS
    ws_bytes = lib.mednext_pw_fwd_workspace_size(n, cin, cout, vox, epi)
    ws = nat.workspace(ws_bytes, a.device) if ws_bytes > 0 else None
    if pro_out is not None and (pro_out.shape != a.shape or pro_out.dtype != a.dtype or not pro_out.is_contiguous()):
        raise ValueError("pro_out must be a contiguous tensor of a's shape and dtype")
    nat.check(
        lib.mednext_pw_fwd_pro_out(
            a.data_ptr(), wt.data_ptr(), y.data_ptr(), prologue, nat.ptr(pro_stats), nat.ptr(pro_gamma),
            nat.ptr(pro_beta), epi, nat.ptr(bias), nat.ptr(residual), nat.ptr(aux), nat.ptr(gn_bwd_stats),
            nat.ptr(pro_out), nat.ptr(ws), 0 if ws is None else ws.numel(), n, cin, cout, vox,
            nat.dtype_code(a.dtype), nat.dtype_code(y.dtype), nat.stream(),
        ),
        "mednext_pw_fwd_pro_out",
    )
    return y, ws


def pw_gemm_gelu_out(
    a: Tensor,
    wt: Tensor,
    cout: int,
    *,
    prologue: int = nat.PRO_NONE,
    pro_stats: Tensor | None = None,
    pro_gamma: Tensor | None = None,
    pro_beta: Tensor | None = None,
    bias: Tensor | None = None,
) -> tuple[Tensor, Tensor] | None:
    """(y, g): y = W @ pro(a) (+ bias) in a's dtype and g = GELU(y) (of y as stored),
    both written by one kernel.  None when the entry point does not cover the call
    (dtype, prologue or shape); the caller then applies GELU as the next GEMM's prologue."""
    nat.require_device(a)
    lib = nat.load()
    n, cin = int(a.shape[0]), int(a.shape[1])
    vox = _vox(a)
    y = torch.empty((n, cout, *a.shape[2:]), dtype=a.dtype, device=a.device)
    g = torch.empty_like(y)
    epi = nat.EPI_BIAS if bias is not None else 0
    ws_bytes = lib.mednext_pw_fwd_workspace_size(n, cin, cout, vox, epi)
    ws = nat.workspace(ws_bytes, a.device) if ws_bytes > 0 else None
    st = lib.mednext_pw_fwd_gelu_out(
        a.data_ptr(), wt.data_ptr(), y.data_ptr(), g.data_ptr(), prologue, nat.ptr(pro_stats), nat.ptr(pro_gamma),
        nat.ptr(pro_beta), nat.ptr(bias), nat.ptr(ws), 0 if ws is None else ws.numel(), n, cin, cout, vox,
        nat.dtype_code(a.dtype), nat.stream(),
    )
    if st == nat.ERR_UNSUPPORTED:
        return None
    nat.check(st, "mednext_pw_fwd_gelu_out")
    return y, g


def pw_wgrad(
    g: Tensor,
    a: Tensor,
    *,
    prologue: int = nat.PRO_NONE,
    pro_stats: Tensor | None = None,
    pro_gamma: Tensor | None = None,
    pro_beta: Tensor | None = None,
    want_bias: bool = True,
) -> tuple[Tensor, Tensor | None]:
    """dw[j, k] = sum_{s,v} g[s,j,v] * pro(a[s,k,v]) (fp32), dbias[j] = sum g."""
    nat.require_device(g)
    lib = nat.load()
    n, cout = int(g.shape[0]), int(g.shape[1])
    cin = int(a.shape[1])
    vox = _vox(g)
    dw = torch.empty((cout, cin), dtype=torch.float32, device=g.device)
    db = torch.empty((cout,), dtype=torch.float32, device=g.device) if want_bias else None
    ws = nat.workspace(lib.mednext_pw_wgrad_workspace_size(n, cin, cout, vox), g.device)
    nat.check(
        lib.mednext_pw_wgrad(
            g.data_ptr(), a.data_ptr(), dw.data_ptr(), nat.ptr(db), prologue, nat.ptr(pro_stats),
            nat.ptr(pro_gamma), nat.ptr(pro_beta), ws.data_ptr(), ws.numel(), n, cin, cout, vox,
            nat.dtype_code(g.dtype), nat.stream(),
        ),
        "mednext_pw_wgrad",
    )
    return dw, db


def gelu_bwd_fused_covers(n: int, c: int, h: int, vox: int, dtype: torch.dtype) -> bool:
    """Whether ``pw_gelu_bwd`` (the compress input grad with its weight grad fused in)
    covers a block whose project GEMM maps h expanded channels to c."""
    return nat.load().mednext_pw_gelu_bwd_workspace_size(n, c, h, vox, nat.dtype_code(dtype)) > 0


def pw_gelu_bwd(dy: Tensor, wpt: Tensor, u: Tensor) -> tuple[Tensor, Tensor, Tensor] | None:
    """Backward of y = W @ GELU(u) in one fused kernel: (du, dW, dbias) with
    du = (W^T dy) * GELU'(u), dW = sum_v dy GELU(u)^T (fp32), dbias = sum_v dy (fp32).
    ``dy``: [S, c, *spatial]; ``wpt`` = W^T: [h, c]; ``u``: [S, h, *spatial].  Returns
    None when the fused kernel does not cover the shape (the caller runs pw_gemm and
    pw_wgrad instead)."""
    nat.require_device(dy)
    lib = nat.load()
    n, c = int(dy.shape[0]), int(dy.shape[1])
    h = int(u.shape[1])
    vox = _vox(dy)
    code = nat.dtype_code(dy.dtype)
    ws_bytes = lib.mednext_pw_gelu_bwd_workspace_size(n, c, h, vox, code)
    if ws_bytes == 0:
        return None
    ws = nat.workspace(ws_bytes, dy.device)
    du = torch.empty_like(u)
    dw = torch.empty((c, h), dtype=torch.float32, device=dy.device)
    db = torch.empty((c,), dtype=torch.float32, device=dy.device)
    st = lib.mednext_pw_gelu_bwd(
        dy.data_ptr(), wpt.data_ptr(), u.data_ptr(), du.data_ptr(), dw.data_ptr(), db.data_ptr(), ws.data_ptr(),
        ws.numel(), n, c, h, vox, code, nat.stream(),
    )
    if st == nat.ERR_UNSUPPORTED:
        return None
    nat.check(st, "mednext_pw_gelu_bwd")
    return du, dw, db


def pw_mlp_fwd(
    t: Tensor, stats: Tensor, gamma: Tensor, beta: Tensor, we: Tensor, be: Tensor, wp: Tensor, bp: Tensor,
    residual: Tensor | None = None,
) -> tuple[Tensor, Tensor] | None:
    """The block's expansion in one kernel: (u, y) with u = we @ GroupNorm(t) + be and
    y = wp @ GELU(u) + bp (+ residual).  ``t``: [S, c, *spatial]; ``we``: [h, c];
    ``wp``: [c2, h] (t's dtype); ``be``, ``bp``, ``gamma``, ``beta``: fp32.  None when
    the fused kernel does not cover the shape."""
    nat.require_device(t)
    n, c = int(t.shape[0]), int(t.shape[1])
    h, c2 = int(we.shape[0]), int(wp.shape[0])
    vox = _vox(t)
    u = torch.empty((n, h, *t.shape[2:]), dtype=t.dtype, device=t.device)
    y = torch.empty((n, c2, *t.shape[2:]), dtype=t.dtype, device=t.device)
    if residual is not None and (residual.dtype != t.dtype or tuple(residual.shape) != tuple(y.shape)):
        return None
    st = nat.load().mednext_pw_mlp_fwd(
        t.data_ptr(), stats.data_ptr(), gamma.data_ptr(), beta.data_ptr(), we.data_ptr(), be.data_ptr(),
        wp.data_ptr(), bp.data_ptr(), nat.ptr(residual), u.data_ptr(), y.data_ptr(), n, c, h, c2, vox,
        nat.dtype_code(t.dtype), nat.stream(),
    )
    if st == nat.ERR_UNSUPPORTED:
        return None
    nat.check(st, "mednext_pw_mlp_fwd")
    return u, y


def pw_gn_bwd_fused(
    du: Tensor, wt: Tensor, t: Tensor, stats: Tensor, gamma: Tensor, beta: Tensor
) -> tuple[Tensor, Tensor, Tensor, Tensor] | None:
    """Backward of u = W @ GroupNorm(t) in one fused kernel: (dz, partials, dW, dbias)
    with dz = W^T du (its GroupNorm-backward partial sums in ``partials``, for
    gn_backward_from_partials), dW = sum_v du GroupNorm(t)^T (fp32) and dbias = sum_v du.
    ``du``: [S, h, *spatial]; ``wt`` = W^T: [c, h]; ``t``: [S, c, *spatial]; ``gamma``,
    ``beta``: fp32 [c].  None when the fused kernel does not cover the shape."""
    nat.require_device(du)
    lib = nat.load()
    n, h = int(du.shape[0]), int(du.shape[1])
    c = int(t.shape[1])
    vox = _vox(du)
    code = nat.dtype_code(du.dtype)
    ws_bytes = lib.mednext_pw_gn_bwd_fused_workspace_size(n, h, c, vox, code)
    if ws_bytes == 0:
        return None
    ws = nat.workspace(ws_bytes, du.device)
    dz = torch.empty_like(t)
    dw = torch.empty((h, c), dtype=torch.float32, device=du.device)
    db = torch.empty((h,), dtype=torch.float32, device=du.device)
    st = lib.mednext_pw_gn_bwd_fused(
        du.data_ptr(), wt.data_ptr(), t.data_ptr(), stats.data_ptr(), gamma.data_ptr(), beta.data_ptr(),
        dz.data_ptr(), dw.data_ptr(), db.data_ptr(), ws.data_ptr(), ws.numel(), n, h, c, vox, code, nat.stream(),
    )
    if st == nat.ERR_UNSUPPORTED:
        return None
    nat.check(st, "mednext_pw_gn_bwd_fused")
    return dz, ws, dw, db


def gn_stats(x: Tensor, eps: float, vox: int | None = None, row_len: int | None = None) -> Tensor:
    """Per-(n, c) mean / rstd.  ``vox``: number of valid voxels when ``x`` is a pitched
    [n, c, pitch] buffer (only the first ``vox`` of each row are statistics).
    ``row_len``: x is row-pitched [n, c, ..., row_pitch] and only the first
    ``row_len`` elements of each last-axis row are statistics."""
    nat.require_device(x)
    lib = nat.load()
    n, c = int(x.shape[0]), int(x.shape[1])
    rows = _vox(x)
    stats = torch.empty((n * c, 2), dtype=torch.float32, device=x.device)
    if row_len is not None:
        rp = int(x.shape[-1])
        ws = nat.workspace(lib.mednext_gn_stats_workspace_size(n, c, rows), x.device)
        nat.check(
            lib.mednext_gn_stats_rows(
                x.data_ptr(), stats.data_ptr(), ws.data_ptr(), ws.numel(), n, c, rows // rp, int(row_len), rp,
                float(eps), nat.dtype_code(x.dtype), nat.stream(),
            ),
            "mednext_gn_stats_rows",
        )
        return stats
    vox = rows if vox is None else int(vox)
    ws = nat.workspace(lib.mednext_gn_stats_workspace_size(n, c, vox), x.device)
    nat.check(
        lib.mednext_gn_stats(
            x.data_ptr(), stats.data_ptr(), ws.data_ptr(), ws.numel(), n, c, vox, rows, float(eps),
            nat.dtype_code(x.dtype), nat.stream(),
        ),
        "mednext_gn_stats",
    )
    return stats


def gn_apply(x: Tensor, stats: Tensor, gamma: Tensor | None, beta: Tensor | None, out_dtype: torch.dtype) -> Tensor:
    nat.require_device(x)
    n, c = int(x.shape[0]), int(x.shape[1])
    y = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    gdt = gamma.dtype if gamma is not None else torch.float32
    nat.check(
        nat.load().mednext_gn_fwd(
            x.data_ptr(), stats.data_ptr(), nat.ptr(gamma), nat.ptr(beta), y.data_ptr(), n, c, _vox(x),
            nat.dtype_code(x.dtype), nat.dtype_code(out_dtype), nat.dtype_code(gdt), nat.stream(),
        ),
        "mednext_gn_fwd",
    )
    return y


def gn_backward(
    dy: Tensor, x: Tensor, stats: Tensor, gamma: Tensor | None, want_param_grads: bool = True
) -> tuple[Tensor, Tensor | None, Tensor | None]:
    nat.require_device(x)
    lib = nat.load()
    n, c = int(x.shape[0]), int(x.shape[1])
    vox = _vox(x)
    dx = torch.empty_like(x)
    dg = torch.empty((c,), dtype=torch.float32, device=x.device) if want_param_grads else None
    db = torch.empty((c,), dtype=torch.float32, device=x.device) if want_param_grads else None
    ws = nat.workspace(lib.mednext_gn_bwd_workspace_size(n, c, vox), x.device)
    gdt = gamma.dtype if gamma is not None else torch.float32
    nat.check(
        lib.mednext_gn_bwd(
            dy.data_ptr(), x.data_ptr(), stats.data_ptr(), nat.ptr(gamma), dx.data_ptr(), nat.ptr(dg), nat.ptr(db),
            ws.data_ptr(), ws.numel(), n, c, vox, nat.dtype_code(dy.dtype), nat.dtype_code(x.dtype),
            nat.dtype_code(x.dtype), nat.dtype_code(gdt), nat.stream(),
        ),
        "mednext_gn_bwd",
    )
    return dx, dg, db


def gn_backward_from_partials(
    dz: Tensor, x: Tensor, stats: Tensor, gamma: Tensor, partials: Tensor, vox: int | None = None
) -> tuple[Tensor, Tensor, Tensor]:
    """GroupNorm backward from the GEMM-epilogue partials (consumed in place).
    ``vox``: valid voxels per row when ``x``/``dz`` are pitched [n, c, pitch] buffers."""
    n, c = int(x.shape[0]), int(x.shape[1])
    rows = _vox(x)
    vox = rows if vox is None else int(vox)
    dx = torch.empty_like(x)
    dg = torch.empty((c,), dtype=torch.float32, device=x.device)
    db = torch.empty((c,), dtype=torch.float32, device=x.device)
    nat.check(
        nat.load().mednext_gn_bwd_from_partials(
            dz.data_ptr(), x.data_ptr(), stats.data_ptr(), gamma.data_ptr(), dx.data_ptr(), dg.data_ptr(),
            db.data_ptr(), partials.data_ptr(), n, c, vox, rows, nat.dtype_code(dz.dtype), nat.dtype_code(x.dtype),
            nat.dtype_code(x.dtype), nat.dtype_code(gamma.dtype), nat.stream(),
        ),
        "mednext_gn_bwd_from_partials",
    )
    return dx, dg, db


# --------------------------------------------------------------------------- pointwise op
def _check_pointwise(x: Tensor, weight: Tensor) -> None:
    if x.ndim != 5 or weight.ndim != 5 or tuple(weight.shape[2:]) != (1, 1, 1):
        raise ValueError("pointwise_conv3d expects NCDHW input and a [Cout, Cin, 1, 1, 1] weight")
    if x.dtype not in (torch.bfloat16, torch.float16) or weight.dtype != x.dtype:
        raise ValueError("pointwise_conv3d computes on the tensor cores in bfloat16 or float16")
    if not x.is_contiguous():
        raise ValueError("contiguous tensors are required")


@custom_op(f"{_NS}::pointwise_conv3d", mutates_args=())
def pointwise_conv3d(x: Tensor, weight: Tensor, bias: Tensor | None) -> Tensor:
    """1x1x1 convolution y = W x + b with fp32 accumulation; x, W, b share a dtype."""
    _check_pointwise(x, weight)
    cout = int(weight.shape[0])
    b = bias.float() if bias is not None else None
    y, _ = pw_gemm(x, weight.reshape(cout, -1).contiguous(), cout, bias=b, out_dtype=x.dtype)
    return y


@pointwise_conv3d.register_fake
def _(x, weight, bias):
    return x.new_empty((x.shape[0], weight.shape[0], *x.shape[2:]))


@custom_op(f"{_NS}::pointwise_conv3d_backward", mutates_args=())
def pointwise_conv3d_backward(
    grad: Tensor, x: Tensor, weight: Tensor, need_input: bool, need_bias: bool
) -> tuple[Tensor, Tensor, Tensor]:
    cout, cin = int(weight.shape[0]), int(weight.shape[1])
    grad = grad.contiguous()
    if need_input:
        wt_t = weight.reshape(cout, cin).t().contiguous()  # [cin, cout]
        dx, _ = pw_gemm(grad, wt_t, cin, out_dtype=x.dtype)
    else:
        dx = x.new_empty((0,))
    dw, db = pw_wgrad(grad, x, want_bias=need_bias)
    return dx, dw.to(weight.dtype).reshape(weight.shape), (db.to(weight.dtype) if db is not None else x.new_empty((0,)))


@pointwise_conv3d_backward.register_fake
def _(grad, x, weight, need_input, need_bias):
    dx = torch.empty_like(x) if need_input else x.new_empty((0,))
    db = weight.new_empty((weight.shape[0],)) if need_bias else x.new_empty((0,))
    return dx, torch.empty_like(weight), db


def _pw_setup(ctx, inputs, output):
    x, weight, bias = inputs
    ctx.save_for_backward(x, weight)
    ctx.has_bias = bias is not None


def _pw_backward(ctx, grad):
    x, weight = ctx.saved_tensors
    need_dx, need_dw, need_db = ctx.needs_input_grad
    need_db = need_db and ctx.has_bias
    dx, dw, db = pointwise_conv3d_backward(grad, x, weight, need_dx, need_db)
    return (dx if need_dx else None), (dw if need_dw else None), (db if need_db else None)


pointwise_conv3d.register_autograd(_pw_backward, setup_context=_pw_setup)


# --------------------------------------------------------------------------- GroupNorm op
@custom_op(f"{_NS}::group_norm", mutates_args=())
def group_norm(x: Tensor, weight: Tensor | None, bias: Tensor | None, eps: float) -> tuple[Tensor, Tensor]:
    """GroupNorm with one group per channel; returns (y, stats[N*C, 2])."""
    if not x.is_contiguous():
        raise ValueError("contiguous tensors are required")
    stats = gn_stats(x, eps)
    return gn_apply(x, stats, weight, bias, x.dtype), stats


@group_norm.register_fake
def _(x, weight, bias, eps):
    return torch.empty_like(x), x.new_empty((x.shape[0] * x.shape[1], 2), dtype=torch.float32)


@custom_op(f"{_NS}::group_norm_backward", mutates_args=())
def group_norm_backward(grad: Tensor, x: Tensor, stats: Tensor, weight: Tensor | None) -> tuple[Tensor, Tensor, Tensor]:
    dx, dg, db = gn_backward(grad.contiguous(), x, stats, weight, True)
    return dx, dg, db


@group_norm_backward.register_fake
def _(grad, x, stats, weight):
    c = x.shape[1]
    return torch.empty_like(x), x.new_empty((c,), dtype=torch.float32), x.new_empty((c,), dtype=torch.float32)


def _gn_setup(ctx, inputs, output):
    x, weight, bias, eps = inputs
    ctx.save_for_backward(x, output[1], weight)
    ctx.mark_non_differentiable(output[1])
    ctx.param_dtype = weight.dtype if weight is not None else None


def _gn_backward(ctx, grad, _grad_stats):
    x, stats, weight = ctx.saved_tensors
    dx, dg, db = group_norm_backward(grad, x, stats, weight)
    need_x, need_w, need_b = ctx.needs_input_grad[:3]
    pdt = ctx.param_dtype
    return (
        dx if need_x else None,
        dg.to(pdt) if need_w and pdt is not None else None,
        db.to(pdt) if need_b and pdt is not None else None,
        None,
    )


group_norm.register_autograd(_gn_backward, setup_context=_gn_setup)

"""Depthwise Conv3d operators for sm_100a behind the reference operator contract.

Names, signatures and argument meaning follow the reference module
``mednext_accel/ops/_triton/depthwise.py``:

* low-level functions ``depthwise_input_grad``, ``depthwise_stride2_input_grad``,
  ``depthwise_weight_grad``, ``depthwise_transpose_weight_grad`` (reference
  lines 271-442), with the same ``ValueError`` checks;
* ``torch.library`` custom ops ``depthwise_conv3d_odd_regular``,
  ``depthwise_conv3d_stride2_regular``, ``depthwise_conv_transpose3d_odd_regular``
  and their gradient ops (reference lines 445-850), registered in the
  ``mednext_accel_b200`` namespace with fake (meta) kernels and autograd.

Differences, all in the direction of doing more on the GPU: the forward passes
and every gradient phase (including the bias gradient and the phases the
reference leaves to ATen) run the kernels of ``libmednext_b200.so``.  The
Triton launch knobs (``dw_splits``, ``dw_block``, ``dx_block``) are accepted for
signature compatibility and ignored: tiling comes from the fixed sm_100a plan.
``custom_dx``/``custom_dw`` are accepted and ignored for the same reason.
"""

from __future__ import annotations

import torch
from torch import Tensor
from torch.library import custom_op

from . import _native as nat

_NS = "mednext_accel_b200"


def _dims(t: Tensor) -> tuple[int, int, int, int, int]:
    n, c, d, h, w = (int(v) for v in t.shape)
    return n, c, d, h, w


def _check_kernel(kernel_size: int) -> None:
    if kernel_size < 1 or kernel_size % 2 == 0:
        raise ValueError("kernel_size must be a positive odd integer")


# --------------------------------------------------------------------------- raw launches
def dw_forward(x: Tensor, weight: Tensor, bias: Tensor | None, kernel_size: int, gn_eps: float | None = None):
    """Stride-1 forward; with ``gn_eps`` also returns GroupNorm(C, C) statistics of y."""
    nat.require_device(x)
    lib = nat.load()
    n, c, d, h, w = _dims(x)
    code = nat.dtype_code(x.dtype)
    y = torch.empty_like(x)
    stats = ws = None
    if gn_eps is not None:
        stats = torch.empty((n * c, 2), dtype=torch.float32, device=x.device)
        ws = nat.workspace(lib.mednext_dw_fwd_workspace_size(n, c, d, h, w, kernel_size, code), x.device)
    nat.check(
        lib.mednext_dw_fwd(
            x.data_ptr(), weight.data_ptr(), nat.ptr(bias), y.data_ptr(), nat.ptr(stats),
            float(gn_eps or 0.0), nat.ptr(ws), 0 if ws is None else ws.numel(),
            n, c, d, h, w, kernel_size, code, nat.stream(),
        ),
        "mednext_dw_fwd",
    )
    return (y, stats) if gn_eps is not None else y


def dw_dgrad(grad: Tensor, weight: Tensor, kernel_size: int, addend: Tensor | None = None) -> Tensor:
    nat.require_device(grad)
    n, c, d, h, w = _dims(grad)
    out = torch.empty_like(grad)
    nat.check(
        nat.load().mednext_dw_dgrad(
            grad.data_ptr(), weight.data_ptr(), nat.ptr(addend), out.data_ptr(), n, c, d, h, w, kernel_size,
            nat.dtype_code(grad.dtype), nat.stream(),
        ),
        "mednext_dw_dgrad",
    )
    return out


def _wgrad_outputs(x: Tensor, kernel_size: int, want_bias: bool, out_dtype: torch.dtype | None):
    """dW / dbias buffers and the entry-point suffix: ``out_dtype=torch.float32`` asks for
    fp32 results (x's dtype rounding, widened) from the ``_f32out`` entry points."""
    c = int(x.shape[1])
    odt = x.dtype if out_dtype is None else out_dtype
    if odt not in (x.dtype, torch.float32):
        raise ValueError(f"weight grads come in {x.dtype} or float32, not {odt}")
    suffix = "_f32out" if odt != x.dtype else ""
    dw = torch.empty((c, 1, kernel_size, kernel_size, kernel_size), dtype=odt, device=x.device)
    db = torch.empty((c,), dtype=odt, device=x.device) if want_bias else None
    return dw, db, suffix


def dw_wgrad(x: Tensor, grad: Tensor, kernel_size: int, want_bias: bool = True,
             out_dtype: torch.dtype | None = None) -> tuple[Tensor, Tensor | None]:
    nat.require_device(x)
    lib = nat.load()
    n, c, d, h, w = _dims(x)
    code = nat.dtype_code(x.dtype)
    dw, db, suffix = _wgrad_outputs(x, kernel_size, want_bias, out_dtype)
    ws = nat.workspace(lib.mednext_dw_wgrad_workspace_size(n, c, d, h, w, kernel_size, code), x.device)
    nat.check(
        getattr(lib, "mednext_dw_wgrad" + suffix)(
            x.data_ptr(), grad.data_ptr(), dw.data_ptr(), nat.ptr(db), ws.data_ptr(), ws.numel(),
            n, c, d, h, w, kernel_size, code, nat.stream(),
        ),
        "mednext_dw_wgrad" + suffix,
    )
    return dw, db


def s2_forward(x: Tensor, weight: Tensor, bias: Tensor | None, kernel_size: int) -> Tensor:
    nat.require_device(x)
    n, c, d, h, w = _dims(x)
    y = torch.empty((n, c, (d + 1) // 2, (h + 1) // 2, (w + 1) // 2), dtype=x.dtype, device=x.device)
    nat.check(
        nat.load().mednext_dw_s2_fwd(
            x.data_ptr(), weight.data_ptr(), nat.ptr(bias), y.data_ptr(), n, c, d, h, w, kernel_size,
            nat.dtype_code(x.dtype), nat.stream(),
        ),
        "mednext_dw_s2_fwd",
    )
    return y


def s2_dgrad(grad: Tensor, weight: Tensor, input_size: tuple[int, int, int], kernel_size: int,
             addend_even: Tensor | None = None) -> Tensor:
    """Input grad of the stride-2 depthwise conv; ``addend_even`` (grad's shape) is
    added at the all-even input positions (the strided 1x1 residual's input grad)."""
    nat.require_device(grad)
    n, c = int(grad.shape[0]), int(grad.shape[1])
    d, h, w = (int(v) for v in input_size)
    if addend_even is not None:
        _check_addend(addend_even, grad.shape, grad.dtype, "addend_even")
        addend_even = addend_even.contiguous()
    out = torch.empty((n, c, d, h, w), dtype=grad.dtype, device=grad.device)
    nat.check(
        nat.load().mednext_dw_s2_dgrad(
            grad.data_ptr(), weight.data_ptr(), nat.ptr(addend_even), out.data_ptr(), n, c, d, h, w, kernel_size,
            nat.dtype_code(grad.dtype), nat.stream(),
        ),
        "mednext_dw_s2_dgrad",
    )
    return out


def s2_wgrad(x: Tensor, grad: Tensor, kernel_size: int, want_bias: bool = True,
             out_dtype: torch.dtype | None = None) -> tuple[Tensor, Tensor | None]:
    nat.require_device(x)
    lib = nat.load()
    n, c, d, h, w = _dims(x)
    code = nat.dtype_code(x.dtype)
    dw, db, suffix = _wgrad_outputs(x, kernel_size, want_bias, out_dtype)
    ws = nat.workspace(lib.mednext_dw_s2_wgrad_workspace_size(n, c, d, h, w, kernel_size, code), x.device)
    nat.check(
        getattr(lib, "mednext_dw_s2_wgrad" + suffix)(
            x.data_ptr(), grad.data_ptr(), dw.data_ptr(), nat.ptr(db), ws.data_ptr(), ws.numel(),
            n, c, d, h, w, kernel_size, code, nat.stream(),
        ),
        "mednext_dw_s2_wgrad" + suffix,
    )
    return dw, db


def t_forward(x: Tensor, weight: Tensor, bias: Tensor | None, kernel_size: int, row_pitch: int = 0) -> Tensor:
    """Transposed stride-2 forward: [n, c, 2d-1, 2h-1, 2w-1].  With ``row_pitch`` > 0
    the result is [n, c, 2d-1, 2h-1, row_pitch]: every W-row is padded to
    ``row_pitch`` elements with zeros (see :func:`pitched_view`)."""
    nat.require_device(x)
    n, c, d, h, w = _dims(x)
    big = (2 * d - 1, 2 * h - 1, 2 * w - 1)
    shape = (n, c, big[0], big[1], int(row_pitch) if row_pitch else big[2])
    y = torch.empty(shape, dtype=x.dtype, device=x.device)
    nat.check(
        nat.load().mednext_dwT_fwd(
            x.data_ptr(), weight.data_ptr(), nat.ptr(bias), y.data_ptr(), n, c, d, h, w, int(row_pitch), kernel_size,
            nat.dtype_code(x.dtype), nat.stream(),
        ),
        "mednext_dwT_fwd",
    )
    return y


def t_forward_stats(x: Tensor, weight: Tensor, bias: Tensor | None, kernel_size: int, gn_eps: float,
                    row_pitch: int = 0) -> tuple[Tensor, Tensor]:
    """:func:`t_forward` plus the GroupNorm statistics of its output over the grid
    voxels: float32 [n*c, 2] (mean, rstd)."""
    nat.require_device(x)
    lib = nat.load()
    n, c, d, h, w = _dims(x)
    big = (2 * d - 1, 2 * h - 1, 2 * w - 1)
    y = torch.empty((n, c, big[0], big[1], int(row_pitch) if row_pitch else big[2]), dtype=x.dtype, device=x.device)
    stats = torch.empty((n * c, 2), dtype=torch.float32, device=x.device)
    code = nat.dtype_code(x.dtype)
    ws = nat.workspace(lib.mednext_dwT_fwd_workspace_size(n, c, d, h, w, int(row_pitch), kernel_size, code), x.device)
    nat.check(
        lib.mednext_dwT_fwd_stats(
            x.data_ptr(), weight.data_ptr(), nat.ptr(bias), y.data_ptr(), stats.data_ptr(), float(gn_eps),
            ws.data_ptr(), ws.numel(), n, c, d, h, w, int(row_pitch), kernel_size, code, nat.stream(),
        ),
        "mednext_dwT_fwd_stats",
    )
    return y, stats


def pitched_view(buf: Tensor, spatial: tuple[int, int, int]) -> Tensor:
    """The [n, c, *spatial] view of the grid voxels of a row-pitched
    [n, c, d, h, row_pitch] buffer (its first ``spatial[2]`` columns)."""
    return buf[..., : int(spatial[2])]


def _row_pitch(t: Tensor, width: int) -> int:
    """W-row pitch of a [n, c, d, h, pitch] grid whose rows hold ``width`` voxels
    (0 when the rows are packed)."""
    if t.ndim != 5 or int(t.shape[4]) < width:
        raise ValueError(f"expected a [n, c, d, h, >= {width}] tensor")
    return 0 if int(t.shape[4]) == width else int(t.shape[4])


def t_dgrad(grad: Tensor, weight: Tensor, kernel_size: int, small: tuple[int, int, int] | None = None,
            addend: Tensor | None = None) -> Tensor:
    """Input grad of the transposed conv.  ``grad`` is [n, c, 2d-1, 2h-1, 2w-1] or,
    when ``small`` = (d, h, w) is given, a row-pitched [n, c, 2d-1, 2h-1, pitch]
    buffer (pad columns ignored).  ``addend`` (the output's shape) is added to the
    result."""
    nat.require_device(grad)
    n, c = int(grad.shape[0]), int(grad.shape[1])
    if small is not None:
        d, h, w = (int(v) for v in small)
    else:
        _, _, od, oh, ow = _dims(grad)
        d, h, w = (od + 1) // 2, (oh + 1) // 2, (ow + 1) // 2
    pitch = _row_pitch(grad, 2 * w - 1)
    out = torch.empty((n, c, d, h, w), dtype=grad.dtype, device=grad.device)
    if addend is not None:
        _check_addend(addend, out.shape, out.dtype, "addend")
        addend = addend.contiguous()
    nat.check(
        nat.load().mednext_dwT_dgrad(
            grad.data_ptr(), weight.data_ptr(), nat.ptr(addend), out.data_ptr(), n, c, d, h, w, pitch, kernel_size,
            nat.dtype_code(grad.dtype), nat.stream(),
        ),
        "mednext_dwT_dgrad",
    )
    return out


def t_wgrad(x: Tensor, grad: Tensor, kernel_size: int, want_bias: bool = True,
            out_dtype: torch.dtype | None = None) -> tuple[Tensor, Tensor | None]:
    """Weight (and bias) grad of the transposed conv; ``grad`` is
    [n, c, 2d-1, 2h-1, 2w-1] or row-pitched [n, c, 2d-1, 2h-1, pitch]."""
    nat.require_device(x)
    lib = nat.load()
    n, c, d, h, w = _dims(x)
    pitch = _row_pitch(grad, 2 * w - 1)
    code = nat.dtype_code(x.dtype)
    dw, db, suffix = _wgrad_outputs(x, kernel_size, want_bias, out_dtype)
    ws = nat.workspace(lib.mednext_dwT_wgrad_workspace_size(n, c, d, h, w, kernel_size, code), x.device)
    nat.check(
        getattr(lib, "mednext_dwT_wgrad" + suffix)(
            x.data_ptr(), grad.data_ptr(), dw.data_ptr(), nat.ptr(db), ws.data_ptr(), ws.numel(),
            n, c, d, h, w, pitch, kernel_size, code, nat.stream(),
        ),
        "mednext_dwT_wgrad" + suffix,
    )
    return dw, db


# --------------------------------------------------------------------------- low-level API
def _check_addend(t: Tensor, shape, dtype, name: str) -> None:
    if not t.is_cuda or tuple(t.shape) != tuple(shape) or t.dtype != dtype:
        raise ValueError(f"{name} must be a CUDA tensor of shape {tuple(shape)} and dtype {dtype}")


def pad_front_add(v: Tensor, spatial: tuple[int, int, int], addend: Tensor | None = None) -> Tensor:
    """``F.pad(pitched_view(v, spatial), (1, 0) * 3) + addend`` in one pass: ``v`` is the
    (d, h, w) grid, packed or row-pitched [n, c, d, h, pitch]; ``addend`` (optional) has
    the padded shape [n, c, d+1, h+1, w+1] and v's dtype."""
    nat.require_device(v)
    n, c = int(v.shape[0]), int(v.shape[1])
    d, h, w = (int(s) for s in spatial)
    pitch = _row_pitch(v, w)
    out = torch.empty((n, c, d + 1, h + 1, w + 1), dtype=v.dtype, device=v.device)
    if addend is not None:
        if addend.shape != out.shape or addend.dtype != v.dtype:
            raise ValueError("addend must have the padded shape and v's dtype")
        addend = addend.contiguous()
    nat.check(
        nat.load().mednext_pad_front_add(
            v.data_ptr(), nat.ptr(addend), out.data_ptr(), n, c, d, h, w, pitch, nat.dtype_code(v.dtype), nat.stream(),
        ),
        "mednext_pad_front_add",
    )
    return out


def unpad_front(padded: Tensor, row_pitch: int = 0) -> Tensor:
    """``padded[:, :, 1:, 1:, 1:]`` as [n, c, d, h, row_pitch] (0: packed rows), zeros in
    the pad columns."""
    nat.require_device(padded)
    n, c = int(padded.shape[0]), int(padded.shape[1])
    d, h, w = (int(s) - 1 for s in padded.shape[2:])
    padded = padded.contiguous()
    v = torch.empty((n, c, d, h, int(row_pitch) if row_pitch else w), dtype=padded.dtype, device=padded.device)
    nat.check(
        nat.load().mednext_unpad_front(
            padded.data_ptr(), v.data_ptr(), n, c, d, h, w, int(row_pitch), nat.dtype_code(padded.dtype), nat.stream(),
        ),
        "mednext_unpad_front",
    )
    return v


def upsample2_fill(small: Tensor, bias: Tensor | None, row_pitch: int = 0) -> Tensor:
    """[n, c, 2d-1, 2h-1, row_pitch] (0: 2w-1) buffer holding small[m] at the all-even
    positions 2m, bias[c] elsewhere and zeros in the pad columns: the output of a
    1x1x1, stride-2 ConvTranspose3d whose per-voxel product (bias included) is
    ``small`` [n, c, d, h, w]."""
    nat.require_device(small)
    n, c, d, h, w = _dims(small)
    small = small.contiguous()
    big = torch.empty((n, c, 2 * d - 1, 2 * h - 1, int(row_pitch) if row_pitch else 2 * w - 1), dtype=small.dtype,
                      device=small.device)
    b = bias.float().contiguous() if bias is not None else None
    nat.check(
        nat.load().mednext_upsample2_fill(
            small.data_ptr(), nat.ptr(b), big.data_ptr(), n, c, d, h, w, int(row_pitch), nat.dtype_code(small.dtype),
            nat.stream(),
        ),
        "mednext_upsample2_fill",
    )
    return big


def _check_pair(a: Tensor, b: Tensor, names: str) -> None:
    if not (a.is_cuda and b.is_cuda):
        raise ValueError("CUDA tensors are required")
    if a.ndim != 5 or b.ndim != 5:
        raise ValueError(f"{names} must be NCDHW and C1KKK tensors")
    if not (a.is_contiguous() and b.is_contiguous()):
        raise ValueError("contiguous tensors are required")


def _check_block(block: int, name: str = "block") -> None:
    if block < 1 or block & (block - 1):
        raise ValueError(f"{name} must be a positive power of two")


def depthwise_input_grad(grad_output: Tensor, weight: Tensor, block: int = 256) -> Tensor:
    """Stride-1, same-padding depthwise dX for cubic odd kernels (reference
    ops/_triton/depthwise.py:271-302)."""
    _check_pair(grad_output, weight, "grad_output and weight")
    channels = grad_output.shape[1]
    if weight.shape[0] != channels or weight.shape[1] != 1 or len(set(weight.shape[2:])) != 1:
        raise ValueError("weight must have shape [C, 1, K, K, K]")
    kernel_size = int(weight.shape[2])
    _check_kernel(kernel_size)
    _check_block(block)
    return dw_dgrad(grad_output, weight, kernel_size)


def depthwise_stride2_input_grad(grad_output: Tensor, weight: Tensor, input_spatial_size, block: int = 256) -> Tensor:
    """Stride-2, same-padding depthwise Conv3d dX (reference lines 305-348)."""
    _check_pair(grad_output, weight, "grad_output and weight")
    if len(input_spatial_size) != 3:
        raise ValueError("input_spatial_size must contain D, H, and W")
    channels = grad_output.shape[1]
    if weight.shape[0] != channels or weight.shape[1] != 1 or len(set(weight.shape[2:])) != 1:
        raise ValueError("weight must have shape [C, 1, K, K, K]")
    kernel_size = int(weight.shape[2])
    _check_kernel(kernel_size)
    _check_block(block)
    size = tuple(int(v) for v in input_spatial_size)
    if tuple(grad_output.shape[2:]) != tuple((v + 1) // 2 for v in size):
        raise ValueError("grad_output shape does not match stride-two same padding")
    return s2_dgrad(grad_output, weight, size, kernel_size)


def depthwise_weight_grad(x: Tensor, grad_output: Tensor, splits: int = 64, block: int = 512, kernel_size: int = 3) -> Tensor:
    """Cubic odd-kernel depthwise dW, deterministic two-pass reduction
    (reference lines 351-390)."""
    if not (x.is_cuda and grad_output.is_cuda):
        raise ValueError("CUDA tensors are required")
    if x.shape != grad_output.shape or x.ndim != 5:
        raise ValueError("x and grad_output must have the same NCDHW shape")
    if not (x.is_contiguous() and grad_output.is_contiguous()):
        raise ValueError("contiguous NCDHW tensors are required")
    if splits < 1 or block < 1 or block & (block - 1):
        raise ValueError("splits must be positive and block must be a power of two")
    _check_kernel(kernel_size)
    return dw_wgrad(x, grad_output, kernel_size, want_bias=False)[0]


def depthwise_transpose_weight_grad(
    x: Tensor, grad_output: Tensor, splits: int = 64, block: int = 512, kernel_size: int = 3
) -> Tensor:
    """Stride-2, same-padding depthwise ConvTranspose3d dW (reference lines 393-442)."""
    if not (x.is_cuda and grad_output.is_cuda):
        raise ValueError("CUDA tensors are required")
    if x.ndim != 5 or grad_output.ndim != 5:
        raise ValueError("x and grad_output must be NCDHW tensors")
    if x.shape[:2] != grad_output.shape[:2]:
        raise ValueError("x and grad_output must have matching batch and channels")
    if not (x.is_contiguous() and grad_output.is_contiguous()):
        raise ValueError("contiguous NCDHW tensors are required")
    if splits < 1 or block < 1 or block & (block - 1):
        raise ValueError("splits must be positive and block must be a power of two")
    _check_kernel(kernel_size)
    if tuple(grad_output.shape[2:]) != tuple(2 * int(v) - 1 for v in x.shape[2:]):
        raise ValueError("grad_output must have spatial shape 2 * x.shape[2:] - 1")
    return t_wgrad(x, grad_output, kernel_size, want_bias=False)[0]


# --------------------------------------------------------------------------- custom ops
def _wshape(channels: int, k: int) -> tuple[int, int, int, int, int]:
    return (channels, 1, k, k, k)


@custom_op(f"{_NS}::depthwise_weight_grad_odd_regular", mutates_args=())
def depthwise_weight_grad_regular(
    x: Tensor, grad_output: Tensor, kernel_size: int, channels: int, spatial_size: int, splits: int, block: int
) -> Tensor:
    return dw_wgrad(x, grad_output, kernel_size, want_bias=False)[0]


@depthwise_weight_grad_regular.register_fake
def _(x, grad_output, kernel_size, channels, spatial_size, splits, block):
    return x.new_empty(_wshape(channels, kernel_size))


@custom_op(f"{_NS}::depthwise_bias_weight_grad_odd_regular", mutates_args=())
def depthwise_weight_bias_grad_regular(x: Tensor, grad_output: Tensor, kernel_size: int) -> tuple[Tensor, Tensor]:
    dw, db = dw_wgrad(x, grad_output, kernel_size, want_bias=True)
    return dw, db


@depthwise_weight_bias_grad_regular.register_fake
def _(x, grad_output, kernel_size):
    c = x.shape[1]
    return x.new_empty(_wshape(c, kernel_size)), x.new_empty((c,))


@custom_op(f"{_NS}::depthwise_input_grad_odd_regular", mutates_args=())
def depthwise_input_grad_regular(
    grad_output: Tensor, weight: Tensor, kernel_size: int, channels: int, spatial_size: int, block: int
) -> Tensor:
    return dw_dgrad(grad_output, weight, kernel_size)


@depthwise_input_grad_regular.register_fake
def _(grad_output, weight, kernel_size, channels, spatial_size, block):
    return torch.empty_like(grad_output)


@custom_op(f"{_NS}::depthwise_conv3d_odd_regular", mutates_args=())
def depthwise_conv3d_regular(
    x: Tensor,
    weight: Tensor,
    bias: Tensor | None,
    kernel_size: int,
    channels: int,
    spatial_size: int,
    dw_splits: int,
    dw_block: int,
    dx_block: int,
    custom_dx: bool = True,
    custom_dw: bool = True,
) -> Tensor:
    return dw_forward(x, weight, bias, kernel_size)


@depthwise_conv3d_regular.register_fake
def _(x, weight, bias, kernel_size, channels, spatial_size, dw_splits, dw_block, dx_block, custom_dx=True, custom_dw=True):
    return torch.empty_like(x)


def _setup_regular(ctx, inputs, output):
    x, weight, bias, kernel_size = inputs[:4]
    ctx.save_for_backward(x, weight)
    ctx.has_bias = bias is not None
    ctx.kernel_size = kernel_size


def _regular_backward(ctx, grad_output):
    x, weight = ctx.saved_tensors
    grad_output = grad_output.contiguous()
    need_dx, need_dw, need_db = ctx.needs_input_grad[:3]
    dx = dw = db = None
    if need_dx:
        dx = depthwise_input_grad_regular(grad_output, weight, ctx.kernel_size, int(x.shape[1]), int(x.shape[2]), 0)
    if need_dw or (need_db and ctx.has_bias):
        dw_all, db_all = depthwise_weight_bias_grad_regular(x, grad_output, ctx.kernel_size)
        dw = dw_all if need_dw else None
        db = db_all if (need_db and ctx.has_bias) else None
    return dx, dw, db, None, None, None, None, None, None, None, None


depthwise_conv3d_regular.register_autograd(_regular_backward, setup_context=_setup_regular)


@custom_op(f"{_NS}::depthwise_input_grad_stride2_regular", mutates_args=())
def depthwise_input_grad_stride2_regular(
    grad_output: Tensor, weight: Tensor, channels: int, spatial_size: int, block: int
) -> Tensor:
    return s2_dgrad(grad_output, weight, (spatial_size,) * 3, int(weight.shape[2]))


@depthwise_input_grad_stride2_regular.register_fake
def _(grad_output, weight, channels, spatial_size, block):
    return grad_output.new_empty((grad_output.shape[0], channels, spatial_size, spatial_size, spatial_size))


@custom_op(f"{_NS}::depthwise_weight_bias_grad_stride2_regular", mutates_args=())
def depthwise_weight_bias_grad_stride2(x: Tensor, grad_output: Tensor, kernel_size: int) -> tuple[Tensor, Tensor]:
    dw, db = s2_wgrad(x, grad_output, kernel_size, want_bias=True)
    return dw, db


@depthwise_weight_bias_grad_stride2.register_fake
def _(x, grad_output, kernel_size):
    c = x.shape[1]
    return x.new_empty(_wshape(c, kernel_size)), x.new_empty((c,))


@custom_op(f"{_NS}::depthwise_conv3d_stride2_regular", mutates_args=())
def depthwise_conv3d_stride2_regular(
    x: Tensor, weight: Tensor, bias: Tensor | None, kernel_size: int, channels: int, spatial_size: int, dx_block: int
) -> Tensor:
    return s2_forward(x, weight, bias, kernel_size)


@depthwise_conv3d_stride2_regular.register_fake
def _(x, weight, bias, kernel_size, channels, spatial_size, dx_block):
    s = (spatial_size + 1) // 2
    return x.new_empty((x.shape[0], channels, s, s, s))


def _setup_stride2(ctx, inputs, output):
    x, weight, bias, kernel_size, channels, spatial_size, dx_block = inputs
    ctx.save_for_backward(x, weight)
    ctx.has_bias = bias is not None
    ctx.kernel_size = kernel_size
    ctx.channels = channels
    ctx.spatial_size = spatial_size


def _stride2_backward(ctx, grad_output):
    x, weight = ctx.saved_tensors
    grad_output = grad_output.contiguous()
    need_dx, need_dw, need_db = ctx.needs_input_grad[:3]
    dx = dw = db = None
    if need_dx:
        dx = depthwise_input_grad_stride2_regular(grad_output, weight, ctx.channels, ctx.spatial_size, 0)
    if need_dw or (need_db and ctx.has_bias):
        dw_all, db_all = depthwise_weight_bias_grad_stride2(x, grad_output, ctx.kernel_size)
        dw = dw_all if need_dw else None
        db = db_all if (need_db and ctx.has_bias) else None
    return dx, dw, db, None, None, None, None


depthwise_conv3d_stride2_regular.register_autograd(_stride2_backward, setup_context=_setup_stride2)


@custom_op(f"{_NS}::depthwise_transpose_weight_grad_odd_regular", mutates_args=())
def depthwise_transpose_weight_grad_regular(
    x: Tensor, grad_output: Tensor, kernel_size: int, channels: int, spatial_size: int, splits: int, block: int
) -> Tensor:
    return t_wgrad(x, grad_output, kernel_size, want_bias=False)[0]


@depthwise_transpose_weight_grad_regular.register_fake
def _(x, grad_output, kernel_size, channels, spatial_size, splits, block):
    return x.new_empty(_wshape(channels, kernel_size))


@custom_op(f"{_NS}::depthwise_transpose_weight_bias_grad", mutates_args=())
def depthwise_transpose_weight_bias_grad(x: Tensor, grad_output: Tensor, kernel_size: int) -> tuple[Tensor, Tensor]:
    dw, db = t_wgrad(x, grad_output, kernel_size, want_bias=True)
    return dw, db


@depthwise_transpose_weight_bias_grad.register_fake
def _(x, grad_output, kernel_size):
    c = x.shape[1]
    return x.new_empty(_wshape(c, kernel_size)), x.new_empty((c,))


@custom_op(f"{_NS}::depthwise_transpose_input_grad", mutates_args=())
def depthwise_transpose_input_grad(grad_output: Tensor, weight: Tensor, kernel_size: int) -> Tensor:
    return t_dgrad(grad_output, weight, kernel_size)


@depthwise_transpose_input_grad.register_fake
def _(grad_output, weight, kernel_size):
    n, c, od, oh, ow = grad_output.shape
    return grad_output.new_empty((n, c, (od + 1) // 2, (oh + 1) // 2, (ow + 1) // 2))


@custom_op(f"{_NS}::depthwise_conv_transpose3d_odd_regular", mutates_args=())
def depthwise_conv_transpose3d_regular(
    x: Tensor, weight: Tensor, bias: Tensor | None, kernel_size: int, channels: int, spatial_size: int,
    dw_splits: int, dw_block: int,
) -> Tensor:
    return t_forward(x, weight, bias, kernel_size)


@depthwise_conv_transpose3d_regular.register_fake
def _(x, weight, bias, kernel_size, channels, spatial_size, dw_splits, dw_block):
    s = 2 * spatial_size - 1
    return x.new_empty((x.shape[0], channels, s, s, s))


def _setup_transpose(ctx, inputs, output):
    x, weight, bias, kernel_size = inputs[:4]
    ctx.save_for_backward(x, weight)
    ctx.has_bias = bias is not None
    ctx.kernel_size = kernel_size


def _transpose_backward(ctx, grad_output):
    x, weight = ctx.saved_tensors
    grad_output = grad_output.contiguous()
    need_dx, need_dw, need_db = ctx.needs_input_grad[:3]
    dx = dw = db = None
    if need_dx:
        dx = depthwise_transpose_input_grad(grad_output, weight, ctx.kernel_size)
    if need_dw or (need_db and ctx.has_bias):
        dw_all, db_all = depthwise_transpose_weight_bias_grad(x, grad_output, ctx.kernel_size)
        dw = dw_all if need_dw else None
        db = db_all if (need_db and ctx.has_bias) else None
    return dx, dw, db, None, None, None, None, None


depthwise_conv_transpose3d_regular.register_autograd(_transpose_backward, setup_context=_setup_transpose)

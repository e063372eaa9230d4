"""MedNeXt v2 Global Response Norm on the sm_100a kernels.

The public surface mirrors the reference's ops/grn.py and ops/_triton/grn.py:

* :func:`global_response_norm3d_reference` — the formula in PyTorch operations
  (ops/grn.py:16-29), the reference path;
* :class:`GlobalResponseNorm3d` — the layer with zero-initialised ``gamma`` and
  ``beta`` of shape (1, C, 1, 1, 1) (ops/grn.py:32-46), so state dicts match;
* :func:`fused_global_response_norm3d` — the fused training op with the same
  argument checks and messages as the reference's (ops/_triton/grn.py:405-438),
  served by ``mednext_grn_fwd`` / ``mednext_grn_bwd`` of the C ABI;
* :class:`AdaptiveGlobalResponseNorm3d` and :func:`install_adaptive_grn` — the
  policy-selected wrapper (ops/grn.py:49-111): training steps on CUDA whose
  decision is an sm_100a GRN id run the fused op, everything else the reference
  formula.

The op ``mednext_accel_b200::grn_forward`` returns (y, norm, den) like the
reference's ``mednext_accel::grn_forward``; its autograd saves x, gamma, norm and
den, and the backward is one ``mednext_grn_bwd`` call (dx, dgamma, dbeta).
"""

from __future__ import annotations

import math
from dataclasses import replace

import torch
from torch import Tensor, nn
from torch.library import custom_op

from . import _native as nat
from .adaptive import ModelOptimizationContext, _context_from_tensor
from .optimization import OperatorDescriptor, PolicyResolver

_NS = "mednext_accel_b200"
GRN_IMPLEMENTATIONS = ("sm100_grn", "triton_fused_grn")


def global_response_norm3d_reference(x: Tensor, gamma: Tensor, beta: Tensor, eps: float = 1e-6) -> Tensor:
    """GRN in PyTorch operations: 16-bit inputs computed in fp32, one final cast."""
    if x.ndim != 5:
        raise ValueError("GRN expects an NCDHW tensor")
    work = x.float() if x.dtype in (torch.float16, torch.bfloat16) else x
    norm = torch.linalg.vector_norm(work, dim=(2, 3, 4), keepdim=True)
    ratio = norm / (norm.sum(dim=1, keepdim=True) + eps)
    out = work + gamma.to(work.dtype) * work * ratio + beta.to(work.dtype)
    return out.to(x.dtype)


class GlobalResponseNorm3d(nn.Module):
    """GRN layer; ``gamma`` and ``beta`` start at zero, so it starts as the identity."""

    def __init__(self, channels: int, eps: float = 1e-6) -> None:
        super().__init__()
        if channels <= 0:
            raise ValueError("channels must be positive")
        if not (math.isfinite(eps) and eps > 0):
            raise ValueError("eps must be finite and positive")
        self.eps = eps
        self.gamma = nn.Parameter(torch.zeros(1, channels, 1, 1, 1))
        self.beta = nn.Parameter(torch.zeros(1, channels, 1, 1, 1))

    def forward(self, x: Tensor) -> Tensor:
        return global_response_norm3d_reference(x, self.gamma, self.beta, self.eps)


def _dims(x: Tensor) -> tuple[int, int, int]:
    return int(x.shape[0]), int(x.shape[1]), int(x.shape[2] * x.shape[3] * x.shape[4])


@custom_op(f"{_NS}::grn_forward", mutates_args=())
def grn_forward(x: Tensor, gamma: Tensor, beta: Tensor, eps: float) -> tuple[Tensor, Tensor, Tensor]:
    """(y, norm [N, C] fp32, den [N] fp32) on the sm_100a kernels."""
    nat.require_device(x)
    lib = nat.load()
    n, c, v = _dims(x)
    code = nat.dtype_code(x.dtype)
    y = torch.empty_like(x)
    norm = torch.empty((n, c), dtype=torch.float32, device=x.device)
    den = torch.empty((n,), dtype=torch.float32, device=x.device)
    ws = nat.workspace(lib.mednext_grn_workspace_size(n, c, v, code), x.device)
    nat.check(
        lib.mednext_grn_fwd(x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), y.data_ptr(), norm.data_ptr(),
                            den.data_ptr(), ws.data_ptr(), ws.numel(), n, c, v, float(eps), code, nat.stream()),
        "mednext_grn_fwd",
    )
    return y, norm, den


@grn_forward.register_fake
def _(x, gamma, beta, eps):
    return (torch.empty_like(x), x.new_empty(x.shape[:2], dtype=torch.float32),
            x.new_empty((x.shape[0],), dtype=torch.float32))


@custom_op(f"{_NS}::grn_backward", mutates_args=())
def grn_backward(dy: Tensor, x: Tensor, gamma: Tensor, norm: Tensor, den: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """(dx, dgamma, dbeta); dgamma and dbeta have gamma's (1, C, 1, 1, 1) shape, fp32."""
    nat.require_device(x)
    lib = nat.load()
    n, c, v = _dims(x)
    code = nat.dtype_code(x.dtype)
    dx = torch.empty_like(x)
    dgamma = torch.empty_like(gamma)
    dbeta = torch.empty_like(gamma)
    ws = nat.workspace(lib.mednext_grn_workspace_size(n, c, v, code), x.device)
    nat.check(
        lib.mednext_grn_bwd(dy.data_ptr(), x.data_ptr(), gamma.data_ptr(), norm.data_ptr(), den.data_ptr(),
                            dx.data_ptr(), dgamma.data_ptr(), dbeta.data_ptr(), ws.data_ptr(), ws.numel(), n, c, v,
                            code, nat.stream()),
        "mednext_grn_bwd",
    )
    return dx, dgamma, dbeta


@grn_backward.register_fake
def _(dy, x, gamma, norm, den):
    return torch.empty_like(x), torch.empty_like(gamma), torch.empty_like(gamma)


def _setup(ctx, inputs, output):
    x, gamma, _beta, _eps = inputs
    _y, norm, den = output
    ctx.save_for_backward(x, gamma, norm, den)
    ctx.mark_non_differentiable(norm, den)
    ctx.set_materialize_grads(False)


def _backward(ctx, dy, _dnorm, _dden):
    if dy is None:
        return None, None, None, None
    x, gamma, norm, den = ctx.saved_tensors
    dx, dgamma, dbeta = grn_backward(dy.contiguous(), x, gamma, norm, den)
    need = ctx.needs_input_grad
    return (dx if need[0] else None, dgamma if need[1] else None, dbeta if need[2] else None, None)


grn_forward.register_autograd(_backward, setup_context=_setup)


def fused_global_response_norm3d(x: Tensor, gamma: Tensor, beta: Tensor, eps: float = 1e-6) -> Tensor:
    """GRN on the sm_100a kernels; unsupported direct calls raise instead of
    falling back (the reference's contract, ops/_triton/grn.py:405-438).  Besides
    the reference's float16 / bfloat16 inputs, float32 inputs are accepted too."""
    if x.ndim != 5:
        raise ValueError("fused GRN expects a rank-5 NCDHW input")
    if not (x.is_cuda and gamma.is_cuda and beta.is_cuda):
        raise ValueError("fused GRN requires CUDA tensors")
    if gamma.device != x.device or beta.device != x.device:
        raise ValueError("fused GRN requires all tensors on the same CUDA device")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError("fused GRN requires a float16, bfloat16 or float32 input")
    if not x.is_contiguous():
        raise ValueError("fused GRN requires a contiguous NCDHW input")
    if any(size == 0 for size in x.shape):
        raise ValueError("fused GRN requires nonempty input dimensions")
    if gamma.dtype != torch.float32 or beta.dtype != torch.float32:
        raise ValueError("fused GRN requires float32 gamma and beta")
    expected = (1, x.shape[1], 1, 1, 1)
    if tuple(gamma.shape) != expected or tuple(beta.shape) != expected:
        raise ValueError("fused GRN requires gamma and beta with shape (1, C, 1, 1, 1)")
    if not (gamma.is_contiguous() and beta.is_contiguous()):
        raise ValueError("fused GRN requires contiguous gamma and beta")
    if not (math.isfinite(eps) and eps > 0):
        raise ValueError("fused GRN requires eps to be finite and positive")
    return grn_forward(x, gamma, beta, float(eps))[0]


class AdaptiveGlobalResponseNorm3d(nn.Module):
    """Policy-selected GRN: training steps the resolver assigns to an sm_100a GRN
    id run :func:`fused_global_response_norm3d`; inference, no-grad calls and
    other decisions run the reference formula.  Keeps the wrapped layer's
    Parameter objects."""

    def __init__(self, module: GlobalResponseNorm3d, resolver: PolicyResolver,
                 model_context: ModelOptimizationContext, role: str | None = None) -> None:
        super().__init__()
        self.gamma = module.gamma
        self.beta = module.beta
        self.eps = module.eps
        self.resolver = resolver
        self.model_context = model_context
        self.descriptor = OperatorDescriptor.normalization(family="global_response_norm3d",
                                                           channels=int(self.gamma.shape[1]), role=role)
        self.train(module.training)

    def _reference(self, x: Tensor) -> Tensor:
        return global_response_norm3d_reference(x, self.gamma, self.beta, self.eps)

    def forward(self, x: Tensor) -> Tensor:
        if not self.training or not torch.is_grad_enabled() or x.ndim != 5:
            return self._reference(x)
        # GRN runs on its input's dtype: autocast does not cast it
        context = replace(_context_from_tensor(x, self.model_context, training=True),
                          dtype=str(x.dtype).split(".")[-1])
        decision = self.resolver.resolve(self.descriptor, context, "training")
        if decision.implementation not in GRN_IMPLEMENTATIONS or not x.is_contiguous():
            return self._reference(x)
        return fused_global_response_norm3d(x, self.gamma, self.beta, self.eps)


def install_adaptive_grn(model: nn.Module, *, resolver: PolicyResolver, model_context: ModelOptimizationContext,
                         _prefix: str = "") -> int:
    """Wrap every GlobalResponseNorm3d child of ``model``; returns how many."""
    count = 0
    for name, child in list(model.named_children()):
        role = f"{_prefix}.{name}" if _prefix else name
        if type(child) is GlobalResponseNorm3d:
            setattr(model, name, AdaptiveGlobalResponseNorm3d(child, resolver, model_context, role))
            count += 1
        else:
            count += install_adaptive_grn(child, resolver=resolver, model_context=model_context, _prefix=role)
    return count

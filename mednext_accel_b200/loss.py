"""Mean cross-entropy on the native kernels: the training step's deep-supervision
loss (reference ``benchmarks/implementations.py:133-190``: five heads, each
``F.cross_entropy(head, target)``).

``cross_entropy(logits, target)`` is a drop-in for ``F.cross_entropy`` with
``reduction="mean"`` on [N, K, *spatial] logits and [N, *spatial] int64 targets.
It computes in fp32 from the stored logits (bf16 under autocast, as autocast's fp32
cast of the logits would) and returns the fp32 loss; the logits' grad comes back in
their own dtype.  Forward is one pass (log-sum-exp and target logit per voxel,
deterministic block partials) and backward one pass (softmax minus one-hot, scaled
on the device by grad / count), both graph-capturable.  Inputs it does not cover fall
back to ``F.cross_entropy``.
"""

from __future__ import annotations

import torch
from torch import Tensor
from torch.library import custom_op
from torch.nn import functional as F

from . import _native as nat

_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


def _dims(logits: Tensor) -> tuple[int, int, int]:
    n, k = int(logits.shape[0]), int(logits.shape[1])
    v = 1
    for s in logits.shape[2:]:
        v *= int(s)
    return n, k, v


@custom_op("mednext_accel_b200::cross_entropy_mean", mutates_args=())
def cross_entropy_mean(logits: Tensor, target: Tensor, ignore_index: int) -> Tensor:
    """[mean loss, number of counted targets] (fp32, on the logits' device)."""
    lib = nat.load()
    n, k, v = _dims(logits)
    out = torch.empty(2, dtype=torch.float32, device=logits.device)
    ws = nat.workspace(lib.mednext_ce_workspace_size(n, k, v), logits.device)
    nat.check(
        lib.mednext_ce_fwd(logits.data_ptr(), target.data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel(), n, k, v,
                           int(ignore_index), nat.dtype_code(logits.dtype), nat.stream()),
        "mednext_ce_fwd",
    )
    return out


@cross_entropy_mean.register_fake
def _(logits, target, ignore_index):
    return logits.new_empty((2,), dtype=torch.float32)


def _setup(ctx, inputs, output):
    logits, target, ignore_index = inputs
    ctx.save_for_backward(logits, target, output)
    ctx.ignore_index = int(ignore_index)


def _backward(ctx, grad):
    logits, target, out = ctx.saved_tensors
    n, k, v = _dims(logits)
    dlogits = torch.empty_like(logits)
    g = grad.float().contiguous()  # grad[0] is d(mean loss); grad[1] (the count) has no effect
    nat.check(
        nat.load().mednext_ce_bwd(logits.data_ptr(), target.data_ptr(), out.data_ptr(), g.data_ptr(),
                                  dlogits.data_ptr(), n, k, v, ctx.ignore_index, nat.dtype_code(logits.dtype),
                                  nat.stream()),
        "mednext_ce_bwd",
    )
    return dlogits, None, None


cross_entropy_mean.register_autograd(_backward, setup_context=_setup)


def cross_entropy(logits: Tensor, target: Tensor, ignore_index: int = -100) -> Tensor:
    """``F.cross_entropy(logits, target, ignore_index=ignore_index)`` (mean reduction)."""
    if (
        logits.is_cuda and logits.ndim >= 2 and logits.dtype in _DTYPES and logits.is_contiguous()
        and target.dtype == torch.int64 and target.is_contiguous() and target.device == logits.device
        and tuple(target.shape) == (logits.shape[0], *logits.shape[2:])
    ):
        return cross_entropy_mean(logits, target, ignore_index)[0]
    return F.cross_entropy(logits, target, ignore_index=ignore_index)

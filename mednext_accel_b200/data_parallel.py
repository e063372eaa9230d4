"""Batch-sharded data parallelism: bucketed gradient all-reduce overlapped with backward.

The reference has no distributed code; MedNeXt training shards naturally over
the batch, so the only exchange per step is the average of the parameter
gradients.  Design (one process per GPU, ``torch.distributed`` with NCCL):

* parameters are grouped, in reverse registration order (roughly the order
  their gradients become final during backward), into flat fp32 buckets of
  about ``bucket_cap_mb``;
* :meth:`GradientBucketReducer.zero_grad` sets every ``param.grad`` to None, so
  autograd stores each gradient as produced (no per-parameter accumulation
  kernel); a post-accumulate-grad hook counts the parameters of each bucket, and
  when a bucket is complete one multi-tensor copy gathers its gradients into the
  flat buffer, whose all-reduce (``ReduceOp.AVG``) is issued on a dedicated
  communication stream that first waits for the compute stream, so early
  buckets (the wide pointwise weights of the decoder) travel under the remaining
  backward; each ``param.grad`` then becomes a view of the reduced buffer;
* :meth:`GradientBucketReducer.finish` makes the compute stream wait for the
  communication stream before the optimizer step.
* With a single process the reducer does nothing beyond ``zero_grad``.

Every rank issues the same collectives in the same order (buckets complete in a
deterministic order because backward is deterministic), which is required for
NCCL and for CUDA-graph capture of the whole step.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.distributed as dist
from torch import nn


@dataclass(eq=False)
class _Bucket:
    params: list[nn.Parameter]
    buffer: torch.Tensor
    index: int = 0
    pending: int = 0
    launched: bool = False
    works: list = field(default_factory=list)


class GradientBucketReducer:
    def __init__(self, model: nn.Module, *, bucket_cap_mb: float = 25.0, group=None, stream: torch.cuda.Stream | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        params = [p for p in model.parameters() if p.requires_grad]
        cap = int(bucket_cap_mb * 2**20 / 4)
        self.buckets: list[_Bucket] = []
        current: list[nn.Parameter] = []
        size = 0
        for p in reversed(params):
            current.append(p)
            size += p.numel()
            if size >= cap:
                self.buckets.append(self._make(current))
                current, size = [], 0
        if current:
            self.buckets.append(self._make(current))
        self.owner = {}
        for i, b in enumerate(self.buckets):
            b.index = i
            for p in b.params:
                self.owner[p] = i
        device = params[0].device
        self.stream = stream or (torch.cuda.Stream(device=device) if device.type == "cuda" else None)
        # NCCL averages in the collective; gloo (CPU tests) has no AVG, so sum and scale
        self.native_avg = (not dist.is_initialized()) or dist.get_backend(group) == "nccl"
        # one process: nothing to reduce, gradients stay where autograd puts them
        self.handles = [p.register_post_accumulate_grad_hook(self._hook) for p in params] if self.world > 1 else []
        self.order: list[int] = []

    @staticmethod
    def _make(params: list[nn.Parameter]) -> _Bucket:
        for p in params:
            if p.dtype != torch.float32:
                raise ValueError("gradient buckets hold fp32 parameters")
        total = sum(p.numel() for p in params)
        buf = torch.zeros(total, dtype=torch.float32, device=params[0].device)
        return _Bucket(params, buf, pending=len(params))

    def _views(self, b: _Bucket) -> list[torch.Tensor]:
        out, offset = [], 0
        for p in b.params:
            out.append(b.buffer[offset : offset + p.numel()].view_as(p))
            offset += p.numel()
        return out

    def zero_grad(self) -> None:
        """Drop the gradients: autograd stores the next ones without accumulation."""
        for b in self.buckets:
            for p in b.params:
                p.grad = None
            b.pending = len(b.params)
            b.launched = False
        self.order.clear()

    def _hook(self, p: nn.Parameter) -> None:
        b = self.buckets[self.owner[p]]
        b.pending -= 1
        if b.pending == 0:
            self._launch(b)

    def _launch(self, b: _Bucket) -> None:
        if b.launched:
            return
        b.launched = True
        self.order.append(b.index)
        if self.world == 1:
            return
        views = self._views(b)
        have = [(v, p.grad) for v, p in zip(views, b.params, strict=True) if p.grad is not None]
        for v, p in zip(views, b.params, strict=True):
            if p.grad is None:
                v.zero_()  # no gradient this step (unused parameter)
        if have:
            torch._foreach_copy_([v for v, _ in have], [g for _, g in have])
        if self.stream is None:
            self._all_reduce_mean(b.buffer)
        else:
            self.stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self.stream):
                self._all_reduce_mean(b.buffer)
        for v, p in zip(views, b.params, strict=True):
            p.grad = v

    def _all_reduce_mean(self, buf: torch.Tensor) -> None:
        if self.native_avg:
            dist.all_reduce(buf, op=dist.ReduceOp.AVG, group=self.group)
        else:
            dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.group)
            buf.div_(self.world)

    def finish(self) -> None:
        """Launch buckets whose parameters got no gradient and join the comm stream."""
        for b in self.buckets:
            if not b.launched:
                self._launch(b)
        if self.stream is not None and self.world > 1:
            torch.cuda.current_stream().wait_stream(self.stream)

    def remove(self) -> None:
        for h in self.handles:
            h.remove()
        self.handles.clear()


def broadcast_parameters(model: nn.Module, src: int = 0, group=None) -> None:
    """Make every rank start from rank ``src``'s weights."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    with torch.no_grad():
        for t in list(model.parameters()) + list(model.buffers()):
            dist.broadcast(t.data, src=src, group=group)

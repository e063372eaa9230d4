"""Batch-sharded data parallelism: bucketed gradient all-reduce overlapped with backward.

The reference has no distributed code; MedNeXt training shards naturally over
the batch, so the only exchange per step is the average of the parameter
gradients.  Design (one process per GPU, ``torch.distributed`` with NCCL):

* parameters are packed, in reverse registration order (roughly the order their
  gradients become final during backward), into flat fp32 buckets of about
  ``bucket_cap_mb``; every ``param.grad`` is a view into its bucket, so no copy
  is needed before or after the collective;
* a post-accumulate-grad hook counts the parameters of each bucket; when a
  bucket is complete its all-reduce (``ReduceOp.AVG``) is issued on a dedicated
  communication stream that first waits for the compute stream, so the
  transfer of early buckets (the wide pointwise weights of the decoder) runs
  under the remaining backward;
* :meth:`GradientBucketReducer.finish` makes the compute stream wait for the
  communication stream before the optimizer step.

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
        self.handles = [p.register_post_accumulate_grad_hook(self._hook) for p in params]
        self.order: list[int] = []

    @staticmethod
    def _make(params: list[nn.Parameter]) -> _Bucket:
        total = sum(p.numel() for p in params)
        buf = torch.zeros(total, dtype=torch.float32, device=params[0].device)
        offset = 0
        for p in params:
            if p.dtype != torch.float32:
                raise ValueError("gradient buckets hold fp32 parameters")
            p.grad = buf[offset : offset + p.numel()].view_as(p)
            offset += p.numel()
        return _Bucket(params, buf, pending=len(params))

    def zero_grad(self) -> None:
        """Zero the buckets in place (grads stay views into them)."""
        for b in self.buckets:
            b.buffer.zero_()
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
        if self.stream is None:
            self._all_reduce_mean(b.buffer)
            return
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            self._all_reduce_mean(b.buffer)

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

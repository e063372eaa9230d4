"""Functional CPU restatement of the reference MedNeXt v1 training step —
TEST/BASELINE INFRASTRUCTURE ONLY (imported by tests and by bench.py's CPU
baseline leg, never by the product).

It evaluates the reference's pure-PyTorch algorithm from a parameter mapping
with the same keys as the reference ``state_dict``:
stem 1x1 conv; per block depthwise conv -> GroupNorm(C, C) -> 1x1 expand ->
exact GELU -> 1x1 project (+ residual) (models/blocks.py:47-91); down blocks
with a stride-2 depthwise conv and a strided 1x1 residual conv (blocks.py:94-136);
up blocks with a stride-2 transposed depthwise conv, transposed 1x1 residual
conv and a one-voxel left pad (blocks.py:139-182); transposed 1x1 output heads
(blocks.py:185-194); the U-Net wiring and deep supervision of
models/mednext_v1.py:187-223; the five-head mean cross-entropy and AdamW step of
benchmarks/implementations.py:140-164.
"""

from __future__ import annotations

import re

import torch
from torch.nn import functional as F

BLOCK_COUNTS = {"small": (2,) * 9, "base": (2,) * 9, "medium": (3, 4, 4, 4, 4, 4, 4, 4, 3),
                "large": (3, 4, 8, 8, 8, 8, 8, 4, 3)}


def _block(p: dict, pre: str, x: torch.Tensor, kind: str, k: int, residual: bool) -> torch.Tensor:
    w = p[pre + "depthwise.weight"]
    b = p[pre + "depthwise.bias"]
    c = w.shape[0]
    if kind == "regular":
        t = F.conv3d(x, w, b, padding=k // 2, groups=c)
    elif kind == "down":
        t = F.conv3d(x, w, b, stride=2, padding=k // 2, groups=c)
    else:
        t = F.conv_transpose3d(x, w, b, stride=2, padding=k // 2, groups=c)
    z = F.group_norm(t, c, p[pre + "norm.weight"], p[pre + "norm.bias"], 1e-5)
    u = F.conv3d(z, p[pre + "expand.weight"], p[pre + "expand.bias"])
    y = F.conv3d(F.gelu(u), p[pre + "project.weight"], p[pre + "project.bias"])
    if kind == "regular":
        return y + x if residual else y
    rw, rb = p.get(pre + "residual.weight"), p.get(pre + "residual.bias")
    if kind == "down":
        return y + F.conv3d(x, rw, rb, stride=2) if rw is not None else y
    out = y + F.conv_transpose3d(x, rw, rb, stride=2) if rw is not None else y
    return F.pad(out, (1, 0) * 3)


def forward(p: dict, x: torch.Tensor, variant: str, k: int, deep_supervision: bool = True) -> list[torch.Tensor]:
    counts = BLOCK_COUNTS[variant]
    x = F.conv3d(x, p["stem.weight"], p["stem.bias"])
    skips = []
    for s in range(4):
        for j in range(counts[s]):
            x = _block(p, f"encoder_stages.{s}.{j}.", x, "regular", k, True)
        skips.append(x)
        x = _block(p, f"downsamples.{s}.", x, "down", k, False)
    for j in range(counts[4]):
        x = _block(p, f"bottleneck.{j}.", x, "regular", k, True)
    aux = []
    for i in range(4):
        s = 3 - i
        if deep_supervision:
            aux.append(F.conv_transpose3d(x, p[f"deep_supervision_heads.{i}.conv.weight"],
                                          p[f"deep_supervision_heads.{i}.conv.bias"]))
        x = _block(p, f"upsamples.{i}.", x, "up", k, False) + skips[s]
        for j in range(counts[8 - s]):
            x = _block(p, f"decoder_stages.{i}.{j}.", x, "regular", k, True)
    primary = F.conv_transpose3d(x, p["head.conv.weight"], p["head.conv.bias"])
    return [primary, *reversed(aux)] if deep_supervision else [primary]


def targets_for(target: torch.Tensor, heads: list[torch.Tensor]) -> list[torch.Tensor]:
    out = []
    for h in heads:
        if h.shape[2:] == target.shape[1:]:
            out.append(target)
        else:
            out.append(F.interpolate(target[:, None].float(), size=h.shape[2:], mode="nearest")[:, 0].long())
    return out


def loss_fn(heads: list[torch.Tensor], targets: list[torch.Tensor]) -> torch.Tensor:
    # fp64 heads stay fp64 (golden-vector checks); anything narrower is taken to fp32
    return sum(F.cross_entropy(h if h.dtype == torch.float64 else h.float(), t)
               for h, t in zip(heads, targets, strict=True)) / len(heads)


class ReferenceTrainer:
    """One MedNeXt training step on CPU (fp32): forward, five-head mean CE,
    backward, AdamW (benchmarks/implementations.py:153-164)."""

    def __init__(self, state: dict[str, torch.Tensor], variant: str = "base", k: int = 3, lr: float = 1e-4):
        self.params = {name: v.detach().float().clone().requires_grad_() for name, v in state.items()
                       if not re.search(r"(running_|num_batches)", name)}
        self.variant = variant
        self.k = k
        self.opt = torch.optim.AdamW(self.params.values(), lr=lr)

    def step(self, x: torch.Tensor, targets: list[torch.Tensor]) -> float:
        self.opt.zero_grad(set_to_none=True)
        heads = forward(self.params, x, self.variant, self.k)
        loss = loss_fn(heads, targets)
        loss.backward()
        self.opt.step()
        return float(loss.detach())

"""MedNeXt v1 network with the reference package's parameter schema.

The module tree (``stem``, ``encoder_stages.i.j.{depthwise,norm,expand,project}``,
``downsamples.i.residual``, ``bottleneck``, ``upsamples``, ``decoder_stages``,
``head.conv``, ``deep_supervision_heads.i.conv``) and every parameter shape match
the reference (models/blocks.py:47-194, models/mednext_v1.py:36-223,
models/config.py:11-98), so ``state_dict`` keys, checkpoints and optimizers are
interchangeable.  What differs is execution: once
:func:`mednext_accel_b200.adaptive.install_adaptive_operators` has run, a
MedNeXt block executes as one fused sm_100a operator (depthwise conv with
GroupNorm statistics, tensor-core expand with GroupNorm applied on load, GELU,
tensor-core compress with the residual added in the epilogue) instead of six
separate PyTorch modules.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass
from os import PathLike
from typing import Literal, TypeAlias

import torch
from torch import Tensor, nn
from torch.nn import functional as F
from torch.utils.checkpoint import checkpoint

DeepSupervisionOutput = Literal["tuple", "list", "stacked"]
OptimizationSource: TypeAlias = Literal["auto", "reference"] | str | PathLike[str] | Mapping[str, object]

# Published variants (reference models/config.py:11-23).
BLOCK_COUNTS: dict[str, tuple[int, ...]] = {
    "small": (2,) * 9,
    "base": (2,) * 9,
    "medium": (3, 4, 4, 4, 4, 4, 4, 4, 3),
    "large": (3, 4, 8, 8, 8, 8, 8, 4, 3),
}
EXPANSION_RATIOS: dict[str, tuple[int, ...]] = {
    "small": (2,) * 9,
    "base": (2, 3, 4, 4, 4, 4, 4, 3, 2),
    "medium": (2, 3, 4, 4, 4, 4, 4, 3, 2),
    "large": (3, 4, 8, 8, 8, 8, 8, 4, 3),
}


def _canonical_stages(stages: object) -> tuple[int, ...]:
    """Sorted tuple of distinct resolution-stage indices in 0..4; ValueError otherwise."""
    values = tuple(stages)  # type: ignore[arg-type]
    if len(values) == 0:
        raise ValueError("stages: give at least one stage, or None for every stage")
    if not all(type(v) is int for v in values):
        raise ValueError(f"stages: expected integers, got {values!r}")
    if len(set(values)) < len(values):
        raise ValueError(f"stages: duplicates are not allowed, got {values!r}")
    if not all(0 <= v <= 4 for v in values):
        raise ValueError(f"stages: every stage must be between 0 and 4 (the five resolutions), got {values!r}")
    return tuple(sorted(values))


@dataclass(frozen=True, slots=True)
class CheckpointConfig:
    """Activation checkpointing for MedNeXt.

    ``style="expansion"`` recomputes each block's expanded branch (expand, GELU,
    compress) in backward; ``style="block"`` recomputes whole blocks.  ``stages``
    names the resolution stages 0..4 it applies to (None: all of them).  Same
    public fields and meaning as the reference's checkpointing.py:11-48."""

    style: Literal["expansion", "block"] = "expansion"
    stages: tuple[int, ...] | None = None

    def __post_init__(self) -> None:
        if self.style not in _CHECKPOINT_STYLES:
            raise ValueError(f"style: unknown checkpointing style {self.style!r} "
                             f"(expected {' or '.join(_CHECKPOINT_STYLES)})")
        if self.stages is not None:
            object.__setattr__(self, "stages", _canonical_stages(self.stages))

    def includes(self, stage: int) -> bool:
        return True if self.stages is None else stage in self.stages

    @property
    def checkpoints_expansion(self) -> bool:
        return self.style == "expansion"

    @property
    def checkpoints_blocks(self) -> bool:
        return self.style == "block"


_CHECKPOINT_STYLES = ("expansion", "block")


@dataclass(frozen=True, slots=True)
class MedNeXtV1Config:
    """Architecture of one MedNeXt v1 network (the reference's models/config.py
    fields, so configs serialise the same way)."""

    variant: str
    spatial_dims: Literal[2, 3]
    in_channels: int
    out_channels: int
    kernel_size: int
    base_channels: int
    block_counts: tuple[int, ...]
    expansion_ratios: tuple[int, ...]
    downsample_expansion_ratios: tuple[int, ...]
    compatibility: Literal["official", "monai"]
    residual_blocks: bool = True
    residual_resampling: bool = True
    deep_supervision: bool = False

    def __post_init__(self) -> None:
        rules = (
            (self.spatial_dims in (2, 3), "spatial_dims must be 2 or 3"),
            (min(self.in_channels, self.out_channels) > 0, "in_channels and out_channels must be positive"),
            (self.base_channels > 0, "base_channels must be positive"),
            (self.kernel_size > 0 and self.kernel_size % 2 == 1, "kernel_size must be a positive odd integer"),
            (len(self.block_counts) == 9, "block_counts needs one entry per stage (nine stages)"),
            (len(self.expansion_ratios) == 9, "expansion_ratios needs one entry per stage (nine stages)"),
            (len(self.downsample_expansion_ratios) == 4,
             "downsample_expansion_ratios needs one entry per down block (four)"),
        )
        for ok, message in rules:
            if not ok:
                raise ValueError(message)


def get_mednext_v1_config(
    variant: str,
    *,
    in_channels: int,
    out_channels: int,
    spatial_dims: Literal[2, 3] = 3,
    kernel_size: int = 3,
    base_channels: int = 32,
    deep_supervision: bool = False,
    compatibility: Literal["official", "monai"] = "official",
) -> MedNeXtV1Config:
    """The published variant ``small`` / ``base`` / ``medium`` / ``large``."""
    key = variant.lower()
    counts = BLOCK_COUNTS.get(key)
    if counts is None:
        raise ValueError(f"unknown MedNeXt v1 variant {variant!r}; known variants: {', '.join(BLOCK_COUNTS)}")
    ratios = EXPANSION_RATIOS[key]
    # Which stage's ratio a down block uses is where the two published
    # implementations differ: the official code takes the ratio of the stage it
    # leads into (i + 1), MONAI the ratio of the stage it leaves (i).
    offsets = {"official": 1, "monai": 0}
    if compatibility not in offsets:
        raise ValueError(f"compatibility must be one of {', '.join(offsets)}, got {compatibility!r}")
    first = offsets[compatibility]
    return MedNeXtV1Config(
        variant=key, spatial_dims=spatial_dims, in_channels=in_channels, out_channels=out_channels,
        kernel_size=kernel_size, base_channels=base_channels, block_counts=counts, expansion_ratios=ratios,
        downsample_expansion_ratios=tuple(ratios[first:first + 4]), compatibility=compatibility,
        deep_supervision=deep_supervision,
    )


def _conv(spatial_dims: int) -> type[nn.Module]:
    if spatial_dims not in (2, 3):
        raise ValueError("spatial_dims must be 2 or 3")
    return nn.Conv3d if spatial_dims == 3 else nn.Conv2d


def _conv_transpose(spatial_dims: int) -> type[nn.Module]:
    if spatial_dims not in (2, 3):
        raise ValueError("spatial_dims must be 2 or 3")
    return nn.ConvTranspose3d if spatial_dims == 3 else nn.ConvTranspose2d


class EvalModeGELU(nn.Module):
    """Exact GELU while training; optionally the tanh form in evaluation."""

    def __init__(self, approximate_eval: bool = False) -> None:
        super().__init__()
        self.approximate_eval = approximate_eval

    def forward(self, x: Tensor) -> Tensor:
        tanh = self.approximate_eval and not self.training
        return F.gelu(x, approximate="tanh" if tanh else "none")

    def extra_repr(self) -> str:
        return f"approximate_eval={self.approximate_eval}"


class MedNeXtBlock(nn.Module):
    """depthwise conv -> GroupNorm(C, C) -> 1x1 expand -> GELU -> 1x1 project (+ x).

    ``kind`` is ``"regular"`` here; the down/up subclasses change the depthwise
    geometry.  When an sm_100a fused implementation has been installed
    (``self._fused`` set by ``install_adaptive_operators``) and the call is a CUDA
    training step, the whole block runs as one autograd node.
    """

    kind = "regular"

    def __init__(
        self,
        *,
        spatial_dims: int,
        in_channels: int,
        out_channels: int,
        expansion_ratio: int,
        kernel_size: int,
        residual: bool = True,
        checkpoint_expansion: bool = False,
        approximate_gelu_eval: bool = False,
    ) -> None:
        super().__init__()
        conv = _conv(spatial_dims)
        self.use_residual = residual
        self.checkpoint_expansion = checkpoint_expansion
        self.depthwise = conv(
            in_channels, in_channels, kernel_size=kernel_size, stride=1, padding=kernel_size // 2,
            groups=in_channels,
        )
        self.norm = nn.GroupNorm(in_channels, in_channels)
        self.expand = conv(in_channels, in_channels * expansion_ratio, kernel_size=1)
        self.activation = EvalModeGELU(approximate_eval=approximate_gelu_eval)
        self.project = conv(in_channels * expansion_ratio, out_channels, kernel_size=1)
        self._fused = None

    def _expansion(self, x: Tensor) -> Tensor:
        return self.project(self.activation(self.expand(x)))

    def _body(self, x: Tensor) -> Tensor:
        y = self.norm(self.depthwise(x))
        if self.checkpoint_expansion and self.training and torch.is_grad_enabled():
            return checkpoint(self._expansion, y, use_reentrant=False)
        return self._expansion(y)

    def _fused_call(self, x: Tensor, addend: Tensor | None, residual_is_input: bool) -> Tensor | None:
        fused = self._fused
        if fused is None:
            return None
        return fused(self, x, addend, residual_is_input)

    def forward(self, x: Tensor) -> Tensor:
        out = self._fused_call(x, None, self.use_residual)
        if out is not None:
            return out
        y = self._body(x)
        return y + x if self.use_residual else y


class MedNeXtDownBlock(MedNeXtBlock):
    """Stride-two block; the residual branch is a strided 1x1 convolution."""

    kind = "down"

    def __init__(
        self,
        *,
        spatial_dims: int,
        in_channels: int,
        out_channels: int,
        expansion_ratio: int,
        kernel_size: int,
        residual: bool = True,
        checkpoint_expansion: bool = False,
        approximate_gelu_eval: bool = False,
    ) -> None:
        super().__init__(
            spatial_dims=spatial_dims, in_channels=in_channels, out_channels=out_channels,
            expansion_ratio=expansion_ratio, kernel_size=kernel_size, residual=False,
            checkpoint_expansion=checkpoint_expansion, approximate_gelu_eval=approximate_gelu_eval,
        )
        conv = _conv(spatial_dims)
        self.depthwise = conv(
            in_channels, in_channels, kernel_size=kernel_size, stride=2, padding=kernel_size // 2,
            groups=in_channels,
        )
        self.residual = conv(in_channels, out_channels, kernel_size=1, stride=2) if residual else None

    def forward(self, x: Tensor) -> Tensor:
        # the fused operator computes the strided residual convolution itself
        out = self._fused_call(x, None, False)
        if out is not None:
            return out
        skip = self.residual(x) if self.residual is not None else None
        y = self._body(x)
        return y + skip if skip is not None else y


class MedNeXtUpBlock(MedNeXtBlock):
    """Stride-two transposed block; output is left-padded by one voxel per axis."""

    kind = "up"

    def __init__(
        self,
        *,
        spatial_dims: int,
        in_channels: int,
        out_channels: int,
        expansion_ratio: int,
        kernel_size: int,
        residual: bool = True,
        checkpoint_expansion: bool = False,
        approximate_gelu_eval: bool = False,
    ) -> None:
        super().__init__(
            spatial_dims=spatial_dims, in_channels=in_channels, out_channels=out_channels,
            expansion_ratio=expansion_ratio, kernel_size=kernel_size, residual=False,
            checkpoint_expansion=checkpoint_expansion, approximate_gelu_eval=approximate_gelu_eval,
        )
        up = _conv_transpose(spatial_dims)
        self.depthwise = up(
            in_channels, in_channels, kernel_size=kernel_size, stride=2, padding=kernel_size // 2,
            groups=in_channels,
        )
        self.residual = up(in_channels, out_channels, kernel_size=1, stride=2) if residual else None
        self._pad = (1, 0) * spatial_dims

    def forward(self, x: Tensor, addend: Tensor | None = None) -> Tensor:
        """``addend`` (optional, the padded output's shape): added to the output, as
        the decoder adds its encoder skip (models/mednext_v1.py:205); the fused
        operator does it in the pass that writes the padded output."""
        # the fused operator computes the strided residual convolution itself and
        # returns the padded output
        out = self._fused_call(x, addend, False)
        if out is not None:
            return out
        skip = self.residual(x) if self.residual is not None else None
        out = self._body(x)
        if skip is not None:
            out = out + skip
        # pad(a) + pad(b) == pad(a + b): one pad after the residual add
        out = F.pad(out, self._pad)
        return out + addend if addend is not None else out


class OutputHead(nn.Module):
    """1x1 transposed convolution, as in the official checkpoints."""

    def __init__(self, *, spatial_dims: int, in_channels: int, out_channels: int) -> None:
        super().__init__()
        self.conv = _conv_transpose(spatial_dims)(in_channels, out_channels, kernel_size=1)

    def forward(self, x: Tensor) -> Tensor:
        return self.conv(x)


class MedNeXtV1(nn.Module):
    """MedNeXt v1 U-Net: stem, 4 encoder stages + down blocks, bottleneck,
    4 up blocks + decoder stages, output head and optional deep-supervision heads."""

    def __init__(
        self,
        config: MedNeXtV1Config,
        *,
        checkpointing: CheckpointConfig | None = None,
        deep_supervision_output: DeepSupervisionOutput = "tuple",
        approximate_gelu_eval: bool = False,
    ) -> None:
        super().__init__()
        if deep_supervision_output not in ("tuple", "list", "stacked"):
            raise ValueError("deep_supervision_output must be 'tuple', 'list', or 'stacked'")
        self.config = config
        self.checkpointing = checkpointing
        self.deep_supervision_output = deep_supervision_output
        self.approximate_gelu_eval = approximate_gelu_eval
        self.optimization_source: OptimizationSource = "reference"
        dims = config.spatial_dims
        k = config.kernel_size
        widths = tuple(config.base_channels * 2**stage for stage in range(5))

        def ckpt_expansion(stage: int) -> bool:
            return bool(
                checkpointing is not None and checkpointing.checkpoints_expansion and checkpointing.includes(stage)
            )

        def blocks(stage: int, count: int, ratio: int) -> nn.Sequential:
            return nn.Sequential(
                *[
                    MedNeXtBlock(
                        spatial_dims=dims, in_channels=widths[stage], out_channels=widths[stage],
                        expansion_ratio=ratio, kernel_size=k, residual=config.residual_blocks,
                        checkpoint_expansion=ckpt_expansion(stage), approximate_gelu_eval=approximate_gelu_eval,
                    )
                    for _ in range(count)
                ]
            )

        self.stem = _conv(dims)(config.in_channels, config.base_channels, kernel_size=1)
        self.encoder_stages = nn.ModuleList(
            blocks(s, config.block_counts[s], config.expansion_ratios[s]) for s in range(4)
        )
        self.downsamples = nn.ModuleList(
            MedNeXtDownBlock(
                spatial_dims=dims, in_channels=widths[s], out_channels=widths[s + 1],
                expansion_ratio=config.downsample_expansion_ratios[s], kernel_size=k,
                residual=config.residual_resampling, checkpoint_expansion=ckpt_expansion(s + 1),
                approximate_gelu_eval=approximate_gelu_eval,
            )
            for s in range(4)
        )
        self.bottleneck = blocks(4, config.block_counts[4], config.expansion_ratios[4])
        self.upsamples = nn.ModuleList()
        self.decoder_stages = nn.ModuleList()
        # decoder stage s (3..0) uses configuration index 8 - s
        for s in (3, 2, 1, 0):
            ratio = config.expansion_ratios[8 - s]
            self.upsamples.append(
                MedNeXtUpBlock(
                    spatial_dims=dims, in_channels=widths[s + 1], out_channels=widths[s],
                    expansion_ratio=ratio, kernel_size=k, residual=config.residual_resampling,
                    checkpoint_expansion=ckpt_expansion(s), approximate_gelu_eval=approximate_gelu_eval,
                )
            )
            self.decoder_stages.append(blocks(s, config.block_counts[8 - s], ratio))
        self.head = OutputHead(spatial_dims=dims, in_channels=widths[0], out_channels=config.out_channels)
        self.deep_supervision_heads = nn.ModuleList()
        if config.deep_supervision:
            self.deep_supervision_heads.extend(
                OutputHead(spatial_dims=dims, in_channels=widths[s], out_channels=config.out_channels)
                for s in (4, 3, 2, 1)
            )

    def _run(self, module: nn.Module, x: Tensor, stage: int, addend: Tensor | None = None) -> Tensor:
        """module(x), or module(x, addend) for an up block given the decoder skip."""
        args = (x,) if addend is None else (x, addend)
        cfg = self.checkpointing
        if (
            cfg is not None and cfg.checkpoints_blocks and cfg.includes(stage) and self.training
            and torch.is_grad_enabled()
        ):
            return checkpoint(module, *args, use_reentrant=False)
        return module(*args)

    def _stage(self, modules: nn.Sequential, x: Tensor, stage: int) -> Tensor:
        for module in modules:
            x = self._run(module, x, stage)
        return x

    def forward(self, x: Tensor) -> Tensor | tuple[Tensor, ...] | list[Tensor]:
        x = self.stem(x)
        skips: list[Tensor] = []
        for stage in range(4):
            x = self._stage(self.encoder_stages[stage], x, stage)
            skips.append(x)
            x = self._run(self.downsamples[stage], x, stage + 1)
        x = self._stage(self.bottleneck, x, 4)
        aux: list[Tensor] = []
        supervise = self.training and self.config.deep_supervision
        for i in range(4):
            stage = 3 - i
            if supervise:
                aux.append(self.deep_supervision_heads[i](x))
            x = self._run(self.upsamples[i], x, stage, skips[stage])
            x = self._stage(self.decoder_stages[i], x, stage)
        primary = self.head(x)
        if not supervise:
            return primary
        outputs = [primary, *reversed(aux)]
        if self.deep_supervision_output == "tuple":
            return tuple(outputs)
        if self.deep_supervision_output == "list":
            return outputs
        size = primary.shape[2:]
        return torch.stack(
            [o if o.shape[2:] == size else F.interpolate(o, size=size) for o in outputs], dim=1
        )


def checkpoint_name(config: CheckpointConfig | None) -> str:
    if config is None:
        return "none"
    if config.stages is None:
        return "all-expansion" if config.style == "expansion" else "whole-block"
    return f"{config.style}:{','.join(map(str, config.stages))}"


def _factory(
    variant: str,
    *,
    in_channels: int,
    out_channels: int,
    spatial_dims: Literal[2, 3] = 3,
    kernel_size: int = 3,
    base_channels: int = 32,
    deep_supervision: bool = False,
    checkpointing: CheckpointConfig | None = None,
    deep_supervision_output: DeepSupervisionOutput = "tuple",
    approximate_gelu_eval: bool = False,
    optimization: OptimizationSource = "auto",
) -> MedNeXtV1:
    config = get_mednext_v1_config(
        variant, in_channels=in_channels, out_channels=out_channels, spatial_dims=spatial_dims,
        kernel_size=kernel_size, base_channels=base_channels, deep_supervision=deep_supervision,
    )
    model = MedNeXtV1(
        config, checkpointing=checkpointing, deep_supervision_output=deep_supervision_output,
        approximate_gelu_eval=approximate_gelu_eval,
    )
    return configure_optimization(model, optimization)


def configure_optimization(model: MedNeXtV1, optimization: OptimizationSource) -> MedNeXtV1:
    """``"reference"`` keeps plain PyTorch modules; ``"auto"`` installs the sm_100a
    operators (reference models/mednext_v1.py:371-392)."""
    from .adaptive import ModelOptimizationContext, install_adaptive_operators
    from .optimization import PolicyResolver

    model.optimization_source = optimization
    if optimization == "reference":
        return model
    if isinstance(optimization, str) and optimization in ("torch", "conservative", "autotune"):
        raise ValueError(f"optimization={optimization!r} was removed; use 'auto' or 'reference'")
    if optimization != "auto":
        raise ValueError(
            "the sm_100a build uses a fixed dispatch table; optimization must be 'auto' or 'reference'"
        )
    resolver = PolicyResolver()
    context = ModelOptimizationContext(
        "mednext_v1", model.config.variant, checkpoint_name(model.checkpointing), model.approximate_gelu_eval
    )
    install_adaptive_operators(model, resolver=resolver, model_context=context)
    model.__dict__["_optimization_resolver"] = resolver
    model.__dict__["_optimization_model_context"] = context
    return model


def _make(variant: str, doc: str):
    def factory(
        *,
        in_channels: int,
        out_channels: int,
        spatial_dims: Literal[2, 3] = 3,
        kernel_size: int = 3,
        base_channels: int = 32,
        deep_supervision: bool = False,
        checkpointing: CheckpointConfig | None = None,
        deep_supervision_output: DeepSupervisionOutput = "tuple",
        approximate_gelu_eval: bool = False,
        optimization: OptimizationSource = "auto",
    ) -> MedNeXtV1:
        return _factory(
            variant, in_channels=in_channels, out_channels=out_channels, spatial_dims=spatial_dims,
            kernel_size=kernel_size, base_channels=base_channels, deep_supervision=deep_supervision,
            checkpointing=checkpointing, deep_supervision_output=deep_supervision_output,
            approximate_gelu_eval=approximate_gelu_eval, optimization=optimization,
        )

    factory.__name__ = f"mednext_{variant}"
    factory.__qualname__ = factory.__name__
    factory.__doc__ = doc
    return factory


mednext_small = _make("small", "Build MedNeXt Small (reference models/mednext_v1.py:395-422).")
mednext_base = _make("base", "Build MedNeXt Base (reference models/mednext_v1.py:425-452).")
mednext_medium = _make("medium", "Build MedNeXt Medium (reference models/mednext_v1.py:455-482).")
mednext_large = _make("large", "Build MedNeXt Large (reference models/mednext_v1.py:485-512).")

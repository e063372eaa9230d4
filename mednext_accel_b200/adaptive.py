"""Drop-in wrappers that keep native module parameters and state-dict keys.

Mirrors the reference's ``mednext_accel/ops/adaptive.py``:
``ModelOptimizationContext``, ``execution_context_for_shape``,
``AdaptivePointwise3d`` (lines 125-200), ``AdaptiveDepthwise3d`` (203-320) and
``install_adaptive_operators`` (351-376), with the same eligibility rules
(323-348) and the same ``Parameter`` objects, so optimizers, checkpoints and
``state_dict`` keys are unchanged.

On a CUDA device of compute capability 10.0 in training, the resolver selects the
sm_100a operators and they run unconditionally: a missing or unloadable
``libmednext_b200.so`` raises instead of silently falling back.  Outside that
context (CPU tensors, evaluation, export, other GPUs) the resolver returns
``"reference"`` and the modules run their native PyTorch definition, which is
the reference package's documented behaviour for those contexts
(ops/adaptive.py:259-268).

Additionally, ``install_adaptive_operators`` attaches a fused implementation to
every :class:`mednext_accel_b200.network.MedNeXtBlock`, so a whole block runs
as a single operator (:mod:`mednext_accel_b200.block`).
"""

from __future__ import annotations

import dataclasses

from dataclasses import dataclass

import torch
from torch import Tensor, nn
from torch.nn import functional as F

from .optimization import ExecutionContext, OperatorDescriptor, PolicyDecision, PolicyResolver

_AUTOCAST_COMPUTE = (torch.bfloat16, torch.float16)


@dataclass(frozen=True, slots=True)
class ModelOptimizationContext:
    """Model-level facts every operator of one model shares (family, variant,
    checkpointing label, approximation opt-in)."""

    family: str
    variant: str
    checkpointing: str
    allow_approximate: bool = False


def _phase(training: bool, export: bool) -> str:
    if export:
        return "export"
    return "training" if training else "inference"


def execution_context_for_shape(
    model_context: ModelOptimizationContext,
    *,
    batch_size: int,
    spatial_shape: tuple[int, ...],
    dtype: torch.dtype | str,
    device_type: str,
    sm: tuple[int, int] | None,
    total_vram_bytes: int,
    training: bool = True,
    export: bool = False,
) -> ExecutionContext:
    """Combine the model's context with the facts of one call into the
    ExecutionContext the resolver reads.  ``dtype`` may be a torch dtype or its
    name ("bfloat16")."""
    dtype_name = dtype if isinstance(dtype, str) else str(dtype).split(".")[-1]
    model = model_context
    return ExecutionContext(_phase(training, export), device_type, sm, total_vram_bytes, dtype_name, batch_size,
                            spatial_shape, model.family, model.variant, model.checkpointing, export,
                            model.allow_approximate)


_DEVICE_FACTS: dict[int, tuple[tuple[int, int], int]] = {}


def _device_facts(device: torch.device) -> tuple[tuple[int, int], int]:
    index = device.index if device.index is not None else torch.cuda.current_device()
    facts = _DEVICE_FACTS.get(index)
    if facts is None:
        props = torch.cuda.get_device_properties(index)
        facts = ((props.major, props.minor), props.total_memory)
        _DEVICE_FACTS[index] = facts
    return facts


def compute_dtype(x: Tensor) -> torch.dtype:
    """The dtype the reference computes convolutions in for this input."""
    if torch.is_autocast_enabled(x.device.type) and x.dtype != torch.float64:
        return torch.get_autocast_dtype(x.device.type)
    return x.dtype


def _context_from_tensor(x: Tensor, model_context: ModelOptimizationContext, *, training: bool) -> ExecutionContext:
    export = torch.jit.is_tracing() or torch.onnx.is_in_onnx_export()
    sm = None
    total = 0
    if x.device.type == "cuda" and not export:
        sm, total = _device_facts(x.device)
    batch = 1 if x.ndim == 4 else int(x.shape[0])
    return execution_context_for_shape(
        model_context,
        batch_size=batch,
        spatial_shape=tuple(int(s) for s in x.shape[-3:]),
        dtype=compute_dtype(x),
        device_type=x.device.type,
        sm=sm,
        total_vram_bytes=total,
        training=training,
        export=export,
    )


def conv_descriptor(conv: nn.Module, *, role: str | None, expansion_ratio: int | None = None) -> OperatorDescriptor:
    transpose = isinstance(conv, (nn.ConvTranspose2d, nn.ConvTranspose3d))
    depthwise = conv.groups == conv.in_channels == conv.out_channels
    dims = len(conv.kernel_size)
    if transpose and depthwise:
        family = "depthwise_conv_transpose"
    elif transpose:
        family = "conv_transpose"
    elif depthwise:
        family = "depthwise_conv"
    elif conv.kernel_size == (1,) * dims and conv.groups == 1:
        family = "pointwise_conv"
    else:
        family = "conv"
    direction = "transpose" if transpose else ("downsample" if conv.stride[0] == 2 else "regular")
    return OperatorDescriptor(
        family=f"{family}{dims}d", direction=direction, in_channels=conv.in_channels,
        out_channels=conv.out_channels, kernel_size=conv.kernel_size, stride=conv.stride,
        padding=conv.padding, dilation=conv.dilation, groups=conv.groups, role=role,
        expansion_ratio=expansion_ratio,
    )


class _AdaptiveConv3d(nn.Module):
    def _warn_for_device(self) -> None:
        if self.weight.device.type == "cuda":
            self.resolver.warn_for_sm(_device_facts(self.weight.device)[0])

    def _apply(self, fn, recurse=True):
        result = super()._apply(fn, recurse=recurse)
        self._warn_for_device()
        return result


class AdaptivePointwise3d(_AdaptiveConv3d):
    """1x1x1 convolution routed to the tensor-core pointwise operator."""

    _mednext_accel_backend_kind = "pointwise_gemm"

    def __init__(self, conv: nn.Conv3d | nn.ConvTranspose3d, resolver: PolicyResolver,
                 model_context: ModelOptimizationContext, *, role: str | None = None) -> None:
        super().__init__()
        self.weight = conv.weight
        self.bias = conv.bias
        for name in ("in_channels", "out_channels", "kernel_size", "stride", "padding", "dilation", "groups"):
            setattr(self, name, getattr(conv, name))
        # a 1x1x1 transposed convolution is the pointwise contraction with weight [cin, cout]
        self.transposed = isinstance(conv, nn.ConvTranspose3d)
        self.descriptor = conv_descriptor(conv, role=role)
        if self.transposed:
            self.descriptor = dataclasses.replace(self.descriptor, family="pointwise_conv3d", direction="regular")
        self.resolver = resolver
        self.model_context = model_context
        self.train(conv.training)
        self._warn_for_device()

    def decision_for_shape(self, *, batch_size: int, spatial_shape: tuple[int, int, int], dtype: torch.dtype | str,
                           device_type: str, sm: tuple[int, int] | None, total_vram_bytes: int) -> PolicyDecision:
        context = execution_context_for_shape(
            self.model_context, batch_size=batch_size, spatial_shape=spatial_shape, dtype=dtype,
            device_type=device_type, sm=sm, total_vram_bytes=total_vram_bytes, training=self.training,
        )
        return self.resolver.resolve(self.descriptor, context, context.phase)

    def forward(self, x: Tensor) -> Tensor:
        context = _context_from_tensor(x, self.model_context, training=self.training)
        decision = self.resolver.resolve(self.descriptor, context, context.phase)
        if decision.implementation != "reference" and torch.is_grad_enabled() and x.ndim == 5 and x.is_contiguous():
            from .pointwise import pointwise_conv3d

            cdt = getattr(torch, context.dtype)
            bias = self.bias.to(cdt) if self.bias is not None else None
            weight = self.weight.transpose(0, 1) if self.transposed else self.weight
            return pointwise_conv3d(x.to(cdt), weight.to(cdt), bias)
        if self.transposed:
            return F.conv_transpose3d(x, self.weight, self.bias)
        return F.conv3d(x, self.weight, self.bias)


class AdaptiveDepthwise3d(_AdaptiveConv3d):
    """Depthwise Conv3d / ConvTranspose3d routed to the sm_100a depthwise operators."""

    _mednext_accel_backend_kind = "depthwise"

    def __init__(self, conv: nn.Conv3d | nn.ConvTranspose3d, resolver: PolicyResolver,
                 model_context: ModelOptimizationContext, *, role: str | None = None) -> None:
        super().__init__()
        self.weight = conv.weight
        self.bias = conv.bias
        for name in ("in_channels", "out_channels", "kernel_size", "stride", "padding", "dilation", "groups"):
            setattr(self, name, getattr(conv, name))
        self.output_padding = getattr(conv, "output_padding", (0, 0, 0))
        self.transpose = isinstance(conv, nn.ConvTranspose3d)
        self.descriptor = conv_descriptor(conv, role=role)
        self.resolver = resolver
        self.model_context = model_context
        self.train(conv.training)
        self._warn_for_device()

    def _reference(self, x: Tensor) -> Tensor:
        if self.transpose:
            return F.conv_transpose3d(x, self.weight, self.bias, self.stride, self.padding, self.output_padding,
                                      self.groups, self.dilation)
        return F.conv3d(x, self.weight, self.bias, self.stride, self.padding, self.dilation, self.groups)

    def forward(self, x: Tensor) -> Tensor:
        context = _context_from_tensor(x, self.model_context, training=self.training)
        if (
            context.phase != "training"
            or context.device_type != "cuda"
            or not torch.is_grad_enabled()
            or x.ndim != 5
            or self.output_padding != (0, 0, 0)
            or not x.is_contiguous()
            or tuple(x.shape[2:]) != (x.shape[2],) * 3
        ):
            return self._reference(x)
        dx = self.resolver.resolve(self.descriptor, context, "backward_input")
        dw = self.resolver.resolve(self.descriptor, context, "backward_weight")
        if dx.implementation == dw.implementation == "reference":
            return self._reference(x)
        from . import depthwise as backend  # no fallback: an import failure propagates

        x = x.to(getattr(torch, context.dtype))
        weight = self.weight.to(x.dtype)
        bias = self.bias.to(x.dtype) if self.bias is not None else None
        size = int(x.shape[2])
        k = self.kernel_size[0]
        if self.transpose:
            return backend.depthwise_conv_transpose3d_regular(x, weight, bias, k, self.in_channels, size, 0, 0)
        if self.stride == (2, 2, 2):
            return backend.depthwise_conv3d_stride2_regular(x, weight, bias, k, self.in_channels, size, 0)
        return backend.depthwise_conv3d_regular(x, weight, bias, k, self.in_channels, size, 0, 0, 0, True, True)


def _pointwise_eligible(module: nn.Module) -> bool:
    """1x1x1, stride-1 Conv3d, or ConvTranspose3d (the output heads), which is the
    same contraction with the weight's first two axes swapped."""
    if type(module) is nn.ConvTranspose3d and module.output_padding != (0, 0, 0):
        return False
    return (
        type(module) in (nn.Conv3d, nn.ConvTranspose3d)
        and module.kernel_size == (1, 1, 1)
        and module.stride == (1, 1, 1)
        and module.padding == (0, 0, 0)
        and module.dilation == (1, 1, 1)
        and module.groups == 1
        and module.padding_mode == "zeros"
    )


def _depthwise_eligible(module: nn.Module) -> bool:
    if type(module) not in (nn.Conv3d, nn.ConvTranspose3d):
        return False
    k = module.kernel_size[0]
    return (
        len(set(module.kernel_size)) == 1
        and k % 2 == 1
        and module.in_channels == module.out_channels == module.groups
        and module.stride in ((1, 1, 1), (2, 2, 2))
        and module.padding == (k // 2,) * 3
        and module.dilation == (1, 1, 1)
        and getattr(module, "padding_mode", "zeros") == "zeros"
        and getattr(module, "output_padding", (0, 0, 0)) == (0, 0, 0)
    )


class FusedBlockRunner:
    """Callable attached to a MedNeXt block: resolves the block descriptor and,
    when the sm_100a fused implementation is selected, runs the block as one
    ``mednext_accel_b200::mednext_block`` operator.  Returns None to let the block
    run its per-module path otherwise."""

    def __init__(self, block: nn.Module, resolver: PolicyResolver, model_context: ModelOptimizationContext,
                 role: str) -> None:
        from .block import KIND_DOWN, KIND_REGULAR, KIND_UP

        dw = block.depthwise
        self.kind = {"regular": KIND_REGULAR, "down": KIND_DOWN, "up": KIND_UP}[block.kind]
        ratio = block.expand.out_channels // block.expand.in_channels
        direction = {"regular": "regular", "down": "downsample", "up": "transpose"}[block.kind]
        self.descriptor = OperatorDescriptor(
            family="mednext_block3d", direction=direction, in_channels=dw.in_channels,
            out_channels=block.project.out_channels, kernel_size=dw.kernel_size, stride=dw.stride,
            padding=dw.padding, dilation=dw.dilation, groups=dw.groups, role=role, expansion_ratio=ratio,
        )
        self.resolver = resolver
        self.model_context = model_context

    def decision(self, block: nn.Module, x: Tensor) -> PolicyDecision:
        context = _context_from_tensor(x, self.model_context, training=block.training)
        return self.resolver.resolve(self.descriptor, context, context.phase)

    def __call__(self, block: nn.Module, x: Tensor, addend: Tensor | None, residual_is_input: bool) -> Tensor | None:
        if not (block.training and torch.is_grad_enabled() and x.device.type == "cuda" and x.ndim == 5):
            return None
        if block.norm.num_groups != block.norm.num_channels or block.activation.approximate_eval and not block.training:
            return None
        decision = self.decision(block, x)
        if decision.implementation == "reference":
            return None
        from .block import KIND_REGULAR, KIND_UP, dtype_code, mednext_block

        cdt = compute_dtype(x)
        if cdt not in _AUTOCAST_COMPUTE:
            return None
        if not x.is_contiguous():
            x = x.contiguous()
        keep = not (block.checkpoint_expansion or decision.parameters.get("recompute_expansion", False))
        # the down / up blocks' strided 1x1 residual convolution runs inside the operator
        # (the up block's addend is added after its pad, so its residual conv stays fused)
        fuse_res = self.kind != KIND_REGULAR and (addend is None or self.kind == KIND_UP)
        res = getattr(block, "residual", None) if fuse_res else None
        res_w = res.weight if res is not None else None
        res_b = res.bias if res is not None else None
        y, _, _, _, _ = mednext_block(
            x, addend, block.depthwise.weight, block.depthwise.bias, block.norm.weight, block.norm.bias,
            block.expand.weight, block.expand.bias, block.project.weight, block.project.bias, res_w, res_b,
            self.kind, int(block.depthwise.kernel_size[0]), float(block.norm.eps), bool(residual_is_input), keep,
            dtype_code(cdt),
        )
        return y


def install_adaptive_operators(
    model: nn.Module,
    *,
    resolver: PolicyResolver,
    model_context: ModelOptimizationContext,
    _prefix: str = "",
) -> int:
    """Install wrappers in place while retaining every Parameter object
    (depthwise and pointwise convolutions, MedNeXt blocks, GRN layers)."""
    from .grn import AdaptiveGlobalResponseNorm3d, GlobalResponseNorm3d
    from .network import MedNeXtBlock

    count = 0
    if isinstance(model, MedNeXtBlock) and model._fused is None:
        model._fused = FusedBlockRunner(model, resolver, model_context, _prefix or "block")
    for name, child in list(model.named_children()):
        role = f"{_prefix}.{name}" if _prefix else name
        if _pointwise_eligible(child):
            setattr(model, name, AdaptivePointwise3d(child, resolver, model_context, role=role))
            count += 1
        elif _depthwise_eligible(child):
            setattr(model, name, AdaptiveDepthwise3d(child, resolver, model_context, role=role))
            count += 1
        elif type(child) is GlobalResponseNorm3d:
            setattr(model, name, AdaptiveGlobalResponseNorm3d(child, resolver, model_context, role))
            count += 1
        else:
            count += install_adaptive_operators(child, resolver=resolver, model_context=model_context, _prefix=role)
    return count

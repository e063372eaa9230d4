"""Operator descriptors, implementation registry and the fixed sm_100a resolver.

The public surface mirrors the reference package's selection API so callers do
not change: ``OperatorDescriptor`` / ``ExecutionContext``
(optimization/descriptors.py:23-156), ``ImplementationSpec`` /
``ImplementationRegistry`` (optimization/implementations.py:87-158),
``PolicyDecision`` and ``PolicyResolver.resolve(descriptor, context, phase)``
(optimization/policy_resolver.py:20-231).

What changes is how a decision is made.  The reference layers YAML policies
(external -> exact SM -> shared NVIDIA -> reference) with per-shape launch
recipes and autotuning evidence.  Here a single fixed table, keyed on the
operator family/direction and on (channels, expansion ratio, kernel size,
spatial size), selects the sm_100a implementation and its launch parameters for
compute capability (10, 0).  Every implementation identifier the reference
defines still resolves: the Triton ids name the same phases, now served by the
sm_100a kernels.
"""

from __future__ import annotations

import warnings
from collections.abc import Callable, Mapping, Sequence
from dataclasses import asdict, dataclass, field
from math import prod
from types import MappingProxyType
from typing import Literal

ExecutionPhase = Literal["training", "inference", "export"]
SemanticEquivalence = Literal["exact", "numerical", "approximate"]
Confidence = Literal["guard", "fixed-table", "measured-exact-context"]
SM100 = (10, 0)


def _spatial_tuple(value: tuple[int, ...], name: str, *, positive: bool = True) -> tuple[int, ...]:
    result = tuple(value)
    if len(result) not in (2, 3) or any(not isinstance(item, int) for item in result):
        raise ValueError(f"{name} must contain two or three integers")
    lower = 1 if positive else 0
    if any(item < lower for item in result):
        raise ValueError(f"{name} values must be >= {lower}")
    return result


@dataclass(frozen=True, slots=True)
class OperatorDescriptor:
    """Shape-independent identity of one optimizable operator."""

    family: str
    direction: str
    in_channels: int
    out_channels: int
    kernel_size: tuple[int, ...] | None = None
    stride: tuple[int, ...] | None = None
    padding: tuple[int, ...] | None = None
    dilation: tuple[int, ...] | None = None
    groups: int | None = None
    role: str | None = None
    expansion_ratio: int | None = None

    def __post_init__(self) -> None:
        if not self.family or not self.direction:
            raise ValueError("family and direction must be non-empty")
        for name in ("in_channels", "out_channels"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")
        geometry = ("kernel_size", "stride", "padding", "dilation", "groups")
        present = tuple(getattr(self, name) is not None for name in geometry)
        if any(present) and not all(present):
            raise ValueError("convolution geometry fields must be supplied together")
        if not any(present):
            return
        if self.groups is None or self.groups <= 0:
            raise ValueError("groups must be positive")
        object.__setattr__(self, "kernel_size", _spatial_tuple(self.kernel_size, "kernel_size"))
        object.__setattr__(self, "stride", _spatial_tuple(self.stride, "stride"))
        object.__setattr__(self, "padding", _spatial_tuple(self.padding, "padding", positive=False))
        object.__setattr__(self, "dilation", _spatial_tuple(self.dilation, "dilation"))

    @property
    def signature(self) -> tuple[object, ...]:
        return (self.family, self.direction, self.in_channels, self.out_channels, self.kernel_size, self.stride)

    def to_primitive(self) -> dict[str, object]:
        value = asdict(self)
        for name in ("kernel_size", "stride", "padding", "dilation"):
            if value[name] is not None:
                value[name] = list(value[name])
        return {name: item for name, item in value.items() if item is not None}


@dataclass(frozen=True, slots=True)
class ExecutionContext:
    """Runtime facts used for implementation resolution."""

    phase: ExecutionPhase
    device_type: str
    sm: tuple[int, int] | None
    total_vram_bytes: int
    dtype: str
    batch_size: int
    spatial_shape: tuple[int, ...]
    model_family: str
    variant: str
    checkpointing: str
    export: bool = False
    allow_approximate: bool = False

    def __post_init__(self) -> None:
        if self.phase not in ("training", "inference", "export"):
            raise ValueError(f"unknown phase {self.phase!r}")
        if self.batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if self.total_vram_bytes < 0:
            raise ValueError("total_vram_bytes must be nonnegative")
        object.__setattr__(self, "spatial_shape", _spatial_tuple(self.spatial_shape, "spatial_shape"))
        if self.sm is not None:
            sm = tuple(self.sm)
            if len(sm) != 2 or any(item < 0 for item in sm):
                raise ValueError("sm must contain two nonnegative integers")
            object.__setattr__(self, "sm", sm)

    @property
    def spatial_volume(self) -> int:
        return prod(self.spatial_shape)

    @property
    def total_vram_gib(self) -> float:
        return self.total_vram_bytes / 2**30

    def to_primitive(self) -> dict[str, object]:
        value = asdict(self)
        value["spatial_shape"] = list(self.spatial_shape)
        value["sm"] = None if self.sm is None else list(self.sm)
        return value


EligibilityGuard = Callable[[OperatorDescriptor, ExecutionContext, str], "str | None"]


@dataclass(frozen=True, slots=True)
class ImplementationSpec:
    identifier: str
    version: int
    families: tuple[str, ...]
    phases: tuple[str, ...]
    equivalence: SemanticEquivalence
    export_safe: bool

    def __post_init__(self) -> None:
        object.__setattr__(self, "families", tuple(self.families))
        object.__setattr__(self, "phases", tuple(self.phases))
        if not self.identifier or self.version <= 0:
            raise ValueError("implementation identifier and version must be valid")
        if not self.families or not self.phases:
            raise ValueError("implementation families and phases must not be empty")
        if self.equivalence not in ("exact", "numerical", "approximate"):
            raise ValueError(f"unknown equivalence {self.equivalence!r}")

    def is_allowed(self, *, allow_approximate: bool, export: bool = False) -> bool:
        return (self.equivalence != "approximate" or allow_approximate) and (not export or self.export_safe)


class ImplementationRegistry:
    """Backend-independent registry keyed by stable public identifiers."""

    def __init__(self) -> None:
        self._specs: dict[str, ImplementationSpec] = {}
        self._eligibility: dict[str, EligibilityGuard | None] = {}
        self._execution_guards: dict[str, tuple[str, ...]] = {}

    def register(
        self,
        spec: ImplementationSpec,
        *,
        eligibility: EligibilityGuard | None = None,
        execution_guards: tuple[str, ...] = (),
    ) -> None:
        if spec.identifier in self._specs:
            raise ValueError(f"implementation {spec.identifier!r} is already registered")
        self._specs[spec.identifier] = spec
        self._eligibility[spec.identifier] = eligibility
        self._execution_guards[spec.identifier] = tuple(execution_guards)

    def resolve_metadata(self, identifier: str) -> ImplementationSpec:
        try:
            return self._specs[identifier]
        except KeyError as error:
            raise ValueError(f"unknown implementation {identifier!r}") from error

    def guard(self, identifier: str, descriptor: OperatorDescriptor, context: ExecutionContext, phase: str) -> str | None:
        self.resolve_metadata(identifier)
        guard = self._eligibility[identifier]
        return None if guard is None else guard(descriptor, context, phase)

    def execution_guards(self, identifier: str) -> tuple[str, ...]:
        self.resolve_metadata(identifier)
        return self._execution_guards[identifier]

    def __contains__(self, identifier: object) -> bool:
        return identifier in self._specs

    def __iter__(self):
        return iter(self._specs.values())


# --------------------------------------------------------------------------- eligibility
_DTYPES = ("bfloat16", "float16", "float32", "float64")
_TC_DTYPES = ("bfloat16", "float16")


def _training_cuda(context: ExecutionContext) -> str | None:
    if context.phase != "training":
        return "implementation requires training"
    if context.device_type != "cuda":
        return "implementation requires CUDA"
    return None


def _depthwise_eligibility(direction: str) -> EligibilityGuard:
    stride = 1 if direction == "regular" else 2

    def guard(descriptor: OperatorDescriptor, context: ExecutionContext, phase: str) -> str | None:
        reason = _training_cuda(context)
        if reason:
            return reason
        if context.dtype not in _DTYPES:
            return "implementation does not support this dtype"
        k = descriptor.kernel_size
        if (
            k is None
            or descriptor.direction != direction
            or k != (k[0],) * 3
            or k[0] not in (1, 3, 5, 7)
            or descriptor.stride != (stride,) * 3
            or descriptor.padding != (k[0] // 2,) * 3
            or descriptor.dilation != (1, 1, 1)
            or not (descriptor.groups == descriptor.in_channels == descriptor.out_channels)
        ):
            return "implementation does not support this geometry"
        return None

    return guard


def _pointwise_eligibility(descriptor: OperatorDescriptor, context: ExecutionContext, phase: str) -> str | None:
    reason = _training_cuda(context)
    if reason:
        return reason
    if context.dtype not in _TC_DTYPES:
        return "tensor-core pointwise requires bfloat16 or float16 compute"
    if (
        descriptor.direction != "regular"
        or descriptor.kernel_size != (1, 1, 1)
        or descriptor.stride != (1, 1, 1)
        or descriptor.padding != (0, 0, 0)
        or descriptor.dilation != (1, 1, 1)
        or descriptor.groups != 1
    ):
        return "implementation does not support this geometry"
    return None


def _block_eligibility(descriptor: OperatorDescriptor, context: ExecutionContext, phase: str) -> str | None:
    reason = _training_cuda(context)
    if reason:
        return reason
    if context.dtype not in _TC_DTYPES:
        return "the fused block computes its GEMMs in bfloat16 or float16"
    k = descriptor.kernel_size
    if k is None or k != (k[0],) * 3 or k[0] not in (1, 3, 5, 7):
        return "implementation does not support this geometry"
    return None


DEPTHWISE_PHASES = ("forward", "backward_input", "backward_weight", "backward_bias")


def default_implementation_registry() -> ImplementationRegistry:
    """Every identifier of the reference registry plus the sm_100a ones."""
    registry = ImplementationRegistry()
    conv_guards = ("grad_enabled", "rank_5", "contiguous", "zero_output_padding")
    all_phases = ("training", "inference", "export", *DEPTHWISE_PHASES)
    definitions: tuple[tuple[str, tuple[str, ...], tuple[str, ...], SemanticEquivalence, bool, EligibilityGuard | None, tuple[str, ...]], ...] = (
        ("reference", ("*",), all_phases, "exact", True, None, ()),
        # sm_100a implementations
        ("sm100_depthwise", ("depthwise_conv3d",), DEPTHWISE_PHASES, "numerical", False,
         _depthwise_eligibility("regular"), conv_guards),
        ("sm100_depthwise_downsample", ("depthwise_conv3d",), DEPTHWISE_PHASES, "numerical", False,
         _depthwise_eligibility("downsample"), conv_guards),
        ("sm100_depthwise_transpose", ("depthwise_conv_transpose3d",), DEPTHWISE_PHASES, "numerical", False,
         _depthwise_eligibility("transpose"), conv_guards),
        ("sm100_pointwise", ("pointwise_conv3d",), ("training",), "numerical", False,
         _pointwise_eligibility, ("grad_enabled", "rank_5", "contiguous")),
        ("sm100_fused_block", ("mednext_block3d",), ("training",), "numerical", False,
         _block_eligibility, ("grad_enabled", "rank_5", "contiguous")),
        # identifiers of the reference registry, served by the sm_100a kernels
        ("pointwise_gemm_per_sample", ("pointwise_conv3d",), ("training",), "numerical", False,
         _pointwise_eligibility, ("grad_enabled", "rank_5", "contiguous")),
        ("triton_depthwise_dx", ("depthwise_conv3d",), ("backward_input",), "numerical", False,
         _depthwise_eligibility("regular"), conv_guards),
        ("triton_split_dw", ("depthwise_conv3d",), ("backward_weight",), "numerical", False,
         _depthwise_eligibility("regular"), conv_guards),
        ("triton_transpose_split_dw", ("depthwise_conv_transpose3d",), ("backward_weight",), "numerical", False,
         _depthwise_eligibility("transpose"), conv_guards),
        ("triton_downsample_dx", ("depthwise_conv3d",), ("backward_input",), "numerical", False,
         _depthwise_eligibility("downsample"), conv_guards),
        ("gelu_tanh", ("gelu",), ("inference",), "approximate", True, None, ()),
    )
    for identifier, families, phases, equivalence, export_safe, eligibility, guards in definitions:
        registry.register(
            ImplementationSpec(identifier, 1, families, phases, equivalence, export_safe),
            eligibility=eligibility,
            execution_guards=guards,
        )
    return registry


# Reference implementation ids that this build serves with its own kernels.
LEGACY_ALIASES: Mapping[str, str] = MappingProxyType(
    {
        "pointwise_gemm_per_sample": "sm100_pointwise",
        "triton_depthwise_dx": "sm100_depthwise",
        "triton_split_dw": "sm100_depthwise",
        "triton_transpose_split_dw": "sm100_depthwise_transpose",
        "triton_downsample_dx": "sm100_depthwise_downsample",
    }
)


@dataclass(frozen=True, slots=True)
class TableRow:
    """One row of the fixed sm_100a dispatch table.

    ``channels``/``ratio``/``kernel``/``spatial`` of None match anything.
    ``parameters`` are the launch choices recorded for the matched shapes."""

    rule: str
    family: str
    direction: str
    implementation: str
    channels: int | None = None
    ratio: int | None = None
    kernel: int | None = None
    spatial: int | None = None
    parameters: Mapping[str, object] = field(default_factory=dict)

    def matches(self, descriptor: OperatorDescriptor, context: ExecutionContext) -> bool:
        if descriptor.family != self.family or descriptor.direction != self.direction:
            return False
        if self.channels is not None and descriptor.in_channels != self.channels:
            return False
        if self.ratio is not None and descriptor.expansion_ratio != self.ratio:
            return False
        if self.kernel is not None and (descriptor.kernel_size or (None,))[0] != self.kernel:
            return False
        if self.spatial is not None and context.spatial_shape[0] != self.spatial:
            return False
        return True


def _block_rows() -> tuple[TableRow, ...]:
    # MedNeXt v1 block shapes at 128^3 input (Base/Large, k 3/5).  The stored
    # expanded activation of the widest high-resolution blocks is recomputed in
    # backward instead of kept (a GEMM is cheaper than the HBM round trip).
    rows = []
    for spatial, channels in ((128, 32), (64, 64), (32, 128), (16, 256), (8, 512)):
        for ratio in (2, 3, 4, 8):
            rows.append(
                TableRow(
                    f"block-c{channels}-r{ratio}-s{spatial}", "mednext_block3d", "regular", "sm100_fused_block",
                    channels=channels, ratio=ratio, spatial=spatial,
                    parameters={"recompute_expansion": False},
                )
            )
    return tuple(rows)


SM100_TABLE: tuple[TableRow, ...] = (
    *_block_rows(),
    TableRow("block-regular", "mednext_block3d", "regular", "sm100_fused_block"),
    TableRow("block-down", "mednext_block3d", "downsample", "sm100_fused_block"),
    TableRow("block-up", "mednext_block3d", "transpose", "sm100_fused_block"),
    TableRow("depthwise-regular", "depthwise_conv3d", "regular", "sm100_depthwise"),
    TableRow("depthwise-downsample", "depthwise_conv3d", "downsample", "sm100_depthwise_downsample"),
    TableRow("depthwise-transpose", "depthwise_conv_transpose3d", "transpose", "sm100_depthwise_transpose"),
    TableRow("pointwise", "pointwise_conv3d", "regular", "sm100_pointwise"),
)


@dataclass(frozen=True, slots=True)
class PolicyDecision:
    descriptor: OperatorDescriptor
    phase: str
    implementation: str
    parameters: Mapping[str, object]
    policy: str
    rule: str
    confidence: Confidence
    warning: str | None = None
    guard_reason: str | None = None
    execution_guards: tuple[str, ...] = ()
    disposition: Literal["custom", "native", "unwrapped"] = "native"

    def __post_init__(self) -> None:
        object.__setattr__(self, "parameters", MappingProxyType(dict(self.parameters)))
        object.__setattr__(self, "execution_guards", tuple(self.execution_guards))


class PolicyResolver:
    """Fixed sm_100a dispatch table, then the built-in reference.

    ``table`` replaces the reference's YAML policy layers; ``overrides`` maps a
    (family, direction) pair to an implementation id for tests and experiments
    (for example forcing ``"reference"`` to compare against native PyTorch)."""

    name = "sm100-fixed"

    def __init__(
        self,
        table: Sequence[TableRow] = SM100_TABLE,
        *,
        registry: ImplementationRegistry | None = None,
        overrides: Mapping[tuple[str, str], str] | None = None,
    ) -> None:
        self.table = tuple(table)
        self.registry = registry or default_implementation_registry()
        self.overrides = dict(overrides or {})
        self._warned: set[str] = set()

    def context_layers(self, context: ExecutionContext) -> tuple[str, ...]:
        if context.device_type != "cuda" or context.sm != SM100:
            return ()
        return (self.name,)

    def warn_for_sm(self, sm: tuple[int, int] | None) -> str | None:
        if sm is None or sm == SM100:
            return None
        message = f"the sm_100a operator table does not cover SM {sm}; using the PyTorch reference path"
        if message not in self._warned:
            warnings.warn(message, UserWarning, stacklevel=3)
            self._warned.add(message)
        return message

    def _reference(self, descriptor, phase, rule, reason, warning=None) -> PolicyDecision:
        return PolicyDecision(descriptor, phase, "reference", {}, "reference", rule, "guard", warning, guard_reason=reason)

    def resolve(self, descriptor: OperatorDescriptor, context: ExecutionContext, phase: str) -> PolicyDecision:
        if context.device_type != "cuda" or context.sm is None:
            return self._reference(descriptor, phase, "context-guard", "requires CUDA with a known NVIDIA SM")
        if context.sm != SM100:
            warning = self.warn_for_sm(context.sm)
            return self._reference(descriptor, phase, "sm-guard", "requires compute capability 10.0", warning)
        override = self.overrides.get((descriptor.family, descriptor.direction))
        if override is not None:
            return self._decide(TableRow("override", descriptor.family, descriptor.direction, override), descriptor, context, phase)
        for row in self.table:
            if row.matches(descriptor, context):
                return self._decide(row, descriptor, context, phase)
        return self._reference(descriptor, phase, "fallback", None)

    def _decide(self, row: TableRow, descriptor, context, phase) -> PolicyDecision:
        impl = row.implementation
        if impl == "reference":
            return PolicyDecision(descriptor, phase, "reference", {}, self.name, row.rule, "fixed-table")
        spec = self.registry.resolve_metadata(impl)
        reason = None
        if "*" not in spec.families and descriptor.family not in spec.families:
            reason = "implementation does not support this operator family"
        elif phase not in spec.phases:
            reason = "implementation does not support this phase"
        elif (context.export or context.phase == "export" or phase == "export") and not spec.export_safe:
            reason = "implementation is not export safe"
        elif spec.equivalence == "approximate" and not context.allow_approximate:
            reason = "approximate implementation requires allow_approximate"
        else:
            reason = self.registry.guard(impl, descriptor, context, phase)
        if reason is not None:
            return self._reference(descriptor, phase, row.rule, reason)
        return PolicyDecision(
            descriptor, phase, LEGACY_ALIASES.get(impl, impl), row.parameters, self.name, row.rule, "fixed-table",
            execution_guards=self.registry.execution_guards(impl), disposition="custom",
        )

    def resolve_all(
        self, descriptors: Sequence[OperatorDescriptor], context: ExecutionContext, phase: str
    ) -> tuple[PolicyDecision, ...]:
        return tuple(self.resolve(d, context, phase) for d in descriptors)


@dataclass(frozen=True, slots=True)
class OptimizationReport:
    """Resolved implementations of a model for one input shape
    (reference optimization/report.py)."""

    policies: tuple[str, ...]
    context: ExecutionContext
    decisions: tuple[PolicyDecision, ...]
    warnings: tuple[str, ...] = ()

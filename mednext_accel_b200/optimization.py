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
from dataclasses import dataclass, field, fields
from math import prod
from types import MappingProxyType
from typing import Literal, NamedTuple

ExecutionPhase = Literal["training", "inference", "export"]
SemanticEquivalence = Literal["exact", "numerical", "approximate"]
Confidence = Literal["guard", "fixed-table", "measured-exact-context"]
SM100 = (10, 0)


# --------------------------------------------------------------------------- descriptors
_CONV_GEOMETRY = ("kernel_size", "stride", "padding", "dilation", "groups")
_PHASES = ("training", "inference", "export")
_EQUIVALENCES = ("exact", "numerical", "approximate")


def _extents(value: object, field_name: str, least: int) -> tuple[int, ...]:
    """Normalise a 2-D or 3-D extent (kernel, stride, padding, ...) to a tuple.

    Raises ValueError naming ``field_name`` when the value is not two or three
    plain integers or when an entry is below ``least``."""
    try:
        dims = tuple(value)  # type: ignore[arg-type]
    except TypeError:
        dims = ()
    if len(dims) not in (2, 3) or not all(type(v) is int for v in dims):
        raise ValueError(f"{field_name}: expected two or three integers, got {value!r}")
    if min(dims) < least:
        raise ValueError(f"{field_name}: every entry must be at least {least}, got {value!r}")
    return dims


@dataclass(frozen=True, slots=True)
class OperatorDescriptor:
    """What an optimizable operator is, independent of the input's size.

    Convolutions carry their full geometry (all five geometry fields, or none for
    operators such as normalisations).  ``expansion_ratio`` is set on MedNeXt
    block descriptors, whose table rows are keyed on it."""

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
        if not (self.family and self.direction):
            raise ValueError("an operator needs a non-empty family and direction")
        if self.in_channels <= 0 or self.out_channels <= 0:
            bad = "in_channels" if self.in_channels <= 0 else "out_channels"
            raise ValueError(f"{bad} must be positive")
        given = [getattr(self, f) is not None for f in _CONV_GEOMETRY]
        if not any(given):
            return
        if not all(given):
            missing = [f for f, g in zip(_CONV_GEOMETRY, given, strict=True) if not g]
            raise ValueError(f"convolution geometry is incomplete: missing {', '.join(missing)}")
        if self.groups <= 0:  # type: ignore[operator]
            raise ValueError("groups must be positive")
        for name, least in (("kernel_size", 1), ("stride", 1), ("padding", 0), ("dilation", 1)):
            object.__setattr__(self, name, _extents(getattr(self, name), name, least))

    @classmethod
    def normalization(cls, *, family: str, channels: int, role: str | None = None) -> OperatorDescriptor:
        """A shape-preserving per-channel operator (GroupNorm, GRN)."""
        return cls(family=family, direction="regular", in_channels=channels, out_channels=channels, role=role)

    @classmethod
    def convolution(cls, *, family: str, direction: str, in_channels: int, out_channels: int,
                    kernel_size: tuple[int, ...], stride: tuple[int, ...], padding: tuple[int, ...],
                    dilation: tuple[int, ...], groups: int, role: str | None = None) -> OperatorDescriptor:
        return cls(family=family, direction=direction, in_channels=in_channels, out_channels=out_channels,
                   kernel_size=kernel_size, stride=stride, padding=padding, dilation=dilation, groups=groups,
                   role=role)

    @property
    def is_convolution(self) -> bool:
        return self.kernel_size is not None

    @property
    def signature(self) -> tuple[object, ...]:
        return (self.family, self.direction, self.in_channels, self.out_channels, self.kernel_size, self.stride)

    def to_primitive(self) -> dict[str, object]:
        out: dict[str, object] = {}
        for f in fields(self):
            v = getattr(self, f.name)
            if isinstance(v, tuple):
                v = list(v)
            if v is not None or self.is_convolution and f.name in _CONV_GEOMETRY + ("role",):
                out[f.name] = v
        return out


@dataclass(frozen=True, slots=True)
class ExecutionContext:
    """The run-time facts a decision depends on: phase, device, dtype, shapes."""

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
        if self.phase not in _PHASES:
            raise ValueError(f"unknown phase {self.phase!r} (expected one of {', '.join(_PHASES)})")
        if self.batch_size < 1:
            raise ValueError(f"batch_size must be positive, got {self.batch_size}")
        if self.total_vram_bytes < 0:
            raise ValueError("total_vram_bytes cannot be negative")
        object.__setattr__(self, "spatial_shape", _extents(self.spatial_shape, "spatial_shape", 1))
        if self.sm is not None:
            sm = tuple(self.sm)
            if len(sm) != 2 or min(sm) < 0:
                raise ValueError(f"sm must be a (major, minor) pair of non-negative integers, got {self.sm!r}")
            object.__setattr__(self, "sm", sm)

    @property
    def spatial_volume(self) -> int:
        return prod(self.spatial_shape)

    @property
    def total_vram_gib(self) -> float:
        return self.total_vram_bytes / float(1 << 30)

    def to_primitive(self) -> dict[str, object]:
        out = {f.name: getattr(self, f.name) for f in fields(self)}
        out["spatial_shape"] = list(self.spatial_shape)
        out["sm"] = list(self.sm) if self.sm is not None else None
        return out


EligibilityGuard = Callable[[OperatorDescriptor, ExecutionContext, str], "str | None"]


@dataclass(frozen=True, slots=True)
class ImplementationSpec:
    """Static facts about one implementation id: what it covers and how exact it is."""

    identifier: str
    version: int
    families: tuple[str, ...]
    phases: tuple[str, ...]
    equivalence: SemanticEquivalence
    export_safe: bool

    def __post_init__(self) -> None:
        if not self.identifier:
            raise ValueError("an implementation needs an identifier")
        if self.version < 1:
            raise ValueError(f"implementation {self.identifier!r}: version must be at least 1")
        object.__setattr__(self, "families", tuple(self.families))
        object.__setattr__(self, "phases", tuple(self.phases))
        if not (self.families and self.phases):
            raise ValueError(f"implementation {self.identifier!r} lists no families or no phases")
        if self.equivalence not in _EQUIVALENCES:
            raise ValueError(f"implementation {self.identifier!r}: unknown equivalence {self.equivalence!r}")

    def is_allowed(self, *, allow_approximate: bool, export: bool = False) -> bool:
        if export and not self.export_safe:
            return False
        return allow_approximate or self.equivalence != "approximate"


class _Registration(NamedTuple):
    spec: ImplementationSpec
    eligibility: EligibilityGuard | None
    execution_guards: tuple[str, ...]


class ImplementationRegistry:
    """Implementation ids -> (spec, eligibility guard, execution guards)."""

    def __init__(self) -> None:
        self._entries: dict[str, _Registration] = {}

    def register(self, spec: ImplementationSpec, *, eligibility: EligibilityGuard | None = None,
                 execution_guards: tuple[str, ...] = ()) -> None:
        if spec.identifier in self._entries:
            raise ValueError(f"duplicate implementation id {spec.identifier!r}")
        self._entries[spec.identifier] = _Registration(spec, eligibility, tuple(execution_guards))

    def _entry(self, identifier: str) -> _Registration:
        entry = self._entries.get(identifier)
        if entry is None:
            raise ValueError(f"no implementation is registered as {identifier!r}")
        return entry

    def resolve_metadata(self, identifier: str) -> ImplementationSpec:
        return self._entry(identifier).spec

    def guard(self, identifier: str, descriptor: OperatorDescriptor, context: ExecutionContext,
              phase: str) -> str | None:
        check = self._entry(identifier).eligibility
        return check(descriptor, context, phase) if check is not None else None

    def execution_guards(self, identifier: str) -> tuple[str, ...]:
        return self._entry(identifier).execution_guards

    def __contains__(self, identifier: object) -> bool:
        return identifier in self._entries

    def __iter__(self):
        return (entry.spec for entry in self._entries.values())


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


def _grn_eligibility(descriptor: OperatorDescriptor, context: ExecutionContext, phase: str) -> str | None:
    if context.phase != "training" or phase != "training":
        return "implementation requires training"
    if context.device_type != "cuda":
        return "implementation requires CUDA"
    if context.dtype not in ("float16", "bfloat16", "float32"):
        return "implementation does not support this dtype"
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
        ("sm100_grn", ("global_response_norm3d",), ("training",), "numerical", False, _grn_eligibility,
         ("grad_enabled", "rank_5", "contiguous")),
        ("triton_fused_grn", ("global_response_norm3d",), ("training",), "numerical", False, _grn_eligibility,
         ("grad_enabled", "rank_5", "contiguous")),
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
        "triton_fused_grn": "sm100_grn",
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
    """One row per MedNeXt v1 regular-block shape (channels, ratio, kernel, spatial at a
    128^3 input), whose parameters are the launch choices the kernels make for it
    (depthwise kernel family and tiling, fused GEMM backward variants, whether the
    expand GEMM stores GELU(u)), each citing the profile that justifies it.  The
    choices are committed as data in :mod:`.sm100_table` and pinned to the
    library's planners by tests."""
    from .sm100_table import SM100_BLOCK_TABLE

    return tuple(
        TableRow(f"block-c{c}-r{r}-k{k}-s{s}", "mednext_block3d", "regular", "sm100_fused_block",
                 channels=c, ratio=r, kernel=k, spatial=s, parameters=plan)
        for (c, r, k, s), plan in SM100_BLOCK_TABLE.items()
    )


SM100_TABLE: tuple[TableRow, ...] = (
    *_block_rows(),
    TableRow("block-regular", "mednext_block3d", "regular", "sm100_fused_block"),
    TableRow("block-down", "mednext_block3d", "downsample", "sm100_fused_block"),
    TableRow("block-up", "mednext_block3d", "transpose", "sm100_fused_block"),
    TableRow("depthwise-regular", "depthwise_conv3d", "regular", "sm100_depthwise"),
    TableRow("depthwise-downsample", "depthwise_conv3d", "downsample", "sm100_depthwise_downsample"),
    TableRow("depthwise-transpose", "depthwise_conv_transpose3d", "transpose", "sm100_depthwise_transpose"),
    TableRow("pointwise", "pointwise_conv3d", "regular", "sm100_pointwise"),
    TableRow("grn", "global_response_norm3d", "regular", "sm100_grn"),
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

"""sm_100a (B200) MedNeXt training operators behind the mednext-accel API.

Public names mirror the reference package ``mednext_accel``: the v1 factories,
``MedNeXtV1`` / ``MedNeXtV1Config`` / ``get_mednext_v1_config``,
``CheckpointConfig``, the adaptive operator wrappers and the
``PolicyResolver`` / ``PolicyDecision`` selection API.  The CUDA kernels live in
``lib/libmednext_b200.so`` (C ABI declared in ``include/mednext_b200.h``) and are
loaded on first use.
"""

from .adaptive import (
    AdaptiveDepthwise3d,
    AdaptivePointwise3d,
    ModelOptimizationContext,
    install_adaptive_operators,
)
from .grn import (
    AdaptiveGlobalResponseNorm3d,
    GlobalResponseNorm3d,
    fused_global_response_norm3d,
    global_response_norm3d_reference,
    install_adaptive_grn,
)
from .loss import cross_entropy
from .network import (
    CheckpointConfig,
    MedNeXtBlock,
    MedNeXtDownBlock,
    MedNeXtUpBlock,
    MedNeXtV1,
    MedNeXtV1Config,
    OutputHead,
    get_mednext_v1_config,
    mednext_base,
    mednext_large,
    mednext_medium,
    mednext_small,
)
from .optimization import (
    ExecutionContext,
    ImplementationRegistry,
    ImplementationSpec,
    OperatorDescriptor,
    OptimizationReport,
    PolicyDecision,
    PolicyResolver,
    default_implementation_registry,
)

__version__ = "0.1.0"

__all__ = [
    "AdaptiveDepthwise3d",
    "AdaptiveGlobalResponseNorm3d",
    "GlobalResponseNorm3d",
    "fused_global_response_norm3d",
    "global_response_norm3d_reference",
    "install_adaptive_grn",
    "AdaptivePointwise3d",
    "CheckpointConfig",
    "ExecutionContext",
    "ImplementationRegistry",
    "ImplementationSpec",
    "MedNeXtBlock",
    "MedNeXtDownBlock",
    "MedNeXtUpBlock",
    "MedNeXtV1",
    "MedNeXtV1Config",
    "ModelOptimizationContext",
    "OperatorDescriptor",
    "OptimizationReport",
    "OutputHead",
    "PolicyDecision",
    "PolicyResolver",
    "cross_entropy",
    "default_implementation_registry",
    "get_mednext_v1_config",
    "install_adaptive_operators",
    "mednext_base",
    "mednext_large",
    "mednext_medium",
    "mednext_small",
]

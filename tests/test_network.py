"""Network structure, initialisation and CPU numerics match the reference
package (pinned by golden fixtures produced from the reference itself)."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch
from torch.nn import functional as F

import mednext_accel_b200 as mx
from mednext_accel_b200.adaptive import AdaptiveDepthwise3d, AdaptivePointwise3d, ModelOptimizationContext
from mednext_accel_b200.optimization import (
    LEGACY_ALIASES,
    ExecutionContext,
    OperatorDescriptor,
    PolicyResolver,
    default_implementation_registry,
)
from tests.conftest import GOLDEN


def test_base_parameter_count_matches_reference():
    model = mx.mednext_base(in_channels=1, out_channels=3, deep_supervision=True)
    assert sum(p.numel() for p in model.parameters()) == 10_529_231


def test_state_dict_keys_and_seeded_init_match_reference():
    ref = json.loads((GOLDEN / "model_init.json").read_text())
    torch.manual_seed(0)
    model = mx.mednext_base(in_channels=1, out_channels=3, deep_supervision=True)
    state = model.state_dict()
    assert list(state) == ref["keys"]
    assert sum(p.numel() for p in model.parameters()) == ref["parameters"]
    for key, (s, sq, head) in ref["checksums"].items():
        v = state[key].double()
        assert float(v.sum()) == pytest.approx(s, rel=1e-12, abs=1e-12), key
        assert float((v**2).sum()) == pytest.approx(sq, rel=1e-12, abs=1e-12), key
        assert [float(a) for a in v.flatten()[:4]] == head, key


@pytest.mark.parametrize("factory", [mx.mednext_small, mx.mednext_base, mx.mednext_medium, mx.mednext_large])
def test_factories_build_declared_variant(factory):
    model = factory(in_channels=1, out_channels=3, base_channels=2)
    assert isinstance(model, mx.MedNeXtV1)
    assert model.config.variant in factory.__name__


def test_cpu_forward_backward_matches_reference_small_model(golden):
    g = golden("small_model.npz")
    torch.manual_seed(0)
    model = mx.mednext_small(in_channels=1, out_channels=3, base_channels=4, deep_supervision=True).double().train()
    for name, p in model.named_parameters():
        np.testing.assert_array_equal(p.detach().numpy(), g[f"param/{name}"], err_msg=name)
    x = torch.from_numpy(g["x"])
    target = torch.from_numpy(g["target"])
    heads = model(x)
    loss = sum(
        F.cross_entropy(h, target if h.shape[2:] == target.shape[1:] else
                        F.interpolate(target[:, None].double(), size=h.shape[2:], mode="nearest")[:, 0].long())
        for h in heads
    ) / len(heads)
    loss.backward()
    assert loss.item() == pytest.approx(float(g["loss"][0]), rel=1e-12)
    for i, h in enumerate(heads):
        np.testing.assert_allclose(h.detach().numpy(), g[f"head{i}"], rtol=1e-10, atol=1e-12)
    for name, p in model.named_parameters():
        np.testing.assert_allclose(p.grad.numpy(), g[f"grad/{name}"], rtol=1e-8, atol=1e-12, err_msg=name)


def test_installation_preserves_parameters_and_state_dict_keys():
    model = torch.nn.Sequential(torch.nn.Conv3d(32, 32, 3, padding=1, groups=32), torch.nn.Conv3d(32, 64, 1))
    params = tuple(model.parameters())
    keys = tuple(model.state_dict())
    count = mx.install_adaptive_operators(
        model, resolver=PolicyResolver(), model_context=ModelOptimizationContext("mednext_v1", "base", "none")
    )
    assert count == 2
    assert tuple(model.parameters()) == params
    assert tuple(model.state_dict()) == keys
    assert isinstance(model[0], AdaptiveDepthwise3d)
    assert isinstance(model[1], AdaptivePointwise3d)


def test_blocks_get_fused_runner_and_keep_keys():
    model = mx.mednext_small(in_channels=1, out_channels=3, base_channels=4)
    ref = mx.mednext_small(in_channels=1, out_channels=3, base_channels=4, optimization="reference")
    assert list(model.state_dict()) == list(ref.state_dict())
    blocks = [m for m in model.modules() if isinstance(m, mx.MedNeXtBlock)]
    assert blocks and all(b._fused is not None for b in blocks)
    assert all(m._fused is None for m in ref.modules() if isinstance(m, mx.MedNeXtBlock))


def test_cpu_forward_uses_reference_path_and_matches():
    torch.manual_seed(3)
    ref = mx.mednext_small(in_channels=1, out_channels=3, base_channels=4, optimization="reference").double()
    cand = mx.mednext_small(in_channels=1, out_channels=3, base_channels=4).double()
    cand.load_state_dict(ref.state_dict())
    x = torch.randn(1, 1, 32, 32, 32, dtype=torch.float64)
    torch.testing.assert_close(cand(x), ref(x))


def _ctx(sm=(10, 0), device="cuda", dtype="bfloat16", spatial=(128, 128, 128), phase="training"):
    return ExecutionContext(phase, device, sm, 180 << 30, dtype, 1, spatial, "mednext_v1", "base", "none")


def _dw(direction="regular", c=32, k=3):
    stride = (2, 2, 2) if direction != "regular" else (1, 1, 1)
    fam = "depthwise_conv_transpose3d" if direction == "transpose" else "depthwise_conv3d"
    return OperatorDescriptor(fam, direction, c, c, (k,) * 3, stride, (k // 2,) * 3, (1, 1, 1), c)


def test_resolver_selects_sm100_kernels_on_b200():
    r = PolicyResolver()
    for direction, impl in (("regular", "sm100_depthwise"), ("downsample", "sm100_depthwise_downsample"),
                            ("transpose", "sm100_depthwise_transpose")):
        for phase in ("backward_input", "backward_weight"):
            d = r.resolve(_dw(direction), _ctx(), phase)
            assert d.implementation == impl and d.disposition == "custom" and d.guard_reason is None
    pw = OperatorDescriptor("pointwise_conv3d", "regular", 32, 64, (1, 1, 1), (1, 1, 1), (0, 0, 0), (1, 1, 1), 1)
    assert r.resolve(pw, _ctx(), "training").implementation == "sm100_pointwise"
    # fp32 compute has no tensor-core pointwise: guarded back to the reference
    d = r.resolve(pw, _ctx(dtype="float32"), "training")
    assert d.implementation == "reference" and d.guard_reason


def test_resolver_guards_other_contexts():
    r = PolicyResolver()
    assert r.resolve(_dw(), _ctx(device="cpu", sm=None), "backward_input").implementation == "reference"
    with pytest.warns(UserWarning):
        d = r.resolve(_dw(), _ctx(sm=(12, 0)), "backward_input")
    assert d.implementation == "reference"
    d = r.resolve(_dw(), _ctx(phase="inference"), "backward_input")
    assert d.implementation == "reference" and "training" in d.guard_reason
    d = r.resolve(_dw(k=4), _ctx(), "backward_input")
    assert d.implementation == "reference"


def test_reference_implementation_ids_still_resolve():
    reg = default_implementation_registry()
    for ident in ("reference", "pointwise_gemm_per_sample", "triton_depthwise_dx", "triton_split_dw",
                  "triton_transpose_split_dw", "triton_downsample_dx", "gelu_tanh"):
        assert ident in reg
    r = PolicyResolver(overrides={("depthwise_conv3d", "regular"): "triton_split_dw"})
    d = r.resolve(_dw(), _ctx(), "backward_weight")
    assert d.implementation == LEGACY_ALIASES["triton_split_dw"] == "sm100_depthwise"


def test_checkpoint_config_validation():
    with pytest.raises(ValueError):
        mx.CheckpointConfig(style="nope")
    with pytest.raises(ValueError):
        mx.CheckpointConfig(stages=(5,))
    assert mx.CheckpointConfig(stages=(1, 0)).stages == (0, 1)
    with pytest.raises(ValueError):
        mx.mednext_base(in_channels=1, out_channels=3, optimization="autotune")


# ---- public configuration API (the reference's tests/test_public_api.py:8-53 and
# tests/optimization/test_descriptors.py, test_implementations.py pin these)
def test_v1_config_downsample_ratios_follow_compatibility():
    from mednext_accel_b200.network import get_mednext_v1_config

    official = get_mednext_v1_config("base", in_channels=1, out_channels=3)
    assert official.block_counts == (2,) * 9
    assert official.expansion_ratios == (2, 3, 4, 4, 4, 4, 4, 3, 2)
    assert official.downsample_expansion_ratios == (3, 4, 4, 4)
    monai = get_mednext_v1_config("base", in_channels=1, out_channels=3, compatibility="monai")
    assert monai.downsample_expansion_ratios == (2, 3, 4, 4)
    with pytest.raises(ValueError, match="variant"):
        get_mednext_v1_config("huge", in_channels=1, out_channels=3)


@pytest.mark.parametrize("stages, message", [((0, 0), "duplicates"), ((-1,), "between 0 and 4"),
                                             ((5,), "between 0 and 4"), ((1.0,), "integers")])
def test_checkpoint_stages_are_validated(stages, message):
    with pytest.raises(ValueError, match=message):
        mx.CheckpointConfig(stages=stages)


def test_checkpoint_config_canonicalises_and_reports_style():
    cfg = mx.CheckpointConfig(style="block", stages=(2, 0, 1))
    assert cfg.stages == (0, 1, 2) and cfg.checkpoints_blocks and not cfg.checkpoints_expansion
    assert cfg.includes(1) and not cfg.includes(3)
    assert mx.CheckpointConfig().includes(4)
    with pytest.raises(ValueError, match="style"):
        mx.CheckpointConfig(style="whole")


def test_descriptor_validation_and_primitive_form():
    from mednext_accel_b200.optimization import ExecutionContext, OperatorDescriptor

    with pytest.raises(ValueError, match="kernel_size"):
        OperatorDescriptor.convolution(family="depthwise_conv3d", direction="regular", in_channels=4,
                                       out_channels=4, kernel_size=(0, 0, 0), stride=(1, 1, 1),
                                       padding=(1, 1, 1), dilation=(1, 1, 1), groups=4)
    with pytest.raises(ValueError, match="geometry"):
        OperatorDescriptor("depthwise_conv3d", "regular", 4, 4, kernel_size=(3, 3, 3))
    norm = OperatorDescriptor.normalization(family="global_response_norm3d", channels=96,
                                            role="encoder_stages.0.0.grn")
    assert norm.to_primitive() == {"family": "global_response_norm3d", "direction": "regular",
                                   "in_channels": 96, "out_channels": 96, "role": "encoder_stages.0.0.grn"}
    conv = OperatorDescriptor.convolution(family="depthwise_conv3d", direction="regular", in_channels=4,
                                          out_channels=4, kernel_size=[3, 3, 3], stride=(1, 1, 1),
                                          padding=(1, 1, 1), dilation=(1, 1, 1), groups=4)
    assert conv.kernel_size == (3, 3, 3)
    assert conv.to_primitive()["kernel_size"] == [3, 3, 3] and conv.to_primitive()["role"] is None
    with pytest.raises(ValueError, match="batch_size"):
        ExecutionContext("training", "cpu", None, 0, "float32", 0, (8, 8, 8), "mednext_v1", "base", "none")
    ctx = ExecutionContext("training", "cuda", (10, 0), 32 << 30, "bfloat16", 3, (128, 128, 128),
                           "mednext_v1", "base", "all-expansion")
    assert ctx.spatial_volume == 128**3 and ctx.total_vram_gib == 32


def test_registry_rejects_duplicates_and_names_unknown_ids():
    from mednext_accel_b200.optimization import (ImplementationRegistry, ImplementationSpec,
                                                  default_implementation_registry)

    reg = ImplementationRegistry()
    spec = ImplementationSpec("reference", 1, ("pointwise_conv3d",), ("training",), "exact", True)
    reg.register(spec)
    with pytest.raises(ValueError, match="reference"):
        reg.register(spec)
    with pytest.raises(ValueError, match="missing_backend"):
        reg.resolve_metadata("missing_backend")
    approx = ImplementationSpec("gelu_tanh", 1, ("gelu",), ("inference",), "approximate", True)
    assert not approx.is_allowed(allow_approximate=False) and approx.is_allowed(allow_approximate=True)
    assert default_implementation_registry().resolve_metadata("triton_split_dw").identifier == "triton_split_dw"


def test_grn_layer_reference_formula_and_argument_contract():
    """GRN starts as the identity (zero gamma/beta, ops/grn.py:32-46) and the fused
    entry point rejects what the reference's rejects, with its messages
    (ops/_triton/grn.py:416-437, tests/ops/test_grn_triton.py:116)."""
    layer = mx.GlobalResponseNorm3d(6)
    x = torch.randn(2, 6, 3, 4, 5)
    assert torch.equal(layer(x), x)
    assert tuple(layer.gamma.shape) == (1, 6, 1, 1, 1) and tuple(layer.beta.shape) == (1, 6, 1, 1, 1)
    with pytest.raises(ValueError, match="GRN expects an NCDHW tensor"):
        mx.global_response_norm3d_reference(torch.randn(2, 6, 3), layer.gamma, layer.beta)
    with pytest.raises(ValueError, match="channels"):
        mx.GlobalResponseNorm3d(0)
    with pytest.raises(ValueError, match="eps"):
        mx.GlobalResponseNorm3d(4, eps=float("nan"))
    with pytest.raises(ValueError, match="^fused GRN requires CUDA tensors$"):
        mx.fused_global_response_norm3d(x, layer.gamma, layer.beta)
    with pytest.raises(ValueError, match="rank-5"):
        mx.fused_global_response_norm3d(torch.randn(2, 6, 3), layer.gamma, layer.beta)

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

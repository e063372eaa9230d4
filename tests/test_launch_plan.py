"""The fixed sm_100a launch table against the library's planners (CPU only).

``mednext_accel_b200/sm100_table.py`` records, for every MedNeXt v1 regular-block
shape (channels, expansion ratio, kernel, spatial size at a 128^3 input), the
launch choices of the sm_100a kernels: the depthwise kernel family and tiling of
the forward / input grad and of the weight grad, the fused GEMM backward
variants, and whether the expand GEMM stores GELU(u).  These tests regenerate it
from the host-side planners (``mednext_dw_plan``, the fused GEMMs' workspace
queries), check that every choice cites a committed profile, and that the policy
resolver hands a block exactly its row."""

from __future__ import annotations

from pathlib import Path

from mednext_accel_b200 import launch_plan
from mednext_accel_b200.optimization import ExecutionContext, OperatorDescriptor, PolicyResolver, SM100_TABLE
from mednext_accel_b200.sm100_table import SM100_BLOCK_TABLE

ROOT = Path(__file__).resolve().parents[1]


def test_committed_table_is_what_the_planners_choose():
    committed = (ROOT / "mednext_accel_b200" / "sm100_table.py").read_text()
    assert committed == launch_plan.emit_table(), (
        "the kernels' planners changed: regenerate with python -m mednext_accel_b200.launch_plan")


def test_table_covers_every_mednext_v1_block_shape():
    assert sorted(SM100_BLOCK_TABLE) == launch_plan.mednext_block_shapes()
    # Base k3 and Large k5 level-0 rows: the measured families of the step profiles
    assert SM100_BLOCK_TABLE[(32, 2, 3, 128)]["depthwise_forward"]["family"] == "packed-fma"
    assert SM100_BLOCK_TABLE[(32, 3, 5, 128)]["depthwise_forward"]["family"] == "tensor-cores"
    assert SM100_BLOCK_TABLE[(32, 3, 5, 128)]["depthwise_weight_grad"]["family"] == "grouped-tma-ring"


def test_every_choice_cites_a_committed_profile():
    for plan in SM100_BLOCK_TABLE.values():
        for key in ("depthwise_forward", "depthwise_weight_grad"):
            assert (ROOT / "profiles" / plan[key]["profile"]).is_file(), plan[key]["profile"]
        assert (ROOT / "profiles" / plan["gemm_profile"]).is_file()


def test_resolver_hands_a_block_its_row():
    resolver = PolicyResolver()
    rows = {row.rule: row for row in SM100_TABLE}
    for (c, r, k, s), plan in SM100_BLOCK_TABLE.items():
        desc = OperatorDescriptor(family="mednext_block3d", direction="regular", in_channels=c, out_channels=c,
                                  kernel_size=(k, k, k), stride=(1, 1, 1), padding=(k // 2,) * 3,
                                  dilation=(1, 1, 1), groups=c, expansion_ratio=r)
        ctx = ExecutionContext(phase="training", device_type="cuda", sm=(10, 0), total_vram_bytes=180 << 30,
                               dtype="bfloat16", batch_size=1, spatial_shape=(s, s, s), model_family="mednext_v1",
                               variant="base", checkpointing="none")
        decision = resolver.resolve(desc, ctx, "training")
        assert decision.implementation == "sm100_fused_block"
        assert decision.rule == f"block-c{c}-r{r}-k{k}-s{s}"
        assert dict(decision.parameters) == plan == dict(rows[decision.rule].parameters)

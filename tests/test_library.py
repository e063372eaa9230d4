"""The C-ABI library loads, exports every symbol include/mednext_b200.h declares,
and rejects bad arguments with status codes before touching the GPU."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from mednext_accel_b200 import _native as nat

HEADER = Path(__file__).resolve().parents[1] / "include" / "mednext_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(mednext_[a-zA-Z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_functions() == sorted(nat.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = nat.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.mednext_abi_version() == 1


def test_library_is_the_in_tree_build():
    assert nat.library_path() == nat.LIB_PATH
    maps = Path("/proc/self/maps").read_text()
    nat.load()
    maps = Path("/proc/self/maps").read_text()
    assert str(nat.LIB_PATH) in maps


def test_status_strings():
    for code in range(9):
        assert nat.status_string(code)
    assert "kernel_size" in nat.status_string(nat.ERR_BAD_KERNEL)


def test_argument_validation_without_gpu():
    lib = nat.load()
    fake = 1 << 20  # never dereferenced: validation fails first
    # even kernel size
    assert lib.mednext_dw_fwd(fake, fake, None, fake, None, 0.0, None, 0, 1, 4, 8, 8, 8, 4, 1, None) == nat.ERR_BAD_KERNEL
    # bad dtype
    assert lib.mednext_dw_dgrad(fake, fake, None, fake, 1, 4, 8, 8, 8, 3, 9, None) == nat.ERR_BAD_DTYPE
    # null pointer
    assert lib.mednext_dw_dgrad(None, fake, None, fake, 1, 4, 8, 8, 8, 3, 1, None) == nat.ERR_NULL_POINTER
    # non-positive size
    assert lib.mednext_dw_s2_fwd(fake, fake, None, fake, 0, 4, 8, 8, 8, 3, 1, None) == nat.ERR_BAD_SHAPE
    # misaligned vector operand
    assert lib.mednext_dw_fwd(fake + 2, fake, None, fake, None, 0.0, None, 0, 1, 4, 8, 8, 8, 3, 1, None) == nat.ERR_ALIGNMENT
    # missing workspace
    assert lib.mednext_dw_wgrad(fake, fake, fake, None, None, 0, 1, 4, 8, 8, 8, 3, 1, None) == nat.ERR_WORKSPACE
    small = lib.mednext_dw_wgrad_workspace_size(1, 4, 8, 8, 8, 3, 1)
    assert small > 0
    assert lib.mednext_dw_wgrad(fake, fake, fake, None, fake, small - 1, 1, 4, 8, 8, 8, 3, 1, None) == nat.ERR_WORKSPACE
    # tensor-core pointwise accepts only 16-bit operands
    assert lib.mednext_pw_fwd(fake, fake, fake, 0, None, None, None, 0, None, None, None, None, None, 0,
                              1, 32, 64, 4096, nat.dtype_code(__import__("torch").float32), 0, None) == nat.ERR_BAD_DTYPE
    # GroupNorm prologue needs its statistics
    assert lib.mednext_pw_fwd(fake, fake, fake, nat.PRO_GROUPNORM, None, None, None, 0, None, None, None, None, None, 0,
                              1, 32, 64, 4096, 1, 1, None) == nat.ERR_NULL_POINTER
    assert lib.mednext_pw_wgrad(fake, fake, fake, None, 0, None, None, None, None, 0, 1, 32, 64, 4096, 1, None) == nat.ERR_WORKSPACE
    assert lib.mednext_gn_stats(fake, fake, None, 0, 1, 4, 512, 0, 1e-5, 1, None) == nat.ERR_WORKSPACE
    code = ctypes.c_int(0)
    assert lib.mednext_device_error(None, None) == nat.ERR_NULL_POINTER


@pytest.mark.parametrize("fn", ["mednext_dw_fwd_workspace_size", "mednext_dw_wgrad_workspace_size",
                                "mednext_dw_s2_wgrad_workspace_size", "mednext_dwT_wgrad_workspace_size"])
def test_workspace_sizes(fn):
    lib = nat.load()
    size = getattr(lib, fn)(1, 32, 128, 128, 128, 3, 1)
    assert 0 < size < 64 << 20
    assert getattr(lib, fn)(1, 32, 128, 128, 128, 4, 1) == 0  # invalid kernel -> 0


def test_pointwise_workspace_sizes():
    lib = nat.load()
    assert lib.mednext_pw_fwd_workspace_size(1, 128, 32, 128**3, 0) == 0
    # one 16-byte partial per (channel, 128-voxel tile, 32-voxel quarter)
    assert lib.mednext_pw_fwd_workspace_size(1, 128, 32, 128**3, nat.EPI_GN_BWD_STATS) == 32 * (128**3 // 128) * 4 * 16
    assert lib.mednext_pw_wgrad_workspace_size(1, 32, 64, 128**3) > 0


@pytest.mark.parametrize("small", [(1, 1, 1), (2, 3, 4), (4, 4, 4), (5, 7, 8), (8, 8, 8), (64, 64, 64), (3, 9, 24)])
@pytest.mark.parametrize("dtype", [0, 1, 2])
def test_transposed_forward_workspace_planning_on_every_grid(small, dtype):
    """The up block's forward-with-statistics workspace query runs the host-side tile
    planner for every grid, including those the packed-FMA kernel declines (small
    W below or not a multiple of 8): it answers a size, never traps."""
    lib = nat.load()
    d, h, w = small
    for pitch in (0, (2 * w - 1 + 7) // 8 * 8):
        for k in (1, 3, 5):
            assert lib.mednext_dwT_fwd_workspace_size(2, 6, d, h, w, pitch, k, dtype) > 0
    if w > 1:  # a pitch below the row length is rejected
        assert lib.mednext_dwT_fwd_workspace_size(2, 6, d, h, w, 2 * w - 2, 3, dtype) == 0


@pytest.mark.parametrize("shape", [(1, 32, 128, 128, 128), (2, 5, 17, 33, 48), (1, 3, 6, 40, 256), (1, 1, 1, 1, 16),
                                   (1, 2, 3, 4, 8), (1, 256, 16, 16, 16)])
@pytest.mark.parametrize("k", [1, 3, 5, 7])
def test_depthwise_forward_workspace_planning(shape, k):
    """The stride-1 forward's workspace query runs the host-side tile planners (the
    packed-FMA and, for k = 5 / 7 on 16-bit types, the tensor-core one) on every
    grid: it answers a size, never traps."""
    lib = nat.load()
    for dtype in (0, 1, 2):
        assert lib.mednext_dw_fwd_workspace_size(*shape, k, dtype) > 0

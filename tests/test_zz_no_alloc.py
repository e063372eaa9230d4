"""mednext_dw_wgrad_noalloc (depthwise weight grad with built-in scratch) through
the C ABI, against mednext_dw_wgrad with a caller workspace.

Collected last so that it also runs after every other test has used the
library.  Each case calls the no-allocation entry point twice in a row, with
scratch left over from the previous case, and compares both results with the
workspace entry point within the depthwise tests' tolerances."""

from __future__ import annotations

import pytest
import torch

from mednext_accel_b200 import _native as nat

pytestmark = pytest.mark.gpu

# depthwise tolerances: fp32 max relative 1e-5; 16-bit outputs to their rounding
TOL = {
    torch.float64: dict(rtol=1e-12, atol=1e-12),
    torch.float32: dict(rtol=1e-5, atol=1e-6),
    torch.bfloat16: dict(rtol=1.6e-2, atol=1e-2),
    torch.float16: dict(rtol=2e-3, atol=1e-3),
}

CASES = [
    (torch.float32, 3, (1, 8, 9, 10, 11)),
    (torch.bfloat16, 3, (1, 32, 64, 64, 64)),
    (torch.bfloat16, 5, (2, 16, 16, 16, 16)),
    (torch.float16, 7, (1, 32, 24, 24, 24)),
    (torch.float64, 3, (1, 4, 8, 8, 8)),
    (torch.bfloat16, 7, (2, 32, 64, 64, 64)),
    (torch.float32, 1, (1, 16, 16, 16, 16)),
]


def _inputs(dtype, shape, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(shape, generator=gen, device="cuda", dtype=torch.float32).to(dtype)
    dy = torch.randn(shape, generator=gen, device="cuda", dtype=torch.float32).to(dtype)
    return x, dy


def _outputs(x, k):
    c = x.shape[1]
    return (torch.full((c, 1, k, k, k), float("nan"), device="cuda", dtype=x.dtype),
            torch.full((c,), float("nan"), device="cuda", dtype=x.dtype))


def with_workspace(x, dy, k):
    lib = nat.load()
    dw, db = _outputs(x, k)
    code = nat.dtype_code(x.dtype)
    ws = nat.workspace(lib.mednext_dw_wgrad_workspace_size(*x.shape, k, code), x.device)
    nat.check(lib.mednext_dw_wgrad(x.data_ptr(), dy.data_ptr(), dw.data_ptr(), db.data_ptr(), ws.data_ptr(),
                                   ws.numel(), *x.shape, k, code, nat.stream()), "mednext_dw_wgrad")
    return dw, db


def no_alloc(x, dy, k, bias=True):
    dw, db = _outputs(x, k)
    status = nat.load().mednext_dw_wgrad_noalloc(x.data_ptr(), dy.data_ptr(), dw.data_ptr(),
                                                 db.data_ptr() if bias else None, *x.shape, k,
                                                 nat.dtype_code(x.dtype), nat.stream())
    nat.check(status, "mednext_dw_wgrad_noalloc")
    return dw, db


@pytest.mark.parametrize("dtype,k,shape", CASES)
def test_no_alloc_matches_workspace_entry_point_twice(dtype, k, shape):
    x, dy = _inputs(dtype, shape, seed=sum(shape) * 10 + k)
    want_dw, want_db = with_workspace(x, dy, k)
    first = no_alloc(x, dy, k)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    second = no_alloc(x, dy, k)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before  # the call after set-up takes no device memory
    for dw, db in (first, second):
        torch.testing.assert_close(dw, want_dw, **TOL[dtype])
        torch.testing.assert_close(db, want_db, **TOL[dtype])


def test_no_alloc_without_bias():
    x, dy = _inputs(torch.bfloat16, (1, 16, 20, 20, 20), seed=3)
    want_dw, _ = with_workspace(x, dy, 3)
    dw, db = no_alloc(x, dy, 3, bias=False)
    torch.cuda.synchronize()
    torch.testing.assert_close(dw, want_dw, **TOL[torch.bfloat16])
    assert torch.isnan(db).all()  # untouched


def test_no_alloc_rejects_shape_beyond_scratch_limit():
    lib = nat.load()
    shape, k = (4, 64, 160, 160, 160), 7  # needs 26.9 MiB
    need = lib.mednext_dw_wgrad_workspace_size(*shape, k, nat.dtype_code(torch.bfloat16))
    assert need > (16 << 20)
    x = torch.zeros(shape, device="cuda", dtype=torch.bfloat16)
    dw, db = _outputs(x, k)
    before = lib.mednext_kernel_launches()
    status = lib.mednext_dw_wgrad_noalloc(x.data_ptr(), x.data_ptr(), dw.data_ptr(), db.data_ptr(), *shape, k,
                                          nat.dtype_code(x.dtype), nat.stream())
    assert status == nat.ERR_SCRATCH_LIMIT
    assert "scratch" in nat.status_string(status)
    assert lib.mednext_kernel_launches() == before
    with pytest.raises(ValueError, match="scratch"):
        nat.check(status, "mednext_dw_wgrad_noalloc")


def test_no_alloc_argument_errors_match_workspace_entry_point():
    lib = nat.load()
    x = torch.zeros((1, 4, 8, 8, 8), device="cuda", dtype=torch.float32)
    dw, db = _outputs(x, 3)
    assert lib.mednext_dw_wgrad_noalloc(x.data_ptr(), x.data_ptr(), dw.data_ptr(), None, 1, 4, 8, 8, 8, 4, 0,
                                        nat.stream()) == nat.ERR_BAD_KERNEL
    assert lib.mednext_dw_wgrad_noalloc(None, x.data_ptr(), dw.data_ptr(), None, 1, 4, 8, 8, 8, 3, 0,
                                        nat.stream()) == nat.ERR_NULL_POINTER
    assert lib.mednext_dw_wgrad_noalloc(x.data_ptr(), x.data_ptr(), dw.data_ptr(), None, 1, 4, 8, 8, 8, 3, 9,
                                        nat.stream()) == nat.ERR_BAD_DTYPE


def test_no_device_error_recorded():
    assert nat.device_error() == 0

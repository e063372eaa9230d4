"""ctypes binding of ``libmednext_b200.so`` (the C ABI in ``include/mednext_b200.h``).

The shared library is built in-tree by :func:`mednext_accel_b200._build.build` and
loaded on first use.  Every wrapper here takes torch tensors that already live on
the current CUDA device, passes raw pointers and sizes to the C entry point on the
current CUDA stream, and converts a non-zero status into an exception:
``ValueError`` for argument errors (the reference raises ``ValueError`` for bad
shapes, dtypes and kernel sizes, ``ops/_triton/depthwise.py:271-286``) and
``RuntimeError`` for launch failures.  There is no fallback: if the library is
missing or the device is not sm_100, the call fails loudly.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_NAME = "libmednext_b200.so"
LIB_PATH = Path(__file__).resolve().parent / "lib" / LIB_NAME

OK = 0
ERR_NULL_POINTER = 1
ERR_BAD_SHAPE = 2
ERR_BAD_KERNEL = 3
ERR_BAD_DTYPE = 4
ERR_WORKSPACE = 5
ERR_ALIGNMENT = 6
ERR_CUDA = 7
ERR_DEVICE = 8
ERR_SCRATCH_LIMIT = 9
ERR_UNSUPPORTED = 10
ERR_BAD_VALUE = 11

PRO_NONE = 0
PRO_GROUPNORM = 1
PRO_GELU = 2
EPI_BIAS = 1
EPI_RESIDUAL = 2
EPI_GELU_GRAD = 4
EPI_GN_BWD_STATS = 8

_DTYPE_CODES = {
    torch.float32: 0,
    torch.bfloat16: 1,
    torch.float16: 2,
    torch.float64: 3,
}

# Every function the header declares, with (restype, argtypes).
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int
_SZ = ctypes.c_size_t
_F = ctypes.c_float
_DIMS5 = [_I64] * 5
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "mednext_abi_version": (_INT, []),
    "mednext_status_string": (ctypes.c_char_p, [_INT]),
    "mednext_last_cuda_error": (_INT, []),
    "mednext_device_error": (_INT, [ctypes.POINTER(_INT), _P]),
    "mednext_check_device": (_INT, []),
    "mednext_kernel_launches": (ctypes.c_uint64, []),
    "mednext_dw_fwd_workspace_size": (_SZ, _DIMS5 + [_INT, _INT]),
    "mednext_dw_fwd": (_INT, [_P, _P, _P, _P, _P, _F, _P, _SZ] + _DIMS5 + [_INT, _INT, _P]),
    "mednext_dw_dgrad": (_INT, [_P, _P, _P, _P] + _DIMS5 + [_INT, _INT, _P]),
    "mednext_dw_wgrad_workspace_size": (_SZ, _DIMS5 + [_INT, _INT]),
    "mednext_dw_wgrad": (_INT, [_P, _P, _P, _P, _P, _SZ] + _DIMS5 + [_INT, _INT, _P]),
    "mednext_dw_wgrad_f32out": (_INT, [_P, _P, _P, _P, _P, _SZ] + _DIMS5 + [_INT, _INT, _P]),
    "mednext_dw_wgrad_noalloc": (_INT, [_P, _P, _P, _P] + _DIMS5 + [_INT, _INT, _P]),
    "mednext_dw_s2_fwd": (_INT, [_P, _P, _P, _P] + _DIMS5 + [_INT, _INT, _P]),
    "mednext_dw_s2_dgrad": (_INT, [_P, _P, _P, _P] + _DIMS5 + [_INT, _INT, _P]),
    "mednext_dw_s2_wgrad_workspace_size": (_SZ, _DIMS5 + [_INT, _INT]),
    "mednext_dw_s2_wgrad": (_INT, [_P, _P, _P, _P, _P, _SZ] + _DIMS5 + [_INT, _INT, _P]),
    "mednext_dw_s2_wgrad_f32out": (_INT, [_P, _P, _P, _P, _P, _SZ] + _DIMS5 + [_INT, _INT, _P]),
    "mednext_dwT_fwd": (_INT, [_P, _P, _P, _P] + _DIMS5 + [_I64, _INT, _INT, _P]),
    "mednext_dwT_fwd_workspace_size": (_SZ, _DIMS5 + [_I64, _INT, _INT]),
    "mednext_dwT_fwd_stats": (_INT, [_P, _P, _P, _P, _P, _F, _P, _SZ] + _DIMS5 + [_I64, _INT, _INT, _P]),
    "mednext_dwT_dgrad": (_INT, [_P, _P, _P, _P] + _DIMS5 + [_I64, _INT, _INT, _P]),
    "mednext_upsample2_fill": (_INT, [_P, _P, _P] + _DIMS5 + [_I64, _INT, _P]),
    "mednext_pad_front_add": (_INT, [_P, _P, _P] + _DIMS5 + [_I64, _INT, _P]),
    "mednext_unpad_front": (_INT, [_P, _P] + _DIMS5 + [_I64, _INT, _P]),
    "mednext_dwT_wgrad_workspace_size": (_SZ, _DIMS5 + [_INT, _INT]),
    "mednext_dwT_wgrad": (_INT, [_P, _P, _P, _P, _P, _SZ] + _DIMS5 + [_I64, _INT, _INT, _P]),
    "mednext_dwT_wgrad_f32out": (_INT, [_P, _P, _P, _P, _P, _SZ] + _DIMS5 + [_I64, _INT, _INT, _P]),
    "mednext_gn_stats_workspace_size": (_SZ, [_I64, _I64, _I64]),
    "mednext_dw_plan": (_INT, _DIMS5 + [_INT, _INT, _INT, _P]),
    "mednext_gn_stats": (_INT, [_P, _P, _P, _SZ, _I64, _I64, _I64, _I64, _F, _INT, _P]),
    "mednext_gn_stats_rows": (_INT, [_P, _P, _P, _SZ, _I64, _I64, _I64, _I64, _I64, _F, _INT, _P]),
    "mednext_gn_fwd": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _INT, _INT, _INT, _P]),
    "mednext_gn_bwd_workspace_size": (_SZ, [_I64, _I64, _I64]),
    "mednext_gn_bwd": (
        _INT,
        [_P, _P, _P, _P, _P, _P, _P, _P, _SZ, _I64, _I64, _I64, _INT, _INT, _INT, _INT, _P],
    ),
    "mednext_pw_fwd_workspace_size": (_SZ, [_I64, _I64, _I64, _I64, _INT]),
    "mednext_pw_fwd": (
        _INT,
        [_P, _P, _P, _INT, _P, _P, _P, _INT, _P, _P, _P, _P, _P, _SZ, _I64, _I64, _I64, _I64, _INT, _INT, _P],
    ),
    "mednext_pw_fwd_pro_out": (
        _INT,
        [_P, _P, _P, _INT, _P, _P, _P, _INT, _P, _P, _P, _P, _P, _P, _SZ, _I64, _I64, _I64, _I64, _INT, _INT, _P],
    ),
    "mednext_pw_fwd_gelu_out": (
        _INT, [_P, _P, _P, _P, _INT, _P, _P, _P, _P, _P, _SZ, _I64, _I64, _I64, _I64, _INT, _P],
    ),
    "mednext_pw_gelu_bwd_workspace_size": (_SZ, [_I64, _I64, _I64, _I64, _INT]),
    "mednext_pw_gelu_bwd": (_INT, [_P, _P, _P, _P, _P, _P, _P, _SZ, _I64, _I64, _I64, _I64, _INT, _P]),
    "mednext_ce_workspace_size": (_SZ, [_I64, _I64, _I64]),
    "mednext_ce_fwd": (_INT, [_P, _P, _P, _P, _SZ, _I64, _I64, _I64, _I64, _INT, _P]),
    "mednext_ce_bwd": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _INT, _P]),
    "mednext_pw_mlp_fwd": (
        _INT, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _INT, _P],
    ),
    "mednext_pw_gn_bwd_fused_workspace_size": (_SZ, [_I64, _I64, _I64, _I64, _INT]),
    "mednext_pw_gn_bwd_fused": (
        _INT, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _I64, _I64, _I64, _I64, _INT, _P],
    ),
    "mednext_pw_wgrad_workspace_size": (_SZ, [_I64, _I64, _I64, _I64]),
    "mednext_pw_wgrad": (
        _INT,
        [_P, _P, _P, _P, _INT, _P, _P, _P, _P, _SZ, _I64, _I64, _I64, _I64, _INT, _P],
    ),
    "mednext_cast_params": (_INT, [_P, _INT, _P]),
    "mednext_grn_workspace_size": (_SZ, [_I64, _I64, _I64, _INT]),
    "mednext_grn_fwd": (_INT, [_P, _P, _P, _P, _P, _P, _P, _SZ, _I64, _I64, _I64, _F, _INT, _P]),
    "mednext_grn_bwd": (_INT, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _I64, _I64, _I64, _INT, _P]),
    "mednext_gn_bwd_from_partials": (
        _INT,
        [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _INT, _INT, _INT, _INT, _P],
    ),
}



class CastEntry(ctypes.Structure):
    """``mednext_cast_entry`` of the header."""

    _fields_ = [("src", _P), ("dst", _P), ("rows", _I64), ("cols", _I64), ("out_dtype", _INT),
                ("via_dtype", _INT), ("transpose", _INT)]


CAST_MAX_ENTRIES = 16

_lib: ctypes.CDLL | None = None
_device_checked: set[int] = set()


def library_path() -> Path:
    override = os.environ.get("MEDNEXT_B200_LIB")
    return Path(override) if override else LIB_PATH


def load() -> ctypes.CDLL:
    """Load the shared library and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.exists():
        raise RuntimeError(
            f"{path} is missing; build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "or `python -m mednext_accel_b200._build`"
        )
    lib = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def status_string(status: int) -> str:
    return load().mednext_status_string(status).decode()


def check(status: int, what: str) -> None:
    if status == OK:
        return
    message = f"{what}: {status_string(status)}"
    if status in (ERR_CUDA,):
        message += f" (cudaError {load().mednext_last_cuda_error()})"
        raise RuntimeError(message)
    if status == ERR_DEVICE:
        raise RuntimeError(message)
    raise ValueError(message)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def require_device(t: torch.Tensor) -> None:
    """Fail loudly unless ``t`` is a CUDA tensor on an sm_100 device."""
    if t.device.type != "cuda":
        raise ValueError("CUDA tensors are required")
    index = t.device.index if t.device.index is not None else torch.cuda.current_device()
    if index in _device_checked:
        return
    with torch.cuda.device(index):
        check(load().mednext_check_device(), "mednext_check_device")
    _device_checked.add(index)


def device_error() -> int:
    """Read and clear the device-side error word (synchronises the current stream)."""
    code = _INT(0)
    check(load().mednext_device_error(ctypes.byref(code), stream()), "mednext_device_error")
    return code.value


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """Scratch buffer from torch's caching allocator (capture-safe)."""
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)

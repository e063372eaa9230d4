"""CPU oracle for the MedNeXt block hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this module, and only as the checker.  The product
(``mednext_accel_b200``) never imports, links or executes anything here.

Layers:
* ``mednext_oracle.c``: fp64 loop restatement of depthwise conv (stride 1,
  stride 2, transpose), GroupNorm, exact GELU, 1x1 convolution and the v2
  Global Response Norm, each citing
  the reference file:line it follows; compiled with gcc into ``_build/``.
* :func:`block_reference`: the reference ``MedNeXtBlock`` forward and backward
  (models/blocks.py:82-91) composed from those primitives, with the roundings
  the reference performs under ``torch.autocast(dtype=bfloat16)``: conv inputs
  and outputs in bf16, GroupNorm in fp32, GELU on bf16 inputs, gradients of
  bf16 tensors rounded to bf16.  With ``round_bf16=False`` every step is fp64.

Parity of this oracle is pinned by tests/test_oracle.py against golden vectors
that tests/golden/make_golden.py produced by running the reference package
itself (its pure-PyTorch path) on seeded inputs.
"""

from __future__ import annotations

import ctypes
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "mednext_oracle.c"
LIB = HERE / "_build" / "libmednext_oracle.so"

_lib: ctypes.CDLL | None = None
_D = ctypes.POINTER(ctypes.c_double)
_I = ctypes.c_int64


def build(force: bool = False) -> Path:
    LIB.parent.mkdir(parents=True, exist_ok=True)
    if force or not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        subprocess.run(
            ["gcc", "-O2", "-fPIC", "-shared", "-std=c11", "-o", str(LIB), str(SRC), "-lm"],
            check=True,
        )
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(str(LIB))
        sig = {
            "oracle_dw_fwd": [_D, _D, _D, _D, _I, _I, _I, _I, _I, ctypes.c_int],
            "oracle_dw_dgrad": [_D, _D, _D, _I, _I, _I, _I, _I, ctypes.c_int],
            "oracle_dw_wgrad": [_D, _D, _D, _D, _I, _I, _I, _I, _I, ctypes.c_int],
            "oracle_s2_gather": [_D, _D, _D, _D, _I, _I, _I, _I, _I, _I, _I, _I, ctypes.c_int],
            "oracle_s2_scatter": [_D, _D, _D, _D, _I, _I, _I, _I, _I, _I, _I, _I, ctypes.c_int],
            "oracle_s2_wgrad": [_D, _D, _D, _I, _I, _I, _I, _I, _I, _I, _I, ctypes.c_int],
            "oracle_channel_sum": [_D, _D, _I, _I, _I],
            "oracle_groupnorm_fwd": [_D, _D, _D, ctypes.c_double, _D, _D, _D, _I, _I, _I],
            "oracle_groupnorm_bwd": [_D, _D, _D, _D, _D, _D, _D, _D, _I, _I, _I],
            "oracle_gelu": [_D, _D, _I],
            "oracle_gelu_grad": [_D, _D, _I],
            "oracle_pointwise_fwd": [_D, _D, _D, _D, _I, _I, _I, _I],
            "oracle_pointwise_bwd": [_D, _D, _D, _D, _D, _D, _I, _I, _I, _I],
            "oracle_grn_fwd": [_D, _D, _D, _D, _D, _D, _I, _I, _I, ctypes.c_double],
            "oracle_grn_bwd": [_D, _D, _D, _D, _D, _D, _D, _D, _I, _I, _I],
        }
        for name, args in sig.items():
            fn = getattr(_lib, name)
            fn.argtypes = args
            fn.restype = None
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == np.float64 and a.flags.c_contiguous
    return a.ctypes.data_as(_D)


def _f64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float64))


def round_bf16(a: np.ndarray) -> np.ndarray:
    """Round to the nearest bfloat16 (ties to even), returned as float64."""
    f = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).astype(np.float64)


# --------------------------------------------------------------------------- primitives
def dw_fwd(x, w, b, k):
    x, w = _f64(x), _f64(w)
    b = None if b is None else _f64(b)
    y = np.empty_like(x)
    lib().oracle_dw_fwd(_p(x), _p(w), _p(b), _p(y), *x.shape, k)
    return y


def dw_dgrad(dy, w, k):
    dy, w = _f64(dy), _f64(w)
    dx = np.empty_like(dy)
    lib().oracle_dw_dgrad(_p(dy), _p(w), _p(dx), *dy.shape, k)
    return dx


def dw_wgrad(x, dy, k):
    x, dy = _f64(x), _f64(dy)
    c = x.shape[1]
    dw = np.empty((c, 1, k, k, k))
    db = np.empty((c,))
    lib().oracle_dw_wgrad(_p(x), _p(dy), _p(dw), _p(db), *x.shape, k)
    return dw, db


def s2_fwd(x, w, b, k):
    """Depthwise Conv3d, stride 2, padding k/2 (down block)."""
    x, w = _f64(x), _f64(w)
    b = None if b is None else _f64(b)
    n, c, d, h, ww = x.shape
    s = ((d + 1) // 2, (h + 1) // 2, (ww + 1) // 2)
    y = np.empty((n, c, *s))
    lib().oracle_s2_gather(_p(x), _p(w), _p(b), _p(y), n, c, d, h, ww, *s, k)
    return y


def s2_dgrad(dy, w, input_size, k):
    dy, w = _f64(dy), _f64(w)
    n, c = dy.shape[:2]
    dx = np.empty((n, c, *input_size))
    lib().oracle_s2_scatter(_p(dy), _p(w), None, _p(dx), n, c, *input_size, *dy.shape[2:], k)
    return dx


def s2_wgrad(x, dy, k):
    x, dy = _f64(x), _f64(dy)
    n, c = x.shape[:2]
    dw = np.empty((c, 1, k, k, k))
    lib().oracle_s2_wgrad(_p(x), _p(dy), _p(dw), n, c, *x.shape[2:], *dy.shape[2:], k)
    return dw, channel_sum(dy)


def t_fwd(x, w, b, k):
    """Depthwise ConvTranspose3d, stride 2, padding k/2 (up block): S -> 2S-1."""
    x, w = _f64(x), _f64(w)
    b = None if b is None else _f64(b)
    n, c, d, h, ww = x.shape
    big = (2 * d - 1, 2 * h - 1, 2 * ww - 1)
    y = np.empty((n, c, *big))
    lib().oracle_s2_scatter(_p(x), _p(w), _p(b), _p(y), n, c, *big, d, h, ww, k)
    return y


def t_dgrad(dy, w, k):
    dy, w = _f64(dy), _f64(w)
    n, c, bd, bh, bw = dy.shape
    small = ((bd + 1) // 2, (bh + 1) // 2, (bw + 1) // 2)
    dx = np.empty((n, c, *small))
    lib().oracle_s2_gather(_p(dy), _p(w), None, _p(dx), n, c, bd, bh, bw, *small, k)
    return dx


def t_wgrad(x, dy, k):
    x, dy = _f64(x), _f64(dy)
    n, c = x.shape[:2]
    dw = np.empty((c, 1, k, k, k))
    lib().oracle_s2_wgrad(_p(dy), _p(x), _p(dw), n, c, *dy.shape[2:], *x.shape[2:], k)
    return dw, channel_sum(dy)


def channel_sum(x):
    x = _f64(x)
    n, c = x.shape[:2]
    out = np.empty((c,))
    lib().oracle_channel_sum(_p(x), _p(out), n, c, int(np.prod(x.shape[2:])))
    return out


def groupnorm_fwd(x, gamma, beta, eps=1e-5):
    x = _f64(x)
    n, c = x.shape[:2]
    vol = int(np.prod(x.shape[2:]))
    y = np.empty_like(x)
    mean = np.empty((n * c,))
    rstd = np.empty((n * c,))
    lib().oracle_groupnorm_fwd(_p(x), _p(None if gamma is None else _f64(gamma)), _p(None if beta is None else _f64(beta)),
                               eps, _p(y), _p(mean), _p(rstd), n, c, vol)
    return y, mean, rstd


def groupnorm_bwd(dy, x, mean, rstd, gamma):
    dy, x = _f64(dy), _f64(x)
    n, c = x.shape[:2]
    vol = int(np.prod(x.shape[2:]))
    dx = np.empty_like(x)
    dg = np.empty((c,))
    db = np.empty((c,))
    lib().oracle_groupnorm_bwd(_p(dy), _p(x), _p(_f64(mean)), _p(_f64(rstd)), _p(None if gamma is None else _f64(gamma)),
                               _p(dx), _p(dg), _p(db), n, c, vol)
    return dx, dg, db


def gelu(x):
    x = _f64(x)
    y = np.empty_like(x)
    lib().oracle_gelu(_p(x), _p(y), x.size)
    return y


def gelu_grad(x):
    x = _f64(x)
    g = np.empty_like(x)
    lib().oracle_gelu_grad(_p(x), _p(g), x.size)
    return g


def grn_fwd(x, gamma, beta, eps=1e-6):
    """MedNeXt v2 GRN forward (ops/grn.py:16-29) in fp64: (y, norm [N, C], den [N])."""
    x = _f64(x)
    n, c = x.shape[:2]
    vol = int(np.prod(x.shape[2:]))
    y = np.empty_like(x)
    norm = np.empty((n, c))
    den = np.empty((n,))
    lib().oracle_grn_fwd(_p(x), _p(_f64(gamma).reshape(-1)), _p(_f64(beta).reshape(-1)), _p(y), _p(norm), _p(den),
                         n, c, vol, float(eps))
    return y, norm, den


def grn_bwd(dy, x, gamma, norm, den):
    """GRN backward in fp64: (dx, dgamma [C], dbeta [C])."""
    dy, x = _f64(dy), _f64(x)
    n, c = x.shape[:2]
    vol = int(np.prod(x.shape[2:]))
    dx = np.empty_like(x)
    dg = np.empty((c,))
    db = np.empty((c,))
    lib().oracle_grn_bwd(_p(dy), _p(x), _p(_f64(gamma).reshape(-1)), _p(_f64(norm)), _p(_f64(den)), _p(dx), _p(dg),
                         _p(db), n, c, vol)
    return dx, dg, db


def pointwise_fwd(x, w, b):
    x, w = _f64(x), _f64(w).reshape(w.shape[0], -1)
    b = None if b is None else _f64(b)
    n, cin = x.shape[:2]
    cout = w.shape[0]
    y = np.empty((n, cout, *x.shape[2:]))
    lib().oracle_pointwise_fwd(_p(x), _p(np.ascontiguousarray(w)), _p(b), _p(y), n, cin, cout, int(np.prod(x.shape[2:])))
    return y


def pointwise_bwd(dy, x, w):
    dy, x = _f64(dy), _f64(x)
    w2 = np.ascontiguousarray(_f64(w).reshape(w.shape[0], -1))
    n, cin = x.shape[:2]
    cout = w2.shape[0]
    dx = np.empty_like(x)
    dw = np.empty((cout, cin))
    db = np.empty((cout,))
    lib().oracle_pointwise_bwd(_p(dy), _p(x), _p(w2), _p(dx), _p(dw), _p(db), n, cin, cout, int(np.prod(x.shape[2:])))
    return dx, dw, db


# --------------------------------------------------------------------------- block
@dataclass
class BlockParams:
    dw_w: np.ndarray
    dw_b: np.ndarray
    gn_w: np.ndarray
    gn_b: np.ndarray
    e_w: np.ndarray
    e_b: np.ndarray
    p_w: np.ndarray
    p_b: np.ndarray

    @classmethod
    def from_state(cls, state: dict, prefix: str = "") -> "BlockParams":
        g = lambda k: np.asarray(state[prefix + k], dtype=np.float64)  # noqa: E731
        return cls(g("depthwise.weight"), g("depthwise.bias"), g("norm.weight"), g("norm.bias"),
                   g("expand.weight"), g("expand.bias"), g("project.weight"), g("project.bias"))


def block_reference(x, dy, p: BlockParams, kind: str = "regular", addend=None, residual_is_input=True,
                    round_bf16_steps: bool = True, eps: float = 1e-5):
    """Reference MedNeXt block forward + backward (models/blocks.py:82-182).

    kind: "regular" (stride-1 depthwise), "down" (stride 2), "up" (transposed).
    ``addend``: extra tensor added to the block output (the down/up residual
    branch); ``residual_is_input``: add x itself (regular block).  Returns
    (y, grads) where grads holds dx, the eight parameter grads and d_addend."""
    r = round_bf16 if round_bf16_steps else (lambda a: _f64(a))
    x = _f64(x)
    k = p.dw_w.shape[-1]
    xb = r(x)
    wdw, bdw = r(p.dw_w), r(p.dw_b)
    if kind == "regular":
        t = r(dw_fwd(xb, wdw, bdw, k))
    elif kind == "down":
        t = r(s2_fwd(xb, wdw, bdw, k))
    else:
        t = r(t_fwd(xb, wdw, bdw, k))
    z, mean, rstd = groupnorm_fwd(t, p.gn_w, p.gn_b, eps)  # fp32 in the reference; fp64 here
    zb = r(z)
    we, be, wp, bp = r(p.e_w), r(p.e_b), r(p.p_w), r(p.p_b)
    u = r(pointwise_fwd(zb, we, be))
    g = r(gelu(u))
    pr = r(pointwise_fwd(g, wp, bp))
    y = pr
    extra = None
    if residual_is_input:
        extra = x
    elif addend is not None:
        extra = _f64(addend)
    if extra is not None:
        y = pr + extra
    # ---- backward ----
    dy = _f64(dy)
    dpr = r(dy)
    dg, dwp, dbp = pointwise_bwd(dpr, g, wp)
    dg = r(dg)
    du = r(dg * gelu_grad(u))
    dzb, dwe, dbe = pointwise_bwd(du, zb, we)
    dzb = r(dzb)
    dt, dgamma, dbeta = groupnorm_bwd(dzb, t, mean, rstd, p.gn_w)
    dt = r(dt)
    if kind == "regular":
        dx = dw_dgrad(dt, wdw, k)
        dwdw, dbdw = dw_wgrad(xb, dt, k)
    elif kind == "down":
        dx = s2_dgrad(dt, wdw, x.shape[2:], k)
        dwdw, dbdw = s2_wgrad(xb, dt, k)
    else:
        dx = t_dgrad(dt, wdw, k)
        dwdw, dbdw = t_wgrad(xb, dt, k)
    dx = r(dx)
    if residual_is_input:
        dx = dx + dy
    grads = {
        # GroupNorm(C, C) follows the depthwise conv, so sum(dt) per channel is
        # analytically zero and its bias grad is pure rounding noise; this is
        # the scale to judge that noise against.
        "depthwise.bias_scale": np.abs(dt).sum(axis=(0, 2, 3, 4)),
        "dx": dx,
        "depthwise.weight": dwdw, "depthwise.bias": dbdw,
        "norm.weight": dgamma, "norm.bias": dbeta,
        "expand.weight": dwe.reshape(p.e_w.shape), "expand.bias": dbe,
        "project.weight": dwp.reshape(p.p_w.shape), "project.bias": dbp,
        "d_addend": dy if (addend is not None and not residual_is_input) else None,
    }
    return y, grads


def rel_l2(a, b) -> float:
    """Relative L2 error, the reference's component validator metric
    (profiling/validation.py:30-64)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b.ravel())
    return float(np.linalg.norm((a - b).ravel()) / (den if den > 0 else 1.0))


def max_rel(a, b) -> float:
    """Max |a-b| / max|b| (scale-relative maximum error)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.max(np.abs(b)) if b.size else 1.0
    return float(np.max(np.abs(a - b)) / (den if den > 0 else 1.0)) if a.size else 0.0

"""Per-operator timings of the sm_100a kernels at MedNeXt-Base level-0 shapes.

    python -m mednext_accel_b200.microbench [CASE-SUBSTRING ...] [--reps N] [--warmup W] [--json]

Each case is one library call (one or a few kernel launches) on inputs that are
larger than the 126 MB L2.  The case is run W times untimed, then timed over N
back-to-back repetitions with CUDA events on the current stream.  The reported GB/s
divides the algorithmic bytes (every input element read once, every output element
written once) by that time.  The same command under ``ncu -k <kernel>`` gives the
per-kernel counters summarised in ``profiles/``.
"""

from __future__ import annotations

import argparse
import json
import sys

import torch

from . import _native as nat
from . import depthwise as dwk
from .pointwise import (
    gn_backward_from_partials, gn_stats, pw_gelu_bwd, pw_gemm, pw_gemm_gelu_out, pw_gn_bwd_fused, pw_mlp_fwd,
    pw_wgrad,
)

V = 128**3  # level-0 voxels
C, RC = 32, 64  # level-0 channels and expanded channels (ratio 2)


def _cases(dev: torch.device) -> dict[str, tuple]:
    torch.manual_seed(0)
    bf = torch.bfloat16

    def r(*shape):
        return torch.randn(*shape, device=dev).to(bf)

    t, u, dy, du, x = r(1, C, V), r(1, RC, V), r(1, C, V), r(1, RC, V), r(1, C, V)
    we, wp = r(RC, C) * 0.2, r(C, RC) * 0.2
    b1, b2 = torch.randn(RC, device=dev), torch.randn(C, device=dev)
    g, bb = torch.ones(C, device=dev), torch.zeros(C, device=dev)
    stats = gn_stats(t, 1e-5)
    dz, part = pw_gemm(du, (r(C, RC) * 0.2), C, aux=t, gn_bwd_stats=stats)
    wp_t, we_t = wp.t().contiguous(), we.t().contiguous()
    gout = torch.empty_like(u)
    vol = (1, C, 128, 128, 128)
    x5, dy5 = x.view(vol), dy.view(vol)
    w3 = (torch.randn(C, 1, 3, 3, 3, device=dev) * 0.2).to(bf)
    w5 = (torch.randn(C, 1, 5, 5, 5, device=dev) * 0.09).to(bf)
    w7 = (torch.randn(C, 1, 7, 7, 7, device=dev) * 0.05).to(bf)
    b3 = torch.randn(C, device=dev).to(bf)
    w3b = (torch.randn(2 * C, 1, 3, 3, 3, device=dev) * 0.2).to(bf)
    ys2 = r(1, C, 64, 64, 64)
    xs, ybig = r(1, 2 * C, 64, 64, 64), r(1, 2 * C, 127, 127, 127)
    # the fused up block's layout: W-rows of the 127^3 grid padded to 128 elements
    ybig_p = r(1, 2 * C, 127, 127, 128)
    up_bytes = 2 * C * 2 * (64**3 + 127**3)
    dy_pad, t_up, y_up = r(1, C, 128, 128, 128), r(1, 2 * C, 127, 127, 128), r(1, C, 127, 127, 128)
    # a deep level of MedNeXt-Base: C256, ratio 4, 16^3 voxels
    vd = 16**3
    t_d, u_d, dy_d = r(1, 256, vd), r(1, 1024, vd), r(1, 256, vd)
    g_d, bb_d = torch.ones(256, device=dev), torch.zeros(256, device=dev)
    stats_d = gn_stats(t_d, 1e-5)
    return {
        "pw compress wgrad C256 16^3 (saved GELU output)": (lambda: pw_wgrad(dy_d, u_d), (256 + 1024) * 2 * vd),
        "pw expand wgrad C256 16^3 (GroupNorm prologue)": (
            lambda: pw_wgrad(u_d, t_d, prologue=nat.PRO_GROUPNORM, pro_stats=stats_d, pro_gamma=g_d, pro_beta=bb_d),
            (256 + 1024) * 2 * vd),
        "pw expand fwd (GroupNorm prologue, bias)": (
            lambda: pw_gemm(t, we, RC, prologue=nat.PRO_GROUPNORM, pro_stats=stats, pro_gamma=g, pro_beta=bb, bias=b1),
            (C + RC) * 2 * V),
        "pw expand fwd + GELU output (GroupNorm prologue, bias)": (
            lambda: pw_gemm_gelu_out(t, we, RC, prologue=nat.PRO_GROUPNORM, pro_stats=stats, pro_gamma=g,
                                     pro_beta=bb, bias=b1),
            (C + 2 * RC) * 2 * V),
        "pw project fwd (no prologue: GELU output read, bias, residual)": (
            lambda: pw_gemm(gout, wp, C, bias=b2, residual=x), (RC + C + C) * 2 * V),
        "pw project fwd (GELU prologue, bias, residual)": (
            lambda: pw_gemm(u, wp, C, prologue=nat.PRO_GELU, bias=b2, residual=x), (RC + C + C) * 2 * V),
        "pw expansion fwd fused (expand + GELU + project)": (
            lambda: pw_mlp_fwd(t, stats, g, bb, we, b1, wp, b2, x), (C + RC + C + C) * 2 * V),
        "pw project fwd + GELU output": (
            lambda: pw_gemm(u, wp, C, prologue=nat.PRO_GELU, bias=b2, residual=x, pro_out=gout),
            (RC + C + C + RC) * 2 * V),
        "pw project dgrad (GELU' epilogue)": (
            lambda: pw_gemm(dy, wp_t, RC, aux=u, gelu_grad=True), (C + RC + RC) * 2 * V),
        "pw project bwd fused (dgrad + wgrad)": (lambda: pw_gelu_bwd(dy, wp_t, u), (C + RC + RC) * 2 * V),
        "pw expand dgrad (GroupNorm-backward sums)": (
            lambda: pw_gemm(du, we_t, C, aux=t, gn_bwd_stats=stats), (RC + C + C) * 2 * V),
        "pw expand bwd fused (dgrad + GroupNorm sums + wgrad)": (
            lambda: pw_gn_bwd_fused(du, we_t, t, stats, g, bb), (RC + C + C) * 2 * V),
        "pw project wgrad (GELU prologue)": (lambda: pw_wgrad(dy, u, prologue=nat.PRO_GELU), (C + RC) * 2 * V),
        "pw project wgrad (saved GELU output)": (lambda: pw_wgrad(dy, gout), (C + RC) * 2 * V),
        "pw expand wgrad (GroupNorm prologue)": (
            lambda: pw_wgrad(du, t, prologue=nat.PRO_GROUPNORM, pro_stats=stats, pro_gamma=g, pro_beta=bb),
            (C + RC) * 2 * V),
        "dw fwd C32 k3": (lambda: dwk.dw_forward(x5, w3, None, 3), 2 * C * 2 * V),
        "dw fwd + GN stats C32 k3": (lambda: dwk.dw_forward(x5, w3, b3, 3, gn_eps=1e-5), 2 * C * 2 * V),
        "dw dgrad + addend C32 k3": (lambda: dwk.dw_dgrad(dy5, w3, 3, addend=x5), 3 * C * 2 * V),
        "dw dgrad C32 k3": (lambda: dwk.dw_dgrad(dy5, w3, 3), 2 * C * 2 * V),
        "dw wgrad C32 k3": (lambda: dwk.dw_wgrad(x5, dy5, 3), 2 * C * 2 * V),
        "dw fwd + GN stats C32 k5 (tensor cores)": (lambda: dwk.dw_forward(x5, w5, w5[:, 0, 0, 0, 0], 5, gn_eps=1e-5),
                                                    2 * C * 2 * V),
        "dw dgrad + addend C32 k5 (tensor cores)": (lambda: dwk.dw_dgrad(dy5, w5, 5, addend=x5), 3 * C * 2 * V),
        "dw wgrad C32 k5": (lambda: dwk.dw_wgrad(x5, dy5, 5), 2 * C * 2 * V),
        "dw fwd C32 k7 (tensor cores)": (lambda: dwk.dw_forward(x5, w7, None, 7), 2 * C * 2 * V),
        "dw dgrad C32 k7 (tensor cores)": (lambda: dwk.dw_dgrad(dy5, w7, 7), 2 * C * 2 * V),
        "s2 fwd C32 k3": (lambda: dwk.s2_forward(x5, w3, None, 3), C * 2 * V * 9 // 8),
        "s2 dgrad C32 k3": (lambda: dwk.s2_dgrad(ys2, w3, (128, 128, 128), 3), C * 2 * V * 9 // 8),
        "s2 wgrad C32 k3": (lambda: dwk.s2_wgrad(x5, ys2, 3), C * 2 * V * 9 // 8),
        "dwT fwd C64 64^3->127^3 k3": (lambda: dwk.t_forward(xs, w3b, None, 3), up_bytes),
        "dwT dgrad C64 k3": (lambda: dwk.t_dgrad(ybig, w3b, 3), up_bytes),
        "dwT wgrad C64 k3": (lambda: dwk.t_wgrad(xs, ybig, 3), up_bytes),
        "dwT fwd C64 row-pitched k3": (lambda: dwk.t_forward(xs, w3b, None, 3, row_pitch=128), up_bytes),
        "dwT dgrad C64 row-pitched + addend k3": (
            lambda: dwk.t_dgrad(ybig_p, w3b, 3, small=(64, 64, 64), addend=xs), up_bytes + 2 * C * 2 * 64**3),
        "dwT wgrad C64 row-pitched k3": (lambda: dwk.t_wgrad(xs, ybig_p, 3), up_bytes),
        "gn stats C64 row-pitched 127^3": (lambda: gn_stats(t_up, 1e-5, row_len=127), 2 * C * 2 * 127**3),
        "unpad_front C32 128^3 -> row-pitched": (lambda: dwk.unpad_front(dy_pad, 128), 2 * C * 2 * 128**3),
        "pad_front_add C32 row-pitched -> 128^3": (
            lambda: dwk.pad_front_add(y_up, (127, 127, 127), dy_pad), 3 * C * 2 * 128**3),
        "gn stats C32": (lambda: gn_stats(t, 1e-5), C * 2 * V),
        "gn bwd C32 (fold + apply)": (lambda: gn_backward_from_partials(dz, t, stats, g, part), 3 * C * 2 * V),
    }


def _grn_cases(dev: torch.device) -> dict[str, tuple]:
    """GRN at the v2 Wide stage-0 expansion: [2, 192, 160^3] bf16 (3.1 GB per tensor).
    Algorithmic bytes: forward x + y, backward dy + x + dx.  The kernels take two
    passes over x (its per-channel norms are needed before any output), so the
    forward moves 1.5x and the backward 5/3x the algorithmic bytes."""
    from .grn import grn_backward, grn_forward

    shape = (2, 192, 160, 160, 160)
    x = torch.randn(shape, device=dev, dtype=torch.bfloat16)
    dy = torch.randn(shape, device=dev, dtype=torch.bfloat16)
    gamma = torch.randn((1, 192, 1, 1, 1), device=dev)
    beta = torch.randn((1, 192, 1, 1, 1), device=dev)
    _, norm, den = grn_forward(x, gamma, beta, 1e-6)
    nbytes = x.numel() * 2
    return {
        "grn fwd 2x192x160^3": (lambda: grn_forward(x, gamma, beta, 1e-6), 2 * nbytes),
        "grn bwd 2x192x160^3": (lambda: grn_backward(dy, x, gamma, norm, den), 3 * nbytes),
    }


def run(patterns: list[str], reps: int = 10, warmup: int = 3) -> dict[str, dict]:
    dev = torch.device("cuda", torch.cuda.current_device())
    results = {}
    cases = _cases(dev)
    if not patterns or any("grn" in p for p in patterns):
        cases.update(_grn_cases(dev))
    for name, (fn, nbytes) in cases.items():
        if patterns and not any(p in name for p in patterns):
            continue
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        results[name] = {"us": round(ms * 1e3, 1), "GB/s": round(nbytes / ms / 1e6, 1), "bytes": nbytes}
    return results


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("cases", nargs="*", help="substrings of case names (default: all)")
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--json", action="store_true")
    args = ap.parse_args(argv)
    res = run(args.cases, args.reps, args.warmup)
    if args.json:
        print(json.dumps(res))
    else:
        for name, r in res.items():
            print(f"{name:48s} {r['us']:9.1f} us {r['GB/s']:9.1f} GB/s")
    err = nat.device_error()
    if err:
        print(f"device error word {err:#x}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""MedNeXt-Base 128^3 bf16 training-step benchmark on B200 (1..8 GPUs, one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|reference-gpu]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Workload: MedNeXt v1 Base, kernel 3, deep supervision, batch 1 per GPU, input
1x1x128^3 ~N(0,1), labels uniform in {0,1,2}, loss = mean of the five heads'
cross-entropy against nearest-downsampled labels, AdamW lr 1e-4, random init
from seed 0, bf16 autocast (the reference's own training benchmark,
benchmarks/implementations.py:137-190).  Each rank draws its own sample (seed
1000+rank); gradients are averaged by NCCL all-reduce overlapped with backward.

``--impl ours`` times the sm_100a path: the whole step (forward, backward,
gradient all-reduce, AdamW) is captured once as a CUDA graph and replayed; K
steps are timed with CUDA events after W warm-up steps, max over ranks.  The
activations (128^3 voxels x 32+ channels) are far larger than the 126 MB L2, so
no flush is needed between steps.

``--impl reference`` times the reference's pure-PyTorch CPU implementation of
the same step (the oracle's functional restatement, fp32, all host threads) on
rank 0; other ranks exit.  A CPU step takes seconds, so at most
``--ref-max-steps`` full-size steps are timed after one full-size warm-up step,
and the line reports the number actually timed.

``--impl reference-gpu`` (opt-in, one GPU) times the unmodified reference
package from ``baseline/_ref`` on the GPU: ``mednext_base(...,
optimization="auto")`` compiled with ``torch.compile(mode="default",
fullgraph=True)`` and ``cudnn.benchmark``, median of per-step CUDA events, as the
reference's benchmarks/implementations.py:137-190 does.

``--workload`` (opt-in) times the other shapes of the reference's benchmark
suite on the same path, without the CPU and roofline legs: ``large-k5``
(MedNeXt-Large k5, block counts [3,4,8,8,8,8,8,4,3], 2 samples per GPU,
all-expansion-stage activation checkpointing) and ``block-k5`` (one MedNeXtBlock,
C = 64, R = 4, k = 5, on a 2x64x64^3 input: forward and backward).  The line
adds the peak allocated device memory.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch
import torch.distributed as dist
from torch.nn import functional as F

ROOT = Path(__file__).resolve().parent
METRIC = "MedNeXt-Base 128³ bf16 train-step ms at 1/2/4/8 B200; depthwise-bwd HBM GB/s"
SPATIAL = 128
HEAD_SIZES = (128, 64, 32, 16, 8)


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference", "reference-gpu"), default="ours")
    p.add_argument("--no-graph", action="store_true", help="time eager steps instead of a CUDA graph replay")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--ref-max-steps", type=int, default=3,
                   help="CPU reference: at most this many full-size steps are timed (median reported)")
    p.add_argument("--ref-optimization", default="auto",
                   help="reference-gpu: the reference factory's optimization argument (auto or reference)")
    p.add_argument("--ref-eager", action="store_true", help="reference-gpu: skip torch.compile")
    p.add_argument("--bucket-mb", type=float, default=6.0, help="gradient all-reduce bucket size (fp32 MB)")
    p.add_argument("--workload", choices=tuple(WORKLOADS), default="base-k3",
                   help="base-k3: the headline step (default); large-k5: MedNeXt-Large k5, 2 samples per GPU, "
                        "all-expansion-stage checkpointing; block-k5: one C64 R4 k5 block forward + backward")
    p.add_argument("--e2e-steps", type=int, default=10)
    p.add_argument("--spatial", type=int, default=SPATIAL, help=argparse.SUPPRESS)
    p.add_argument("--profile-step", action="store_true",
                   help="after warm-up run one eager step between cudaProfilerStart/Stop and exit "
                        "(for ncu --profile-from-start off: the launch list of one whole step, "
                        "backward-thread kernels included)")
    return p.parse_args(argv)


# --------------------------------------------------------------------------- helpers
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def downsampled_targets(target: torch.Tensor) -> dict[tuple[int, ...], torch.Tensor]:
    out = {}
    for s in HEAD_SIZES:
        size = (target.shape[1] * s // SPATIAL,) * 3
        if size == tuple(target.shape[1:]):
            out[size] = target
        else:
            out[size] = F.interpolate(target[:, None].float(), size=size, mode="nearest")[:, 0].long()
    return out


def end_to_end_ms(run_step, x, x_host, target, t_host, targets, steps, device, world, labels):
    """The step driven from pinned host memory: every step copies its input (and its
    class labels, sent as uint8 since there are 3 classes) host -> device and reads its
    loss back to the host, as a training loop with a pinned-memory loader does.

    The copies of step i + 1 run on a copy stream while step i computes: they land in
    staging buffers and enter the step's (graph-captured) inputs by one device copy, the
    labels widened to int64 and the deep-supervision targets taken as their all-multiple
    positions (equal to nearest interpolation at these power-of-two sizes).  Each
    step's loss is copied to pinned memory on the compute stream and read by the host
    one step later, so the host never stalls the GPU.  The timed region spans the first
    copy to the last loss read, on the device clock.  Returns (ms per step, H2D bytes
    per step)."""
    main = torch.cuda.current_stream(device)
    copy = torch.cuda.Stream(device=device)
    t_src = t_host.to(torch.uint8).pin_memory() if labels else t_host
    x_stage = torch.empty(x_host.shape, dtype=x_host.dtype, device=device)
    t_stage = torch.empty(t_src.shape, dtype=t_src.dtype, device=device)
    loss_host = torch.empty(steps, dtype=torch.float32).pin_memory()
    full = target.shape[1] if labels else 1

    def upload():
        with torch.cuda.stream(copy):
            x_stage.copy_(x_host, non_blocking=True)
            t_stage.copy_(t_src, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(copy)
        return ev

    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(main)
    copy.wait_stream(main)
    landed = upload()
    done = []
    for i in range(steps):
        main.wait_event(landed)
        with torch.no_grad():
            x.copy_(x_stage)
            target.copy_(t_stage)
            for size, t in targets.items():
                if t is not target:
                    f = full // size[0]
                    t.copy_(target[:, ::f, ::f, ::f])
        consumed = torch.cuda.Event()
        consumed.record(main)
        if i + 1 < steps:
            copy.wait_event(consumed)
            landed = upload()
        out = run_step()
        loss_host[i : i + 1].copy_(out.detach().float().reshape(1), non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(main)
        done.append(ev)
        if i > 0:
            done[i - 1].synchronize()
            _ = float(loss_host[i - 1])  # the previous step's loss, on the host
    e1.record(main)
    done[-1].synchronize()
    _ = float(loss_host[steps - 1])
    torch.cuda.synchronize()
    e2e = torch.tensor([e0.elapsed_time(e1)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e, op=dist.ReduceOp.MAX)
    h2d = x_host.numel() * x_host.element_size() + t_src.numel() * t_src.element_size()
    return float(e2e.item()) / steps, h2d


WORKLOADS = {
    "base-k3": "MedNeXt-Base k3 {S}^3 B1/GPU train step: 5-head deep-supervision CE + AdamW",
    "large-k5": ("MedNeXt-Large k5 {S}^3 B2/GPU train step, all-expansion-stage activation checkpointing: "
                 "5-head deep-supervision CE + AdamW"),
    "block-k5": "one MedNeXtBlock C64 R4 k5 forward + backward on 2x64x{S}^3 input, bf16 autocast",
}


def five_head_loss(heads, targets):
    """Mean over the five heads of the mean cross-entropy (the reference's deep
    supervision loss), on the package's native cross-entropy kernels."""
    from mednext_accel_b200.loss import cross_entropy

    return sum(cross_entropy(h, targets[tuple(h.shape[2:])]) for h in heads) / len(heads)


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None
            return self
        # nvidia-smi takes a moment to start (longer with several ranks starting it at
        # once): wait, bounded, for its first sample, then keep only the samples taken
        # from here on, i.e. during the timed region
        t0 = time.perf_counter()
        while not self.lines and time.perf_counter() - t0 < 5.0 and self.proc.poll() is None:
            time.sleep(0.01)
        self.lines.clear()
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9], strict=True):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


# --------------------------------------------------------------------------- depthwise-bwd roofline
def depthwise_backward_roofline(device: torch.device, reps: int = 10) -> dict:
    """Time the dominant depthwise backward (C=32 at 128^3, bf16, k=3: input grad +
    weight grad, the pair the metric names) with CUDA events on the launching
    stream.  Algorithmic bytes = dgrad (read dy, write dx) + wgrad (read x, read dy)."""
    from mednext_accel_b200 import depthwise as dwk

    g = torch.Generator(device=device).manual_seed(7)
    shape = (1, 32, SPATIAL, SPATIAL, SPATIAL)
    x = torch.randn(shape, device=device, generator=g, dtype=torch.float32).to(torch.bfloat16)
    dy = torch.randn(shape, device=device, generator=g, dtype=torch.float32).to(torch.bfloat16)
    w = (torch.randn((32, 1, 3, 3, 3), device=device, generator=g) / 27**0.5).to(torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    for _ in range(3):
        dwk.dw_dgrad(dy, w, 3)
        dwk.dw_wgrad(x, dy, 3)
    tg, tw = [], []
    s = torch.cuda.current_stream()
    for _ in range(reps):
        flush.zero_()
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(s)
        dwk.dw_dgrad(dy, w, 3)
        e1.record(s)
        flush.zero_()
        e1b = torch.cuda.Event(enable_timing=True)
        e1b.record(s)
        dwk.dw_wgrad(x, dy, 3)
        e2.record(s)
        torch.cuda.synchronize()
        tg.append(e0.elapsed_time(e1))
        tw.append(e1b.elapsed_time(e2))
    elem = x.numel() * x.element_size()
    algo_bytes = 4 * elem  # dgrad: dy + dx; wgrad: x + dy
    t_ms = statistics.median(tg) + statistics.median(tw)
    achieved = algo_bytes / (t_ms * 1e-3) / 1e9
    peak, kind = measured_peaks()
    traffic = None
    prof = ROOT / "profiles" / "depthwise_bwd_c32_128.json"
    if prof.exists():
        try:
            traffic = json.loads(prof.read_text()).get("dram_bytes_per_pair")
        except ValueError:
            traffic = None
    return {
        "bound": "hbm",
        "kernel": "depthwise dgrad + wgrad (C32 128^3 bf16 k3)",
        "achieved": round(achieved, 1),
        "peak": peak,
        "peak_kind": kind,
        "unit": "GB/s",
        "frac": round(achieved / peak, 4),
        "traffic": traffic,
        "algorithmic_bytes": algo_bytes,
        "dgrad_ms": round(statistics.median(tg), 4),
        "wgrad_ms": round(statistics.median(tw), 4),
        **fma_floor(2 * 2 * 27 * x.numel(), algo_bytes, peak, t_ms, device),
    }


def fma_floor(flops: int, algo_bytes: int, hbm_gbs: float, t_ms: float, device: torch.device) -> dict:
    """The depthwise convolution does 27 FMAs per 4 bytes at k = 3, past the FP32
    ridge point, so its floor is the larger of bytes / HBM bandwidth and FLOPs /
    FP32 FMA peak.  The FMA peak is nominal: SMs x 128 FP32 lanes x 2 FLOP x the
    maximum SM clock (nvidia-smi clocks.max.sm)."""
    props = torch.cuda.get_device_properties(device)
    try:
        mhz = float(subprocess.run(["nvidia-smi", f"--id={device.index or 0}", "--query-gpu=clocks.max.sm",
                                    "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                   timeout=10).stdout.strip().splitlines()[0])
    except (OSError, ValueError, IndexError, subprocess.TimeoutExpired):
        mhz = 1965.0
    fp32_tflops = props.multi_processor_count * 128 * 2 * mhz * 1e6 / 1e12
    floor_us = max(algo_bytes / (hbm_gbs * 1e9), flops / (fp32_tflops * 1e12)) * 1e6
    return {"flops": flops, "fp32_fma_peak_tflops": round(fp32_tflops, 1),
            "floor_us": round(floor_us, 1), "frac_of_floor": round(floor_us / (t_ms * 1e3), 4)}


def compress_forward_roofline(device: torch.device, reps: int = 10) -> dict:
    """Time the step's dominant tensor-core GEMM instance: level 0's compress
    forward (1x1x1 conv 64 -> 32 at 128^3, bf16: GELU applied to the A tile as it
    is loaded, bias and residual added in the epilogue), with CUDA events on the
    launching stream and L2 flushed before each launch.

    Algorithmic bytes = read u (64 ch) + read residual (32 ch) + write y (32 ch),
    2 B each, per voxel; FLOPs = 2 * 64 * 32 per voxel.  K = 64 and N = 32 make
    it HBM-bound (36 FLOP/B against a ridge of about 250), so the fraction is
    taken against the measured HBM copy bandwidth; the tensor-pipe fraction is
    reported beside it."""
    from mednext_accel_b200 import _native as nat
    from mednext_accel_b200.pointwise import pw_gemm

    g = torch.Generator(device=device).manual_seed(11)
    vox = SPATIAL ** 3
    cin, cout = 64, 32
    bf = torch.bfloat16
    u = torch.randn((1, cin, SPATIAL, SPATIAL, SPATIAL), device=device, generator=g).to(bf)
    res = torch.randn((1, cout, SPATIAL, SPATIAL, SPATIAL), device=device, generator=g).to(bf)
    w = (torch.randn((cout, cin), device=device, generator=g) / cin**0.5).to(bf)
    b = torch.randn((cout,), device=device, generator=g).to(bf).float()
    y = torch.empty_like(res)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    for _ in range(3):
        pw_gemm(u, w, cout, out_dtype=bf, prologue=nat.PRO_GELU, bias=b, residual=res, out=y)
    s = torch.cuda.current_stream()
    times = []
    for _ in range(reps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        pw_gemm(u, w, cout, out_dtype=bf, prologue=nat.PRO_GELU, bias=b, residual=res, out=y)
        e1.record(s)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    t_ms = statistics.median(times)
    algo_bytes = vox * 2 * (cin + 2 * cout)
    flops = 2 * cin * cout * vox
    achieved = algo_bytes / (t_ms * 1e-3) / 1e9
    peak, kind = measured_peaks()
    tflops_peak = None
    try:
        tflops_peak = float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        tflops_peak = 1590.0
    traffic = None
    prof = ROOT / "profiles" / "pw_compress_fwd_c32_128.json"
    if prof.exists():
        try:
            traffic = json.loads(prof.read_text()).get("dram_bytes_per_launch")
        except ValueError:
            traffic = None
    return {
        "bound": "hbm",
        "kernel": "pw_tma_fwd_kernel compress forward 64->32 at 128^3 bf16 (GELU prologue, bias+residual epilogue)",
        "achieved": round(achieved, 1),
        "peak": peak,
        "peak_kind": kind,
        "unit": "GB/s",
        "frac": round(achieved / peak, 4),
        "traffic": traffic,
        "algorithmic_bytes": algo_bytes,
        "ms": round(t_ms, 4),
        "tflops": round(flops / (t_ms * 1e-3) / 1e12, 2),
        "tensor_frac_of_bf16_peak": round(flops / (t_ms * 1e-3) / 1e12 / tflops_peak, 5),
    }


# --------------------------------------------------------------------------- CPU reference
def cpu_reference_step_ms(steps: int, spatial: int = SPATIAL, warmup: int = 1,
                          budget_s: float = 120.0) -> tuple[float, dict, int]:
    """The reference's pure-PyTorch training step on the host CPU (fp32, all threads).

    ``warmup`` full-size steps (thread pools, allocator, first-touch pages), then
    up to ``steps`` timed full-size steps, stopping early once ``budget_s`` of
    timed work has run.  Returns (median ms, description, steps timed)."""
    sys.path.insert(0, str(ROOT))
    from oracle.reference_model import ReferenceTrainer, forward, targets_for

    import mednext_accel_b200 as mx

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    torch.manual_seed(0)
    model = mx.mednext_base(in_channels=1, out_channels=3, kernel_size=3, deep_supervision=True,
                            optimization="reference")
    trainer = ReferenceTrainer(model.state_dict(), "base", 3)
    gen = torch.Generator().manual_seed(1000)
    x = torch.randn((1, 1, spatial, spatial, spatial), generator=gen)
    target = torch.randint(0, 3, (1, spatial, spatial, spatial), generator=gen)
    with torch.no_grad():
        tg = targets_for(target, forward(trainer.params, x, "base", 3))
    for _ in range(max(1, warmup)):
        trainer.step(x, tg)
    times = []
    t_start = time.perf_counter()
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        trainer.step(x, tg)
        times.append((time.perf_counter() - t0) * 1e3)
        if time.perf_counter() - t_start > budget_s:
            break
    ms = statistics.median(times)
    info = {"cores": threads, "kind": "port",
            "sample": f"median of {len(times)} fp32 train step(s) after {max(1, warmup)} full-size warm-up "
                      f"step(s): the reference's pure-PyTorch MedNeXt-Base (oracle/reference_model.py) "
                      f"at {spatial}^3 B1 on {threads} host threads"}
    return ms, info, len(times)


def run_reference(args) -> int:
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    ms, info, timed = cpu_reference_step_ms(min(args.steps, args.ref_max_steps), warmup=1)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(ms, 3),
        "unit": "ms",
        "n_gpus": args.gpus,
        "steps": timed,
        "steps_requested": args.steps,
        "warmup": 1,
        "ms_per_step": round(ms, 3),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "MedNeXt-Base k3 128^3 B1 train step (5-head CE, AdamW), host CPU",
                   "global_batch": 1, "spatial": SPATIAL,
                   "timing": "median of the timed steps (a CPU step takes seconds; see cpu_baseline.sample)"},
        "cpu_baseline": {"value": round(ms, 3), "unit": "ms", **info},
        "e2e": {"value": round(ms, 3), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------- reference on the GPU
def run_reference_gpu(args) -> int:
    """The unmodified reference package on one B200: the GPU bar of the comparison.

    Mirrors the reference's benchmarks/implementations.py:137-190: the stock
    factory (``optimization="auto"`` by default), ``torch.compile(mode="default",
    fullgraph=True)``, ``cudnn.benchmark``, a resident synthetic sample, the
    five-head mean cross-entropy under bf16 autocast and AdamW; per-step CUDA
    events after the warm-up, median reported."""
    world, rank, local = dist_env()
    if rank != 0:
        return 0
    ref_root = ROOT / "baseline" / "_ref"
    if not (ref_root / "mednext_accel").is_dir():
        print(json.dumps({"impl": "reference-gpu", "unavailable": "baseline/_ref/mednext_accel is absent"}),
              flush=True)
        return 0
    if not torch.cuda.is_available():
        print(json.dumps({"impl": "reference-gpu", "unavailable": "CUDA is not available"}), flush=True)
        return 0
    sys.path.insert(0, str(ref_root))
    import mednext_accel as ref

    torch.cuda.set_device(local)
    torch.backends.cudnn.benchmark = True
    torch.manual_seed(0)
    if args.workload == "block-k5":
        print(json.dumps({"impl": "reference-gpu", "unavailable": "the block workload has no reference factory"}),
              flush=True)
        return 0
    batch = 1
    if args.workload == "large-k5":
        batch = 2
        model = ref.mednext_large(in_channels=1, out_channels=3, kernel_size=5, deep_supervision=True,
                                  optimization=args.ref_optimization,
                                  checkpointing=ref.CheckpointConfig(style="expansion"))
    else:
        model = ref.mednext_base(in_channels=1, out_channels=3, kernel_size=3, deep_supervision=True,
                                 optimization=args.ref_optimization)
    model = model.cuda().train()
    compiled = not args.ref_eager
    if compiled:
        model = torch.compile(model, mode="default", fullgraph=True)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4)
    gen = torch.Generator().manual_seed(1000)
    x = torch.randn((batch, 1, SPATIAL, SPATIAL, SPATIAL), generator=gen).cuda()
    target = torch.randint(0, 3, (batch, SPATIAL, SPATIAL, SPATIAL), generator=gen).cuda()
    targets = downsampled_targets(target)

    def step():
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            heads = model(x)
            if isinstance(heads, torch.Tensor):
                heads = (heads,)
            loss = sum(F.cross_entropy(h, targets[tuple(h.shape[2:])]) for h in heads) / len(heads)
        loss.backward()
        opt.step()
        return loss

    t0 = time.perf_counter()
    for _ in range(max(3, args.warmup)):
        loss = step()
    torch.cuda.synchronize()
    warm_s = time.perf_counter() - t0
    events = []
    with ClockSampler(local) as clocks:
        for _ in range(args.steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            loss = step()
            e1.record()
            events.append((e0, e1))
        torch.cuda.synchronize()
    times = [a.elapsed_time(b) for a, b in events]
    ms = statistics.median(times)
    line = {
        "impl": "reference-gpu",
        "metric": METRIC if args.workload == "base-k3" else f"{args.workload} step ms on B200 (bf16; see config.workload)",
        "value": round(ms, 3),
        "unit": "ms",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": max(3, args.warmup),
        "ms_per_step": round(ms, 3),
        "mean_ms": round(statistics.fmean(times), 3),
        "higher_is_better": False,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": WORKLOADS[args.workload].format(S=SPATIAL) + ", reference package on GPU",
                   "optimization": args.ref_optimization, "compiled": compiled,
                   "compile": "torch.compile(mode='default', fullgraph=True)" if compiled else None,
                   "cudnn_benchmark": True, "timing": "median of per-step CUDA events"},
        "warmup_wall_s": round(warm_s, 1),
        "peak_allocated_mib": round(torch.cuda.max_memory_allocated() / 2**20),
        "final_loss": round(float(loss.item()), 5),
        "clocks": clocks.summary(),
        "device": torch.cuda.get_device_name(),
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------- ours
def run_ours(args) -> int:
    world, rank, local = dist_env()
    if not torch.cuda.is_available():
        print(json.dumps({"impl": "ours", "error": "CUDA is not available"}), flush=True)
        return 1
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    import mednext_accel_b200 as mx
    from mednext_accel_b200 import _native as nat
    from mednext_accel_b200.data_parallel import GradientBucketReducer, broadcast_parameters
    from mednext_accel_b200.adaptive import ModelOptimizationContext

    torch.backends.cudnn.benchmark = True
    S = args.spatial
    wl = args.workload
    torch.manual_seed(0)
    gen = torch.Generator().manual_seed(1000 + rank)
    if wl == "block-k5":
        # one MedNeXtBlock forward + backward: y = block(x), then y.backward(dy)
        S = 64 if args.spatial == SPATIAL else S
        block = mx.MedNeXtBlock(spatial_dims=3, in_channels=64, out_channels=64, expansion_ratio=4, kernel_size=5)
        mx.install_adaptive_operators(block, resolver=mx.PolicyResolver(),
                                      model_context=ModelOptimizationContext("mednext_v1", "base", "none"))
        block = block.to(device).train()
        x_host = torch.randn((2, 64, S, S, S), generator=gen).pin_memory()
        t_host = torch.randn((2, 64, S, S, S), generator=gen).to(torch.bfloat16).pin_memory()  # upstream grad
        x = x_host.to(device).requires_grad_()
        target = t_host.to(device)
        reducer = None

        def step():
            for prm in block.parameters():
                prm.grad = None
            x.grad = None
            with torch.autocast("cuda", dtype=torch.bfloat16):
                y = block(x)
            y.backward(target)
            return y[0, 0, 0, 0, :1].float().sum()
    else:
        if wl == "large-k5":
            model = mx.mednext_large(in_channels=1, out_channels=3, kernel_size=5, deep_supervision=True,
                                     checkpointing=mx.CheckpointConfig("expansion"))
            batch = 2
        else:
            model = mx.mednext_base(in_channels=1, out_channels=3, kernel_size=3, deep_supervision=True)
            batch = 1
        model = model.to(device).train()
        broadcast_parameters(model)
        reducer = GradientBucketReducer(model, bucket_cap_mb=args.bucket_mb)
        opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True, capturable=True)
        x_host = torch.randn((batch, 1, S, S, S), generator=gen).pin_memory()
        t_host = torch.randint(0, 3, (batch, S, S, S), generator=gen).pin_memory()
        x = x_host.to(device)
        target = t_host.to(device)
    targets = downsampled_targets(target) if wl != "block-k5" else {}

    if wl != "block-k5":
        def step():
            reducer.zero_grad()
            with torch.autocast("cuda", dtype=torch.bfloat16):
                heads = model(x)
                loss = five_head_loss(heads, targets)
            loss.backward()
            reducer.finish()
            opt.step()
            return loss

    # Warm-up on the stream the graph is captured on (required before capture).
    # Autograd's AccumulateGrad nodes remember the stream of their first use, so
    # warming up on any other stream leaves them on that stream during capture;
    # dropping the last warm-up loss frees its graph before the capture begins.
    side = torch.cuda.Stream(device=device)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(max(3, args.warmup)):
            loss = step()
        del loss
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()

    if args.profile_step:
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        step()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        if world > 1:
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"profile_step": True, "device_error": nat.device_error()}), flush=True)
        return 0

    graph = None
    mode = "eager"
    launches_before = nat.load().mednext_kernel_launches()
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            static_loss = step()
        mode = "cuda-graph"
        per_step_launches = nat.load().mednext_kernel_launches() - launches_before

        def run_step():
            graph.replay()
            return static_loss
    else:
        run_step = step
        step()
        per_step_launches = nat.load().mednext_kernel_launches() - launches_before
    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # ---------------- timed region (device time, max over ranks)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        start.record()
        for _ in range(args.steps):
            loss = run_step()
        end.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    elapsed = torch.tensor([start.elapsed_time(end)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
    ms = float(elapsed.item()) / args.steps
    final_loss = float(loss.item())

    # ---------------- end to end: host inputs in, loss out, through the same step
    e2e_steps = max(1, args.e2e_steps)
    e2e_ms, h2d = end_to_end_ms(run_step, x, x_host, target, t_host, targets, e2e_steps, device, world,
                                labels=wl != "block-k5")

    headline = wl == "base-k3"
    roof = depthwise_backward_roofline(device) if rank == 0 and headline else None
    roof_gemm = compress_forward_roofline(device) if rank == 0 and headline else None
    dev_err = nat.device_error()
    peak_mib = round(torch.cuda.max_memory_allocated(device) / 2**20)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and headline:
        cpu_ms, info, timed = cpu_reference_step_ms(3, spatial=S, warmup=1)
        cpu = {"value": round(cpu_ms, 1), "unit": "ms", "steps": timed, **info}

    if graph is not None:
        del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC if headline else f"{wl} step ms on B200 (bf16; see config.workload)",
        "value": round(ms, 3),
        "unit": "ms",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {
            "workload": WORKLOADS[wl].format(S=S),
            "global_batch": world * (2 if wl != "base-k3" else 1),
            "spatial": S,
            "parallelism": f"dp{world}",
            "step_mode": mode,
            "l2": "inputs and activations larger than L2 (no flush)",
        },
        "roofline": roof,
        "roofline_gemm": roof_gemm,
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_ms, 3), "unit": "ms", "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4,
                "copies": "step i+1's inputs copied on a copy stream during step i; labels sent as uint8; "
                          "each loss read on the host one step later"},
        "gpu_launches": int(per_step_launches * args.steps),
        "clocks": clocks.summary(),
        "final_loss": round(final_loss, 5),
        "peak_allocated_mib": peak_mib,
        "device_error": dev_err,
    }
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.impl == "reference":
        return run_reference(args)
    if args.impl == "reference-gpu":
        return run_reference_gpu(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

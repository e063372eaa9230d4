"""Build ``lib/libmednext_b200.so`` in-tree with nvcc for sm_100a.

One translation unit per kernel family is compiled in parallel and linked into a
plain C-ABI shared library (static CUDA runtime, no torch headers).  A unit is
recompiled only when a source or header is newer than its object file.

    python -m mednext_accel_b200._build [--force] [--ptxas-verbose]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build_obj"
LIB = PKG / "lib" / "libmednext_b200.so"
UNITS = ("api.cu", "launch_dw_s1.cu", "launch_dw_s2.cu", "launch_gn.cu", "launch_pw.cu", "pw_fwd_bf16.cu", "pw_fwd_bf16_f32.cu",
         "pw_fwd_f16.cu", "noalloc_dw_wgrad.cu", "params.cu", "loss.cu", "grn.cu")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    raise RuntimeError("nvcc not found (set CUDA_HOME)")


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [ROOT / "include" / "mednext_b200.h"]


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _compile(unit: str, force: bool, ptxas_verbose: bool) -> tuple[str, str]:
    src = CSRC / unit
    obj = BUILD / (Path(unit).stem + ".o")
    if not force and not _stale(obj, [src, *_deps()]):
        return unit, "up to date"
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {unit}:\n{proc.stdout}\n{proc.stderr}")
    return unit, proc.stderr


def build(force: bool = False, ptxas_verbose: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    with ThreadPoolExecutor(max_workers=len(UNITS)) as pool:
        results = list(pool.map(lambda u: _compile(u, force, ptxas_verbose), UNITS))
    if verbose or ptxas_verbose:
        for unit, log in results:
            print(f"[{unit}] {log.strip()[:20000]}")
    objs = [BUILD / (Path(u).stem + ".o") for u in UNITS]
    if force or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    return LIB


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--ptxas-verbose", action="store_true")
    args = parser.parse_args(argv)
    path = build(force=args.force, ptxas_verbose=args.ptxas_verbose, verbose=True)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())

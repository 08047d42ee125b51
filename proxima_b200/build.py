"""Build the native libraries in-tree (no JIT cache, so they travel with the repo).

* ``proxima_b200/lib/libproxima_cuda.so`` — the sm_100a kernels behind the C ABI
  declared in ``include/proxima_cuda.h`` (nvcc, ``-gencode arch=compute_100a,code=sm_100a``).
* ``proxima_b200/lib/libpxfix.so`` — host-side synthetic workload generators
  (C++, deterministic, multi-threaded).

Run ``python -m proxima_b200.build`` (or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
BUILD = PKG / "_build"
INCLUDE = ROOT / "include"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    f"-I{INCLUDE}", f"-I{CSRC}",
]
CUDA_SOURCES = ["ctx.cu", "flat.cu", "kmeans.cu", "ivfpq.cu", "sq.cu", "filter.cu", "snapshot.cu", "hostcopy.cu"]
HEADERS = ["common.cuh", "sm100.cuh", "flat_tc.cuh", "topk.cuh", "tmap.cuh", "kmeans_tc.cuh",
           "seqsum.cuh", "rng.h", "kmeans_api.h", "select.cuh", "refdist.cuh", "sq_tc.cuh", "fp32scan.cuh",
           "ivfpq.cuh", "hostcopy.cuh"]
CXX = os.environ.get("CXX", shutil.which("g++") or "g++")


def _newer(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ... (exit {proc.returncode})")


def build_cuda(verbose: bool = False) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    LIB.mkdir(parents=True, exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + [INCLUDE / "proxima_cuda.h"]
    objs = []
    jobs = []
    for src in CUDA_SOURCES:
        s = CSRC / src
        o = BUILD / (src + ".o")
        objs.append(o)
        if _newer(o, [s] + headers + [Path(__file__)]):
            jobs.append([NVCC, *ARCH, *NVCC_FLAGS, "-c", str(s), "-o", str(o)])
    if jobs:
        with ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            list(ex.map(_run, jobs))
    out = LIB / "libproxima_cuda.so"
    if _newer(out, objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(out), *map(str, objs), "-cudart", "static", "-ldl"])
    return out


def build_fixtures() -> Path:
    LIB.mkdir(parents=True, exist_ok=True)
    src = CSRC / "fixtures.cpp"
    out = LIB / "libpxfix.so"
    if _newer(out, [src, Path(__file__)]):
        _run([CXX, "-std=c++17", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-pthread",
              "-shared", "-o", str(out), str(src)])
    return out


def build_all() -> list[Path]:
    return [build_cuda(), build_fixtures()]


if __name__ == "__main__":
    for p in build_all():
        print(p)

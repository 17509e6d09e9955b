"""Builds the CUDA library of the sampler in-tree: verbo_b200/_lib/libverbo_cuda.so.

One nvcc invocation, sm_100a only, no fast-math (the penalty and the softmax
tail must round exactly as the reference does).  The C++ host (capi.cpp) and
the kernels (kernels.cu) link into one shared library exposing only the
symbols of include/verbo_cuda.h (-fvisibility=hidden + VERBO_CUDA_API).

    python -m verbo_b200.build
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libverbo_cuda.so"
SOURCES = [CSRC / "kernels.cu", CSRC / "nucleus.cu", CSRC / "tail.cu", CSRC / "capi.cpp"]
HEADERS = [CSRC / "device.cuh", CSRC / "kernels.cuh", CSRC / "rowdev.cuh", CSRC / "tail.cuh",
           ROOT / "include" / "verbo_cuda.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-fvisibility=hidden,-O2",
    "-shared", "-cudart", "static",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, f"-I{ROOT / 'include'}", f"-I{CSRC}", "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libverbo_cuda.so")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))

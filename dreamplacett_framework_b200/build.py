"""Build libepb200.so in-tree for sm_100a (B200).

    python -m dreamplacett_framework_b200.build [--verbose]

The library is a plain C-ABI shared object (include/epb.h); it links only
the CUDA runtime.  nvcc cross-compiles without a GPU.
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libepb200.so")
SOURCES = ["epb_engine.cu"]
HEADERS = ["epb_kernels.cuh", "fft.cuh", "geometry.cuh", "placement_kernels.cuh", "tile_kernels.cuh", "wirelength.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-cudart", "static",
]


def _nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose=False, force=False, extra=None):
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS] + [os.path.join(ROOT, "include", "epb.h")]
    if not force and not _stale(LIB, deps):
        return LIB
    cmd = [_nvcc()] + NVCC_FLAGS + list(extra or []) + \
        [os.path.join(CSRC, s) for s in SOURCES] + ["-o", LIB]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    v = "--verbose" in sys.argv
    extra = ["-Xptxas", "-v"] if "--ptxas" in sys.argv else None
    print(build(verbose=v, force="--force" in sys.argv or extra is not None, extra=extra))

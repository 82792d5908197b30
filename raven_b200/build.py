"""Compile the engine's shared library (CUDA for sm_100a + host C++) in-tree.

    python -m raven_b200.build            # -> raven_b200/lib/libraven_gpu.so

The library exports only the C ABI declared in include/raven_gpu.h.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libraven_gpu.so")

SOURCES = ["raven_gpu.cu", "host_index.cpp"]
DEPS = SOURCES + ["search_kernel.cuh", "search_cta.cuh", "knn_tc.cuh", "host_index.h"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    files = [os.path.join(CSRC, f) for f in DEPS] + [os.path.join(ROOT, "include", "raven_gpu.h"), __file__]
    return any(os.path.getmtime(f) > t for f in files)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    os.makedirs(LIBDIR, exist_ok=True)
    tmp = LIB + ".tmp"
    cmd = [
        nvcc_path(),
        "-std=c++17",
        "-O3",
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-lineinfo",
        "-shared",
        "-Xcompiler", "-fPIC,-fopenmp,-O3,-mavx2,-mfma,-fvisibility=hidden",
        "-Xptxas", "-v" if verbose else "-O3",
        "-I", os.path.join(ROOT, "include"),
        "-DRAVEN_BUILD",
        *[os.path.join(CSRC, f) for f in SOURCES],
        "-o", tmp,
        "-lgomp",
    ]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libraven_gpu.so")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)

"""Builds libfastssim.so in-tree with nvcc for sm_100a (no JIT, no torch extension).

``python build.py`` from any directory, or ``build()`` from Python.  The result
is ``lib/libfastssim.so`` next to this file; the CUDA runtime is linked
statically, so the library only needs the NVIDIA driver at run time.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = [os.path.join(HERE, "csrc", "fssim.cu"), os.path.join(HERE, "csrc", "fssim_dist.cu")]
DEPS = SRC + sorted(glob.glob(os.path.join(HERE, "csrc", "*.cuh"))) + [os.path.join(ROOT, "include", "fastssim.h")]
OUT = os.path.join(HERE, "lib", "libfastssim.so")
# The same sources with every global access bounds-checked (tests only).
OUT_BOUNDS = os.path.join(HERE, "lib", "libfastssim_bounds.so")

NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-shared", "-cudart", "static", "-ldl"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def build(force: bool = False, verbose: bool = False, bounds: bool = False) -> str:
    """Build the library (or, with ``bounds``, its bounds-checked variant) unless it
    is newer than every source."""
    out = OUT_BOUNDS if bounds else OUT
    os.makedirs(os.path.dirname(out), exist_ok=True)
    if not force and os.path.exists(out):
        newest = max(os.path.getmtime(p) for p in DEPS)
        if os.path.getmtime(out) >= newest:
            return out
    cmd = [nvcc(), *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-I", os.path.join(HERE, "csrc"),
           "-o", out, *SRC]
    if bounds:
        cmd.insert(1, "-DFSSIM_DEBUG_BOUNDS")
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return out


if __name__ == "__main__":
    force, verbose = "--force" in sys.argv, "-v" in sys.argv
    print(build(force=force, verbose=verbose))
    if "--bounds" in sys.argv:
        print(build(force=force, verbose=verbose, bounds=True))

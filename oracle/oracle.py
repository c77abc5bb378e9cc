"""ctypes front end of the CPU oracle (``liboracle_ssim.so``, built from ``ssim_oracle.c``).

TEST INFRASTRUCTURE ONLY.  This module gives the reference values for the parity tests, the
``smoke()`` check and the CPU-baseline leg of ``bench.py``.  Product code never
imports it.

Array convention: every image batch is a numpy array whose *shape* is the
canonical Julia size ``(C, H, W, N)`` and whose memory is column-major
(Fortran order), exactly like FastCUDASSIM.jl's ``CuArray{T,4}`` (reference
``src/core.jl:898-908``).  The oracle follows ``src/core.jl`` of FastCUDASSIM.jl
v0.2.1; see ``ssim_oracle.c`` for the line-by-line citations.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_ssim.so")
_lib = None

SKIP_SSIM = 1
SKIP_BACKWARD = 2
USE_DSSIM = 4
DIVIDE_BY_TWO = 8


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc); returns the library path."""
    src = os.path.join(_HERE, "ssim_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    i64 = ctypes.c_int64
    lib.oracle_kernel_weights.argtypes = [ctypes.POINTER(ctypes.c_float)]
    lib.oracle_kernel_weights.restype = None
    lib.oracle_c1.restype = ctypes.c_float
    lib.oracle_c2.restype = ctypes.c_float
    lib.oracle_ssim_f32.argtypes = [ctypes.c_void_p, ctypes.c_void_p, i64, i64, i64, i64,
                                    ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    lib.oracle_ssim_f32.restype = ctypes.c_int
    lib.oracle_ssim_f64.argtypes = lib.oracle_ssim_f32.argtypes
    lib.oracle_ssim_f64.restype = ctypes.c_int
    lib.oracle_n0f8_to_f32.argtypes = [ctypes.c_void_p, ctypes.c_void_p, i64]
    lib.oracle_n0f8_to_f32.restype = None
    _lib = lib
    return lib


def kernel_weights() -> np.ndarray:
    """The 11 Float32 Gaussian weights (reference ``src/core.jl:40-46``)."""
    k = (ctypes.c_float * 11)()
    _load().oracle_kernel_weights(k)
    return np.array(list(k), dtype=np.float32)


def constants() -> tuple[np.float32, np.float32]:
    """``(C1, C2)`` as Float32 values (reference ``src/core.jl:49-50``)."""
    lib = _load()
    return np.float32(lib.oracle_c1()), np.float32(lib.oracle_c2())


def to_compute(a: np.ndarray, dtype) -> np.ndarray:
    """Convert an input batch to the oracle's compute type.

    ``uint8`` is read as N0f8 (value = raw/255, correctly rounded in Float32);
    ``float16`` converts exactly.  The result keeps Fortran order."""
    a = np.asarray(a)
    if a.dtype == np.uint8:
        src = np.asfortranarray(a)
        out = np.empty(src.shape, dtype=np.float32, order="F")
        _load().oracle_n0f8_to_f32(src.ctypes.data, out.ctypes.data, src.size)
        return out.astype(dtype, order="F") if dtype != np.float32 else out
    return np.asfortranarray(a.astype(dtype, copy=False))


def _canon4(a: np.ndarray) -> np.ndarray:
    if a.ndim == 2:
        a = a.reshape((1,) + a.shape, order="F")
    if a.ndim == 3:
        a = a.reshape(a.shape + (1,), order="F")
    if a.ndim != 4:
        raise ValueError("expected a (C,H,W,N), (C,H,W) or (H,W) array")
    return a


def ssim(x, y, *, flags: int = 0, precision: str = "f32", nthreads: int | None = None):
    """Run the oracle.  Returns ``(ssims, grad)``.

    ``ssims``: float64 array of the final (D)SSIM values (length N; the f32 mode's
    values are Float32 numbers widened to float64), or None with SKIP_SSIM.
    ``grad``: dL/dx in canonical (C,H,W,N) Fortran layout (float32 or float64),
    or None with SKIP_BACKWARD."""
    if nthreads is None:
        nthreads = os.cpu_count() or 1
    dt = np.float32 if precision == "f32" else np.float64
    xs = _canon4(to_compute(x, dt))
    ys = _canon4(to_compute(y, dt))
    if xs.shape != ys.shape:
        raise ValueError(f"shape mismatch {xs.shape} vs {ys.shape}")
    C, H, W, N = xs.shape
    ssims = np.zeros(N, dtype=np.float64)
    grad = None if flags & SKIP_BACKWARD else np.zeros((C, H, W, N), dtype=dt, order="F")
    fn = _load().oracle_ssim_f32 if dt == np.float32 else _load().oracle_ssim_f64
    rc = fn(xs.ctypes.data, ys.ctypes.data, C, H, W, N, flags, ssims.ctypes.data,
            None if grad is None else grad.ctypes.data, int(nthreads))
    if rc != 0:
        raise RuntimeError(f"oracle failed with code {rc}")
    return (None if flags & SKIP_SSIM else ssims), grad

"""ctypes binding of ``libfastssim.so`` (C ABI declared in ``include/fastssim.h``).

The library is built in-tree by ``build.py`` into ``lib/libfastssim.so``.  There
is no fallback: if the library is missing or cannot be loaded, every call raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# FASTSSIM_LIB selects another build of the same library (e.g. a tuning variant).
LIB_PATH = os.environ.get("FASTSSIM_LIB") or os.path.join(_HERE, "lib", "libfastssim.so")

# enum fssim_dtype
FLOAT32, FLOAT16, N0F8, FLOAT64 = 0, 1, 2, 3
# enum fssim_flags
SKIP_SSIM = 1 << 0
SKIP_BACKWARD = 1 << 1
USE_DSSIM = 1 << 2
DIVIDE_BY_TWO = 1 << 3
SHOULD_ZERO = 1 << 4
# enum fssim_status
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_DIMENSION_MISMATCH = 2
ERR_UNSUPPORTED_DTYPE = 3
ERR_WORKSPACE = 4
ERR_MISALIGNED = 5
ERR_CUDA = 6
ERR_COMM = 7
ERR_TIMEOUT = 8

EXPORTED_SYMBOLS = ("fssim_version", "fssim_last_error", "fssim_workspace_size", "fssim_fwd_bwd",
                    "fssim_fwd_bwd_scaled", "fssim_fwd_bwd_noalloc", "fssim_debug_bounds_status",
                    "fssim_comm_unique_id", "fssim_comm_init", "fssim_comm_destroy", "fssim_sharded_workspace_size",
                    "fssim_fwd_bwd_sharded", "fssim_comm_wait")
# Size of the scratch array behind fssim_fwd_bwd_noalloc (FSSIM_NOALLOC_SCRATCH_BYTES).
NOALLOC_SCRATCH_BYTES = 4 << 20


class FastSSIMError(RuntimeError):
    """A nonzero status returned by the native library."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[fastssim status {status}] {message}")
        self.status = status


class DimensionMismatch(ValueError):
    """Mirror of Julia's ``DimensionMismatch`` thrown by the reference's driver."""


_lib = None


def load() -> ctypes.CDLL:
    """Load the native library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FastSSIMError(ERR_CUDA, f"native library not built: {LIB_PATH} is missing "
                                      "(run __graft_entry__.build() or fastcudassim build.py)")
    lib = ctypes.CDLL(LIB_PATH)
    i64, u32, vp, sz = ctypes.c_int64, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t
    lib.fssim_version.argtypes = []
    lib.fssim_version.restype = ctypes.c_char_p
    lib.fssim_last_error.argtypes = [ctypes.c_char_p, sz]
    lib.fssim_last_error.restype = ctypes.c_int
    lib.fssim_workspace_size.argtypes = [i64, i64, i64, i64, u32, ctypes.POINTER(sz)]
    lib.fssim_workspace_size.restype = ctypes.c_int
    lib.fssim_fwd_bwd.argtypes = [vp, ctypes.c_int, i64, vp, ctypes.c_int, vp, ctypes.c_int, vp, ctypes.c_int,
                                  vp, i64, i64, i64, i64, u32, vp, sz, vp]
    lib.fssim_fwd_bwd.restype = ctypes.c_int
    lib.fssim_fwd_bwd_scaled.argtypes = [vp, ctypes.c_int, i64, vp, ctypes.c_int, vp, ctypes.c_int, vp,
                                         ctypes.c_int, i64, i64, i64, i64, u32, vp, ctypes.c_int, vp, sz, vp]
    lib.fssim_fwd_bwd_scaled.restype = ctypes.c_int
    lib.fssim_fwd_bwd_noalloc.argtypes = [vp, ctypes.c_int, i64, vp, ctypes.c_int, vp, ctypes.c_int, vp,
                                          ctypes.c_int, i64, i64, i64, i64, u32, vp]
    lib.fssim_fwd_bwd_noalloc.restype = ctypes.c_int
    lib.fssim_debug_bounds_status.argtypes = [ctypes.POINTER(ctypes.c_uint), ctypes.POINTER(ctypes.c_ulonglong),
                                              ctypes.c_int]
    lib.fssim_debug_bounds_status.restype = ctypes.c_int
    lib.fssim_comm_unique_id.argtypes = [ctypes.c_char_p]
    lib.fssim_comm_unique_id.restype = ctypes.c_int
    lib.fssim_comm_init.argtypes = [ctypes.POINTER(vp), ctypes.c_int, ctypes.c_int, ctypes.c_char_p, ctypes.c_double]
    lib.fssim_comm_init.restype = ctypes.c_int
    lib.fssim_comm_destroy.argtypes = [vp, ctypes.c_int]
    lib.fssim_comm_destroy.restype = ctypes.c_int
    lib.fssim_sharded_workspace_size.argtypes = [i64, i64, i64, i64, ctypes.c_int, ctypes.c_int, u32, ctypes.c_int,
                                                 ctypes.POINTER(sz)]
    lib.fssim_sharded_workspace_size.restype = ctypes.c_int
    lib.fssim_fwd_bwd_sharded.argtypes = [vp, ctypes.c_int, i64, vp, ctypes.c_int, vp, ctypes.c_int, vp, ctypes.c_int,
                                          i64, i64, i64, i64, u32, vp, ctypes.c_int, ctypes.c_int, vp, sz, vp]
    lib.fssim_fwd_bwd_sharded.restype = ctypes.c_int
    lib.fssim_comm_wait.argtypes = [vp, vp, ctypes.c_double]
    lib.fssim_comm_wait.restype = ctypes.c_int
    _lib = lib
    return lib


def last_error() -> tuple[int, str]:
    buf = ctypes.create_string_buffer(512)
    st = load().fssim_last_error(buf, len(buf))
    return st, buf.value.decode(errors="replace")


def check(status: int) -> None:
    """Raise the Python exception that matches a nonzero status."""
    if status == OK:
        return
    _, msg = last_error()
    if status == ERR_DIMENSION_MISMATCH:
        raise DimensionMismatch(msg)
    raise FastSSIMError(status, msg)


def version() -> str:
    return load().fssim_version().decode()


def workspace_size(c: int, h: int, w: int, n: int, flags: int) -> int:
    out = ctypes.c_size_t(0)
    check(load().fssim_workspace_size(c, h, w, n, flags, ctypes.byref(out)))
    return int(out.value)


def fwd_bwd(ssims_ptr: int, ssims_dtype: int, ssims_len: int, grad_ptr: int, grad_dtype: int,
            x_ptr: int, x_dtype: int, y_ptr: int, y_dtype: int, qmp_ptr: int,
            c: int, h: int, w: int, n: int, flags: int, ws_ptr: int, ws_bytes: int, stream: int) -> None:
    check(load().fssim_fwd_bwd(ssims_ptr or None, ssims_dtype, ssims_len, grad_ptr or None, grad_dtype,
                               x_ptr or None, x_dtype, y_ptr or None, y_dtype, qmp_ptr or None,
                               c, h, w, n, flags, ws_ptr or None, ws_bytes, stream or None))


def fwd_bwd_scaled(ssims_ptr: int, ssims_dtype: int, ssims_len: int, grad_ptr: int, grad_dtype: int,
                   x_ptr: int, x_dtype: int, y_ptr: int, y_dtype: int, c: int, h: int, w: int, n: int,
                   flags: int, scale_ptr: int, scale_dtype: int, ws_ptr: int, ws_bytes: int, stream: int) -> None:
    """``fssim_fwd_bwd_scaled``: the gradient of image i comes out multiplied by
    ``scale[i]`` (the pullback's cotangent), with no separate broadcast."""
    check(load().fssim_fwd_bwd_scaled(ssims_ptr or None, ssims_dtype, ssims_len, grad_ptr or None, grad_dtype,
                                      x_ptr or None, x_dtype, y_ptr or None, y_dtype, c, h, w, n, flags,
                                      scale_ptr or None, scale_dtype, ws_ptr or None, ws_bytes, stream or None))


def fwd_bwd_noalloc(ssims_ptr: int, ssims_dtype: int, ssims_len: int, grad_ptr: int, grad_dtype: int,
                    x_ptr: int, x_dtype: int, y_ptr: int, y_dtype: int,
                    c: int, h: int, w: int, n: int, flags: int, stream: int) -> None:
    """``fssim_fwd_bwd_noalloc``: the same computation with the library's built-in
    scratch instead of a caller workspace, for callers that cannot allocate device
    memory.  Calls on different streams that overlap on the GPU share that scratch
    and race."""
    check(load().fssim_fwd_bwd_noalloc(ssims_ptr or None, ssims_dtype, ssims_len, grad_ptr or None, grad_dtype,
                                       x_ptr or None, x_dtype, y_ptr or None, y_dtype, c, h, w, n, flags,
                                       stream or None))


def debug_bounds_status(reset: bool = True) -> tuple[int, int]:
    """``fssim_debug_bounds_status`` of a bounds-checked build: (first failing site, count)."""
    site, count = ctypes.c_uint(0), ctypes.c_ulonglong(0)
    check(load().fssim_debug_bounds_status(ctypes.byref(site), ctypes.byref(count), int(reset)))
    return int(site.value), int(count.value)


# ---- multi-GPU (one process per GPU, NCCL loaded by the library) ----

class CommTimeout(FastSSIMError):
    """A collective did not finish within its deadline; the communicator was aborted."""


def _check_comm(status: int) -> None:
    if status == ERR_TIMEOUT:
        raise CommTimeout(status, last_error()[1])
    check(status)


def comm_unique_id() -> bytes:
    """``fssim_comm_unique_id``: 128 bytes to send from one rank to the others."""
    buf = ctypes.create_string_buffer(128)
    check(load().fssim_comm_unique_id(buf))
    return buf.raw


def comm_init(world: int, rank: int, unique_id: bytes, deadline_s: float = 60.0) -> int:
    """``fssim_comm_init``: an NCCL communicator handle (raises CommTimeout if a rank never joins)."""
    comm = ctypes.c_void_p(0)
    _check_comm(load().fssim_comm_init(ctypes.byref(comm), world, rank, unique_id, deadline_s))
    return int(comm.value)


def comm_destroy(comm: int, abort: bool = False) -> None:
    check(load().fssim_comm_destroy(comm, int(abort)))


def sharded_workspace_size(c: int, h: int, w: int, n_total: int, world: int, rank: int, flags: int,
                           ssims_dtype: int) -> int:
    out = ctypes.c_size_t(0)
    check(load().fssim_sharded_workspace_size(c, h, w, n_total, world, rank, flags, ssims_dtype, ctypes.byref(out)))
    return int(out.value)


def fwd_bwd_sharded(all_ptr: int, ssims_dtype: int, n_total: int, grad_ptr: int, grad_dtype: int,
                    x_ptr: int, x_dtype: int, y_ptr: int, y_dtype: int, c: int, h: int, w: int, n_local: int,
                    flags: int, comm: int, world: int, rank: int, ws_ptr: int, ws_bytes: int, stream: int) -> None:
    """``fssim_fwd_bwd_sharded``: this rank's shard, then the all-gather of the values."""
    _check_comm(load().fssim_fwd_bwd_sharded(all_ptr or None, ssims_dtype, n_total, grad_ptr or None, grad_dtype,
                                             x_ptr or None, x_dtype, y_ptr or None, y_dtype, c, h, w, n_local, flags,
                                             comm or None, world, rank, ws_ptr or None, ws_bytes, stream or None))


def comm_wait(comm: int, stream: int, deadline_s: float) -> None:
    """``fssim_comm_wait``: raises CommTimeout (or FastSSIMError) after aborting the communicator."""
    _check_comm(load().fssim_comm_wait(comm or None, stream or None, deadline_s))

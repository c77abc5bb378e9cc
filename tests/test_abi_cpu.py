"""The C ABI library loads without a GPU and exports every symbol include/fastssim.h declares."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    with open(os.path.join(ROOT, "include", "fastssim.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_ ]+\*?\s*(fssim_\w+)\s*\(", text, re.M)))


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    for s in ("fssim_version", "fssim_last_error", "fssim_workspace_size", "fssim_fwd_bwd"):
        assert s in syms


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._native.load()
    for s in declared_symbols():
        assert hasattr(lib, s), s
    assert set(pkg._native.EXPORTED_SYMBOLS) <= set(declared_symbols())


def test_version_and_error_channel(pkg):
    assert pkg._native.version().startswith("fastssim")
    lib = pkg._native.load()
    # argument errors are reported before any CUDA call
    st = lib.fssim_fwd_bwd(None, 0, 1, None, 0, None, 0, None, 0, None, 1, 1, 1, 1, 0, None, 0, None)
    assert st == pkg._native.ERR_INVALID_ARGUMENT
    code, msg = pkg._native.last_error()
    assert code == st and "NULL" in msg
    st = lib.fssim_fwd_bwd(None, 0, 1, None, 0, ctypes.c_void_p(16), 0, ctypes.c_void_p(16), 0, None,
                           0, 1, 1, 1, 0, None, 0, None)
    assert st == pkg._native.ERR_INVALID_ARGUMENT
    st = lib.fssim_fwd_bwd(None, 0, 1, None, 0, ctypes.c_void_p(16), 7, ctypes.c_void_p(16), 0, None,
                           1, 1, 1, 1, 0, None, 0, None)
    assert st == pkg._native.ERR_UNSUPPORTED_DTYPE
    st = lib.fssim_fwd_bwd(ctypes.c_void_p(16), 0, 2, None, 0, ctypes.c_void_p(16), 0, ctypes.c_void_p(16), 0,
                           None, 1, 1, 1, 1, pkg._native.SKIP_BACKWARD, None, 0, None)
    assert st == pkg._native.ERR_DIMENSION_MISMATCH
    with pytest.raises(pkg.DimensionMismatch):
        pkg._native.check(st)
    st = lib.fssim_fwd_bwd(None, 0, 1, None, 0, ctypes.c_void_p(16), 0, ctypes.c_void_p(16), 0, None,
                           1, 1, 1, 1, 1 << 9, None, 0, None)
    assert st == pkg._native.ERR_INVALID_ARGUMENT
    st = lib.fssim_fwd_bwd(None, 0, 1, None, 0, ctypes.c_void_p(17), 0, ctypes.c_void_p(16), 0, None,
                           1, 1, 1, 1, 0, None, 0, None)
    assert st == pkg._native.ERR_MISALIGNED


def test_nothing_requested_is_a_no_op(pkg):
    lib = pkg._native.load()
    flags = pkg._native.SKIP_SSIM | pkg._native.SKIP_BACKWARD
    st = lib.fssim_fwd_bwd(None, 0, 1, None, 0, ctypes.c_void_p(16), 0, ctypes.c_void_p(16), 0, None,
                           3, 8, 8, 2, flags, None, 0, None)
    assert st == pkg._native.OK


def test_scaled_entry_point_argument_errors(pkg):
    lib = pkg._native.load()
    nat = pkg._native
    x = ctypes.c_void_p(16)
    # a missing factor vector, a factor vector of a non-float type, a misaligned one
    st = lib.fssim_fwd_bwd_scaled(None, 0, 1, x, 0, x, 0, x, 0, 1, 8, 8, 1, nat.SKIP_SSIM, None, 0, None, 0, None)
    assert st == nat.ERR_INVALID_ARGUMENT
    st = lib.fssim_fwd_bwd_scaled(None, 0, 1, x, 0, x, 0, x, 0, 1, 8, 8, 1, nat.SKIP_SSIM, x, nat.N0F8,
                                  None, 0, None)
    assert st == nat.ERR_UNSUPPORTED_DTYPE
    st = lib.fssim_fwd_bwd_scaled(None, 0, 1, x, 0, x, 0, x, 0, 1, 8, 8, 1, nat.SKIP_SSIM, ctypes.c_void_p(18),
                                  nat.FLOAT32, None, 0, None)
    assert st == nat.ERR_MISALIGNED
    # the remaining checks are those of fssim_fwd_bwd
    st = lib.fssim_fwd_bwd_scaled(None, 0, 1, x, 0, x, 0, x, 0, 0, 8, 8, 1, nat.SKIP_SSIM, x, nat.FLOAT32,
                                  None, 0, None)
    assert st == nat.ERR_INVALID_ARGUMENT


def test_bounds_status_needs_the_checked_build(pkg):
    lib = pkg._native.load()
    site, count = ctypes.c_uint(7), ctypes.c_ulonglong(7)
    st = lib.fssim_debug_bounds_status(ctypes.byref(site), ctypes.byref(count), 0)
    assert st == pkg._native.ERR_INVALID_ARGUMENT
    assert "FSSIM_DEBUG_BOUNDS" in pkg._native.last_error()[1]


def test_outputs_overlapping_inputs_are_refused(pkg):
    """Checked before any CUDA call: 1 x 8 x 8 x 1 Float32 arrays span 256 bytes."""
    lib = pkg._native.load()
    nat = pkg._native
    x, y = 1 << 20, 1 << 21
    for grad in (x, x + 128, y - 128):
        st = lib.fssim_fwd_bwd(None, 0, 1, ctypes.c_void_p(grad), 0, ctypes.c_void_p(x), 0, ctypes.c_void_p(y), 0,
                               None, 1, 8, 8, 1, nat.SKIP_SSIM, None, 0, None)
        assert st == nat.ERR_INVALID_ARGUMENT and "overlaps" in nat.last_error()[1]
    st = lib.fssim_fwd_bwd(ctypes.c_void_p(y + 64), 0, 1, None, 0, ctypes.c_void_p(x), 0, ctypes.c_void_p(y), 0,
                           None, 1, 8, 8, 1, nat.SKIP_BACKWARD, None, 0, None)
    assert st == nat.ERR_INVALID_ARGUMENT and "overlaps" in nat.last_error()[1]


def test_absurd_sizes_are_refused_before_any_cuda_call(pkg):
    lib = pkg._native.load()
    nat = pkg._native
    x = ctypes.c_void_p(1 << 20)
    size = ctypes.c_size_t(0)
    # element count beyond int64 headroom: c*h*w = 2^40, n = 2^30
    assert lib.fssim_workspace_size(1, 1 << 20, 1 << 20, 1 << 30, 0, ctypes.byref(size)) == nat.ERR_INVALID_ARGUMENT
    st = lib.fssim_fwd_bwd(None, 0, 1, None, 0, x, 0, x, 0, None, 1, 1 << 20, 1 << 20, 1 << 30,
                           nat.SKIP_SSIM | nat.SKIP_BACKWARD, None, 0, None)
    assert st == nat.ERR_INVALID_ARGUMENT and "out of range" in nat.last_error()[1]


def test_sharded_entry_checks_its_shard_before_any_cuda_call(pkg):
    """fssim_fwd_bwd_sharded rejects a rank outside the group and a shard whose size is not
    the rank's contiguous share (the first n_total % world ranks hold one image more)."""
    nat = pkg._native
    lib = nat.load()
    args = lambda n_total, n_local, world, rank: (ctypes.c_void_p(256), nat.FLOAT32, n_total, ctypes.c_void_p(512),
                                                  nat.FLOAT32, ctypes.c_void_p(1024), nat.FLOAT32,
                                                  ctypes.c_void_p(2048), nat.FLOAT32, 3, 8, 8, n_local, 0,
                                                  ctypes.c_void_p(64), world, rank, None, 0, None)
    assert lib.fssim_fwd_bwd_sharded(*args(5, 2, 2, 2)) == nat.ERR_INVALID_ARGUMENT      # rank >= world
    assert lib.fssim_fwd_bwd_sharded(*args(5, 2, 2, 0)) == nat.ERR_DIMENSION_MISMATCH    # rank 0 holds 3 of 5
    code, msg = nat.last_error()
    assert "expected a shard of 3 images, got 2" in msg
    assert lib.fssim_fwd_bwd_sharded(*args(5, 3, 0, 0)) == nat.ERR_INVALID_ARGUMENT      # empty group

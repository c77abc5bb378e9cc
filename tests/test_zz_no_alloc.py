"""The allocation-free entry point, fssim_fwd_bwd_noalloc, against fssim_fwd_bwd.

Callers that cannot allocate device memory (a plugin host whose pool owns all
device memory, a real-time loop that forbids allocation after start-up) use
fssim_fwd_bwd_noalloc: it keeps the reduction scratch in an array compiled into
the library instead of a caller workspace.  These tests call it through the C
ABI and check that it returns what the workspace entry point returns, on two
calls in a row (the scratch is shared between calls and must not leak state).
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SSIM_ATOL = 1e-5
GRAD_RTOL_L2 = 1e-4


def _rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _noalloc(pkg, s, g, xt, yt, flags):
    nat = pkg._native
    C, H, W, N = (int(v) for v in xt.shape)
    nat.fwd_bwd_noalloc(s.data_ptr() if s is not None else 0, nat.FLOAT32, N,
                        g.data_ptr() if g is not None else 0, nat.FLOAT32,
                        xt.data_ptr(), nat.FLOAT32, yt.data_ptr(), nat.FLOAT32,
                        C, H, W, N, flags, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("shape", [(3, 200, 170, 4), (1, 135, 240, 2)])
def test_noalloc_matches_workspace_entry_point_twice(pkg, shape):
    nat = pkg._native
    syn = __import__(pkg.__name__ + ".synthetic", fromlist=["x"])
    C, H, W, N = shape
    # two calls in a row, different inputs and flags
    for seed, dssim in ((31, False), (32, True)):
        x, y = syn.host_pair(seed, shape, 0.1)
        xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
        ref_s = torch.empty(N, dtype=torch.float32, device="cuda")
        ref_g = pkg.jl_empty(shape)
        if dssim:
            pkg.dssim_with_gradient_(ref_s, ref_g, xt, yt, None, True)
        else:
            pkg.ssim_with_gradient_(ref_s, ref_g, xt, yt, None, True)
        s = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
        g = pkg.jl_zeros(shape)
        flags = nat.SHOULD_ZERO | (nat.USE_DSSIM if dssim else 0)
        _noalloc(pkg, s, g, xt, yt, flags)
        torch.cuda.synchronize()
        assert np.max(np.abs(s.cpu().numpy() - ref_s.cpu().numpy())) <= SSIM_ATOL
        assert _rel_l2(pkg.jl_to_numpy(g), pkg.jl_to_numpy(ref_g)) <= GRAD_RTOL_L2


def test_noalloc_forward_only_twice(pkg):
    nat = pkg._native
    syn = __import__(pkg.__name__ + ".synthetic", fromlist=["x"])
    shape = (3, 270, 480, 3)
    for seed in (41, 42):
        x, y = syn.host_pair(seed, shape, 0.05)
        xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
        ref = torch.empty(3, dtype=torch.float32, device="cuda")
        pkg.ssim_(ref, xt, yt)
        s = torch.full((3,), float("nan"), dtype=torch.float32, device="cuda")
        _noalloc(pkg, s, None, xt, yt, nat.SHOULD_ZERO | nat.SKIP_BACKWARD)
        torch.cuda.synchronize()
        assert np.max(np.abs(s.cpu().numpy() - ref.cpu().numpy())) <= SSIM_ATOL


def test_noalloc_rejects_sizes_beyond_its_scratch(pkg):
    nat = pkg._native
    n = 600_000           # 600k tiny images: the per-image counters alone exceed the scratch
    need = nat.workspace_size(1, 8, 8, n, 0)
    assert need > nat.NOALLOC_SCRATCH_BYTES
    with pytest.raises(nat.FastSSIMError, match="built-in scratch"):
        nat.fwd_bwd_noalloc(16, nat.FLOAT32, n, 16, nat.FLOAT32, 16, nat.FLOAT32, 16, nat.FLOAT32,
                            1, 8, 8, n, 0, 0)
    assert nat.last_error()[0] == nat.ERR_WORKSPACE

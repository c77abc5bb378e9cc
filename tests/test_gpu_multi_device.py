"""Calls on a second GPU of the same process.

The library caches per device: kernel attributes and occupancy, and the address of
the no-alloc scratch array (a device symbol has its own address on each device).
These tests run every kind of call on cuda:1 after cuda:0 and expect bitwise the
results of cuda:0 (the kernels are deterministic).  Skipped on one-GPU machines.
"""
import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")]


def _pair(pkg, shape, dev, dtype=np.float32):
    syn = __import__(pkg.__name__ + ".synthetic", fromlist=["x"])
    x, y = syn.host_pair(71, shape, 0.1, dtype=np.uint8 if dtype == np.uint8 else np.float32)
    if dtype not in (np.uint8, np.float32):
        x, y = np.asfortranarray(x.astype(dtype)), np.asfortranarray(y.astype(dtype))
    return pkg.jl_from_numpy(x, dev), pkg.jl_from_numpy(y, dev)


def _all_calls(pkg, dev):
    """Fused (Float32, N0f8), forward (tiles and streaming), Float64, and the no-alloc
    entry point, all with tensors on `dev` and the current device left at cuda:0."""
    nat = pkg._native
    out = []
    x, y = _pair(pkg, (3, 130, 110, 2), dev)
    out += list(pkg.ssim_with_gradient(x, y))
    x8, y8 = _pair(pkg, (3, 130, 110, 2), dev, np.uint8)
    out += list(pkg.dssim_with_gradient(x8, y8))
    out.append(pkg.ssim(x, y))                                    # tiles
    xs, ys = _pair(pkg, (1, 2100, 2100, 1), dev)
    out.append(pkg.ssim(xs, ys))                                  # streaming
    xd, yd = _pair(pkg, (2, 70, 50, 2), dev, np.float64)
    out += list(pkg.ssim_with_gradient(xd, yd))
    s = torch.empty(2, dtype=torch.float32, device=dev)
    g = pkg.jl_empty((3, 130, 110, 2), torch.float32, dev)
    with torch.cuda.device(dev):
        nat.fwd_bwd_noalloc(s.data_ptr(), nat.FLOAT32, 2, g.data_ptr(), nat.FLOAT32, x.data_ptr(), nat.FLOAT32,
                            y.data_ptr(), nat.FLOAT32, 3, 130, 110, 2, nat.SHOULD_ZERO,
                            torch.cuda.current_stream(dev).cuda_stream)
        torch.cuda.synchronize(dev)
    out += [s, g]
    torch.cuda.synchronize(dev)
    return [v.cpu().numpy() if isinstance(v, torch.Tensor) else np.asarray(v) for v in out]


def test_every_call_on_the_second_gpu_equals_the_first(pkg):
    assert torch.cuda.current_device() == 0
    first = _all_calls(pkg, "cuda:0")
    second = _all_calls(pkg, "cuda:1")
    assert torch.cuda.current_device() == 0
    assert len(first) == len(second)
    for a, b in zip(first, second):
        np.testing.assert_array_equal(a, b)
    third = _all_calls(pkg, "cuda:0")                             # and back, after cuda:1
    for a, b in zip(first, third):
        np.testing.assert_array_equal(a, b)

"""Parity at the exact shapes and input recipes of the five benchmark workloads.

Each workload is run through the public API at its own size, so the launch geometry
is the one the benchmark times (band heights, width segments, tiles or streaming),
and compared with the CPU oracle in both modes: the single-precision mode (the
reference's operation order, src/core.jl:256-389 and :640-782) and the float64 mode.

  1  1 x 1080 x 1920 Float32, y = clamp(x + N(0, 0.1^2)), SSIM forward
  2  3 x 1080 x 1920 Float32, y = clamp(x + N(0, 0.05^2)), SSIM forward
  3  32 x 3 x 256 x 256 Float32, x and y independent U[0,1], dssim_with_gradient!
  4  64 x 3 x 512 x 512 in N0f8 and in Float16, Float32 gradient (ssim_with_gradient);
     odd sizes 3 x 1023 x 767 and 1 x 37 x 5 in Float32, Float16 and N0f8
  5  2048 x 3 x 512 x 512 Float32, y = clamp(x + N(0, 0.1^2)), SSIM + gradient: the whole
     batch runs on the device; images are independent (src/core.jl:186), so a sample of
     them (first, last and six seeded picks) is checked against the oracle

Tolerances: per-image (D)SSIM within 1e-5 absolute, gradient within 1e-4 relative L2.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SSIM_ATOL = 1e-5
GRAD_RTOL_L2 = 1e-4


def _syn(pkg):
    return __import__(pkg.__name__ + ".synthetic", fromlist=["x"])


def _rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _check(v, g, orc, x, y, flags=0):
    for prec in ("f32", "f64"):
        rv, rg = orc.ssim(x, y, flags=flags, precision=prec)
        if v is not None:
            err = float(np.max(np.abs(np.asarray(v, np.float64) - rv)))
            assert err <= SSIM_ATOL, (prec, err)
        if g is not None:
            rel = _rel_l2(g, rg)
            assert rel <= GRAD_RTOL_L2, (prec, rel)


@pytest.mark.parametrize("channels,noise", [(1, 0.1), (3, 0.05)], ids=["config1_1x1080x1920", "config2_3x1080x1920"])
def test_fullhd_forward_at_benchmark_shape(pkg, orc, channels, noise):
    x, y = _syn(pkg).host_pair(101 + channels, (channels, 1080, 1920, 1), noise)
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    s = torch.empty(1, dtype=torch.float32, device="cuda")
    pkg.ssim_(s, xt, yt)
    torch.cuda.synchronize()
    _check(s.cpu().numpy(), None, orc, x, y, flags=orc.SKIP_BACKWARD)
    # the scalar API (a 3-D image returns a Python number) gives the same value
    assert abs(pkg.ssim(xt[..., 0], yt[..., 0]) - float(s[0])) == 0.0


def test_config3_batch32_dssim_with_gradient(pkg, orc):
    x, y = _syn(pkg).host_pair(103, (3, 256, 256, 32), None)
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    d = torch.empty(32, dtype=torch.float32, device="cuda")
    g = pkg.jl_empty((3, 256, 256, 32), torch.float32)
    pkg.dssim_with_gradient_(d, g, xt, yt, None, True)
    torch.cuda.synchronize()
    _check(d.cpu().numpy(), pkg.jl_to_numpy(g), orc, x, y, flags=orc.USE_DSSIM)


@pytest.mark.parametrize("dt", ["n0f8", "f16"])
def test_config4_batch64_converted_inputs_with_gradient(pkg, orc, dt):
    shape = (3, 512, 512, 64)
    syn = _syn(pkg)
    if dt == "n0f8":   # raw bytes ~ U{0..255}, read as raw/255
        x = np.asfortranarray((syn._splitmix(104, int(np.prod(shape))) >> np.uint64(56))
                              .astype(np.uint8).reshape(shape, order="F"))
        y = np.asfortranarray((syn._splitmix(105, int(np.prod(shape))) >> np.uint64(56))
                              .astype(np.uint8).reshape(shape, order="F"))
    else:              # Float16 ~ U[0,1]
        x = np.asfortranarray(syn.host_uniform(106, shape).astype(np.float16))
        y = np.asfortranarray(syn.host_uniform(107, shape).astype(np.float16))
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    v, g = pkg.ssim_with_gradient(xt, yt)
    torch.cuda.synchronize()
    assert v.dtype == torch.float32 and g.dtype == torch.float32   # promote_type(T, T, Float32)
    _check(v.cpu().numpy(), pkg.jl_to_numpy(g), orc, x, y)


@pytest.mark.parametrize("dt", ["f32", "f16", "n0f8"])
@pytest.mark.parametrize("shape", [(3, 1023, 767, 1), (1, 37, 5, 1)], ids=["3x1023x767", "1x37x5"])
def test_config4_odd_sizes_every_input_dtype(pkg, orc, dt, shape):
    syn = _syn(pkg)
    if dt == "n0f8":
        x, y = syn.host_pair(108, shape, 0.1, dtype=np.uint8)
    else:
        x, y = syn.host_pair(108, shape, 0.1)
        if dt == "f16":
            x, y = np.asfortranarray(x.astype(np.float16)), np.asfortranarray(y.astype(np.float16))
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    v, g = pkg.ssim_with_gradient(xt, yt)
    fv = torch.empty(shape[3], dtype=torch.float32, device="cuda")
    pkg.ssim_(fv, xt, yt)
    torch.cuda.synchronize()
    _check(v.cpu().numpy(), pkg.jl_to_numpy(g), orc, x, y)
    _check(fv.cpu().numpy(), None, orc, x, y, flags=orc.SKIP_BACKWARD)


def sample_images(n, seed=2048, extra=6):
    """First, last and `extra` seeded picks of n images (sorted, distinct)."""
    rng = np.random.default_rng(seed)
    picks = {0, n - 1} | {int(i) for i in rng.choice(n, size=min(extra, n), replace=False)}
    return sorted(picks)


def test_config5_2048_images_sampled_against_the_oracle(pkg, orc):
    if torch.cuda.get_device_properties(0).total_memory < 40 * 2**30:
        pytest.skip("needs about 20 GB of device memory")
    shape = (3, 512, 512, 2048)
    x, y = _syn(pkg).device_pair(shape, 0.1, seed=1000)
    s = torch.empty(2048, dtype=torch.float32, device="cuda")
    g = pkg.jl_empty(shape, torch.float32)
    pkg.ssim_with_gradient_(s, g, x, y, None, True)
    torch.cuda.synchronize()
    picks = sample_images(2048)
    for i in picks:
        xi, yi = pkg.jl_to_numpy(x[..., i:i + 1]), pkg.jl_to_numpy(y[..., i:i + 1])
        _check(s[i:i + 1].cpu().numpy(), pkg.jl_to_numpy(g[..., i:i + 1]), orc, xi, yi)
    # The same images as a batch of their own: the gradient is bitwise the same (every
    # pixel's arithmetic is independent of the launch geometry); the values agree to
    # rounding (a smaller batch may split the width into more segments, which changes
    # the order of the per-image sum).
    idx = torch.tensor(picks, device="cuda")
    xs, ys = x.index_select(3, idx), y.index_select(3, idx)
    xs2, ys2 = pkg.jl_empty(xs.shape), pkg.jl_empty(ys.shape)
    xs2.copy_(xs)
    ys2.copy_(ys)
    v2, g2 = pkg.ssim_with_gradient(xs2, ys2)
    torch.cuda.synchronize()
    np.testing.assert_allclose(v2.cpu().numpy(), s[idx].cpu().numpy(), rtol=0, atol=1e-6)
    np.testing.assert_array_equal(pkg.jl_to_numpy(g2), pkg.jl_to_numpy(g.index_select(3, idx)))

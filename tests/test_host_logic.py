"""Host-side logic of the Python mirror, on CPU tensors (no kernel runs)."""
import numpy as np
import pytest
import torch


def test_julia_layout_helpers(pkg):
    t = pkg.jl_empty((3, 4, 5, 2), torch.float32, "cpu")
    assert tuple(t.shape) == (3, 4, 5, 2)
    assert t.stride() == (1, 3, 12, 60)
    a = np.arange(24, dtype=np.float32).reshape((2, 3, 4), order="F")
    tt = pkg.jl_from_numpy(a, "cpu")
    assert tuple(tt.shape) == (2, 3, 4) and tt.stride() == (1, 2, 6)
    np.testing.assert_array_equal(pkg.jl_to_numpy(tt), a)
    r = pkg.jl_reshape(tt, (1, 2, 3, 4))
    assert r.data_ptr() == tt.data_ptr()
    np.testing.assert_array_equal(pkg.jl_to_numpy(r), a.reshape((1, 2, 3, 4), order="F"))


def test_canonicalize_image_rules(pkg):
    conv = __import__(pkg.__name__ + ".conversions", fromlist=["x"])
    h, w = 7, 9
    assert tuple(conv.canonicalize_image(pkg.jl_empty((h, w), device="cpu")).shape) == (1, h, w, 1)
    assert tuple(conv.canonicalize_image(pkg.jl_empty((3, h, w), device="cpu")).shape) == (3, h, w, 1)
    assert tuple(conv.canonicalize_image(pkg.jl_empty((2, h, w, 4), device="cpu")).shape) == (2, h, w, 4)
    assert tuple(conv.canonicalize_gradient_buffer(pkg.jl_empty((h, 3, w), device="cpu")).shape) == (h, 3, 1, w, 1)
    assert tuple(conv.canonicalize_gradient_buffer(pkg.jl_empty((h, 3, 2, w), device="cpu")).shape) == (h, 3, 2, w, 1)
    with pytest.raises(ValueError):
        conv.canonicalize_image(pkg.jl_empty((5,), device="cpu"))


def test_dimension_mismatch_before_any_device_work(pkg):
    a = pkg.jl_empty((3, 10, 12, 1), device="cpu")
    b = pkg.jl_empty((3, 10, 13, 1), device="cpu")
    with pytest.raises(pkg.DimensionMismatch, match="same dimensions"):
        pkg.ssim(a, b)
    with pytest.raises(pkg.DimensionMismatch, match="length the batch size"):
        pkg.ssim_(torch.zeros(2), a, a)
    with pytest.raises(pkg.DimensionMismatch, match="N_dssims_dQMP"):
        pkg.ssim_with_gradient_(None, None, a, a, pkg.jl_empty((10, 3, 2, 12, 1), device="cpu"))
    with pytest.raises(pkg.DimensionMismatch, match="dL_dimgs1"):
        pkg.ssim_gradient_(pkg.jl_empty((3, 10, 11, 1), device="cpu"), a, a, None)
    # shapes are fine but the arrays live on the host: the engine refuses to upload
    with pytest.raises(ValueError, match="CUDA device"):
        pkg.ssim(a, a)


def test_row_major_arrays_are_detected(pkg):
    conv = __import__(pkg.__name__ + ".conversions", fromlist=["x"])
    assert conv.is_column_major(pkg.jl_empty((3, 4, 5), device="cpu"))
    assert not conv.is_column_major(torch.empty(3, 4, 5))
    assert conv.is_column_major(torch.empty(1, 1, 5).permute(2, 1, 0))


def test_dtype_promotion_rule(pkg):
    core = __import__(pkg.__name__ + ".core", fromlist=["x"])
    f32, f16, u8, f64 = torch.float32, torch.float16, torch.uint8, torch.float64
    assert core.promote_dtype(u8, u8) == f32
    assert core.promote_dtype(f16, f16) == f32
    assert core.promote_dtype(f32, f64) == f64
    assert core.promote_dtype(u8, f32) == f32


def test_shard_ranges_cover_the_batch(pkg):
    sh = __import__(pkg.__name__ + ".sharded", fromlist=["x"])
    for n in (1, 7, 2048, 2049):
        for world in (1, 2, 3, 4, 8):
            parts = [sh.shard_range(n, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in parts]
            assert max(sizes) - min(sizes) <= 1


def test_synthetic_generator_is_reproducible(pkg):
    syn = __import__(pkg.__name__ + ".synthetic", fromlist=["x"])
    a = syn.host_uniform(5, (3, 4, 5))
    b = syn.host_uniform(5, (3, 4, 5))
    np.testing.assert_array_equal(a, b)
    assert a.flags.f_contiguous and a.dtype == np.float32 and 0 <= a.min() and a.max() < 1
    x, y = syn.host_pair(5, (2, 50, 40, 1), 0.1)
    assert 0 <= y.min() and y.max() <= 1 and abs(float(np.std(y - x)) - 0.1) < 0.02


def test_n0f8_conversion_formula_is_correctly_rounded():
    """The kernels convert N0f8 as fma(r, hi, r * lo) with hi = fl(1/255) and
    lo = fl(1/255 - hi) (the bit patterns in n0f8_to_f32); exact rational arithmetic
    shows it equals the correctly rounded r/255 for all 256 bytes (FixedPointNumbers'
    value), while r * fl(1/255) alone does not."""
    from fractions import Fraction

    def rne32(q: Fraction) -> np.float32:
        c = np.float32(float(q))
        cands = [np.nextafter(c, np.float32(-1)), c, np.nextafter(c, np.float32(2))]
        return min(cands, key=lambda v: (abs(Fraction(float(v)) - q), int(np.array(v).view(np.uint32)) & 1))

    hi = np.array(0x3B808081, np.uint32).view(np.float32)
    lo = np.array(0xAF7EFEFF, np.uint32).view(np.float32)
    assert hi == rne32(Fraction(1, 255)) and lo == rne32(Fraction(1, 255) - Fraction(float(hi)))
    plain_off = 0
    for r in range(256):
        p = rne32(Fraction(r) * Fraction(float(lo)))                          # r * lo
        got = rne32(Fraction(r) * Fraction(float(hi)) + Fraction(float(p)))   # one rounding (FMA)
        want = rne32(Fraction(r, 255))
        assert got == want, r
        plain_off += rne32(Fraction(r) * Fraction(float(hi))) != want
    assert plain_off > 0

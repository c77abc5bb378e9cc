"""Pins the CPU oracle to the reference's own known answers before it is trusted.

FastCUDASSIM.jl cannot run here (no Julia), so the pins are the closed forms and
known values in its test suite (test/single_pixel.jl, test/sanity_checks.jl,
test/dssim.jl, test/batch_order.jl) plus an independent float64 scipy
restatement (tests/golden/make_golden.py).  The fused_ssim golden values of
test/correctness.jl need TestImages.jl images that are not available: unpinned.
"""
import math

import numpy as np
import pytest

RTOL_F32 = math.sqrt(np.finfo(np.float32).eps)   # Julia's default isapprox rtol for Float32


def test_weights_match_reference_recipe(orc, golden):
    ka, _ = golden
    k = orc.kernel_weights()
    assert k.dtype == np.float32 and k.shape == (11,)
    np.testing.assert_array_equal(k, np.array(ka["weights_f32"], dtype=np.float32))
    np.testing.assert_array_equal(k, k[::-1])                      # symmetric
    assert abs(float(k.astype(np.float64).sum()) - 1.0) < 1e-6
    c1, c2 = orc.constants()
    assert c1 == np.float32(0.01) * np.float32(0.01) and c2 == np.float32(0.03) * np.float32(0.03)


@pytest.mark.parametrize("precision", ["f32", "f64"])
@pytest.mark.parametrize("i", [0, 1, 2])
def test_single_pixel_closed_form(orc, golden, precision, i):
    """test/single_pixel.jl:42-56: SSIM and gradient of a 1x1x1x1 image."""
    ka, _ = golden
    case = ka["single_pixel"][i]
    a, b = np.float32(case["a"]), np.float32(case["b"])
    x = np.full((1, 1, 1, 1), a, np.float32, order="F")
    y = np.full((1, 1, 1, 1), b, np.float32, order="F")
    s, g = orc.ssim(x, y, precision=precision)
    es, eg = case["f64"]
    assert s[0] == pytest.approx(es, rel=RTOL_F32)
    assert float(g.ravel()[0]) == pytest.approx(eg, rel=RTOL_F32)


def test_single_pixel_sanity_of_the_closed_form(golden):
    """test/single_pixel.jl:34-40: s(1, 0) and ds(1, 0) in closed form."""
    ka, _ = golden
    K = np.array(ka["weights_f32"], np.float64)
    W = K[5] ** 2
    C1, C2 = ka["C1"], ka["C2"]
    import sys, os
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    import make_golden
    s, ds = make_golden.single_pixel(1.0, 0.0, np.float32(ka["weights_f32"]), np.float64)
    assert s == pytest.approx(C1 * C2 / ((W ** 2 + C1) * (W - W ** 2 + C2)), rel=1e-9)
    assert ds == pytest.approx(-C1 * C2 * (4 * W ** 2 * (W - W ** 2) + 2 * (W - W ** 2) * C1 + 2 * W ** 2 * C2)
                               / ((W ** 2 + C1) * (W - W ** 2 + C2)) ** 2, rel=1e-9)


@pytest.mark.parametrize("precision", ["f32", "f64"])
def test_sanity_checks(orc, golden, precision):
    """test/sanity_checks.jl:2-16 on 200x300 zeros / ones."""
    ka, _ = golden
    z = np.zeros((1, 200, 300, 1), np.float32, order="F")
    o = np.ones((1, 200, 300, 1), np.float32, order="F")
    C1 = ka["C1"]
    s00 = orc.ssim(z, z, precision=precision)[0][0]
    s11 = orc.ssim(o, o, precision=precision)[0][0]
    s01 = orc.ssim(z, o, precision=precision)[0][0]
    assert s00 == pytest.approx(1.0, rel=RTOL_F32)
    assert s11 == pytest.approx(1.0, rel=RTOL_F32)
    assert abs(s01 - C1 / (1 + C1)) <= 1e-5
    d01 = orc.ssim(z, o, flags=orc.USE_DSSIM, precision=precision)[0][0]
    d01h = orc.ssim(z, o, flags=orc.USE_DSSIM | orc.DIVIDE_BY_TWO, precision=precision)[0][0]
    assert d01 == pytest.approx(1.0, rel=RTOL_F32)
    assert d01h == pytest.approx(0.5, rel=RTOL_F32)


def test_dssim_relations(orc):
    """test/dssim.jl:9-13 on the reference's ramp fixtures (3x200x300x1)."""
    import make_golden
    x, y = make_golden.ramps(3, 200, 300, 1)
    s, g = orc.ssim(x, y)
    d, dg = orc.ssim(x, y, flags=orc.USE_DSSIM)
    d2, dg2 = orc.ssim(x, y, flags=orc.USE_DSSIM | orc.DIVIDE_BY_TWO)
    assert d[0] == pytest.approx(1 - s[0], rel=RTOL_F32)
    assert d2[0] == pytest.approx((1 - s[0]) / 2, rel=RTOL_F32)
    np.testing.assert_allclose(dg, -g, rtol=1e-6, atol=0)
    np.testing.assert_allclose(dg2, -g / 2, rtol=1e-6, atol=0)


def test_batch_order_and_symmetry(orc):
    """test/batch_order.jl:2-22: images are independent; ssim(a,b) == ssim(b,a)."""
    import make_golden
    a, _ = make_golden.ramps(1, 200, 300, 1)
    _, b = make_golden.ramps(1, 200, 300, 1)
    x = np.asfortranarray(np.concatenate([a, b, a, b], axis=3))
    y = np.asfortranarray(np.concatenate([b, a, b, a], axis=3))
    s, g = orc.ssim(x, y)
    assert np.allclose(s, s[0], rtol=RTOL_F32)
    np.testing.assert_array_equal(g[..., 0], g[..., 2])
    np.testing.assert_array_equal(g[..., 1], g[..., 3])


@pytest.mark.parametrize("precision", ["f32", "f64"])
def test_oracle_against_independent_scipy_restatement(orc, golden, precision):
    _, cases = golden
    for name, c in cases.items():
        s, g = orc.ssim(c["x"], c["y"], flags=int(c["flags"]), precision=precision)
        np.testing.assert_allclose(s, c["vals"], rtol=0, atol=1e-6 if precision == "f32" else 1e-12,
                                   err_msg=name)
        ref = c["grad"].astype(np.float64)
        err = np.linalg.norm(g.astype(np.float64) - ref) / max(np.linalg.norm(ref), 1e-30)
        # Float32 rounding of the reference's own algorithm reaches ~8e-5 (relative
        # L2) on the smooth ramps, where local variances are small next to C2.
        assert err <= (1e-4 if precision == "f32" else 1e-6), (name, err)


def test_f32_mode_tracks_f64_mode_on_seeded_inputs(orc, pkg):
    syn = __import__(pkg.__name__ + ".synthetic", fromlist=["x"])
    x, y = syn.host_pair(3, (3, 96, 80, 2), noise=0.1)
    s32, g32 = orc.ssim(x, y, precision="f32")
    s64, g64 = orc.ssim(x, y, precision="f64")
    assert np.max(np.abs(s32 - s64)) < 1e-6
    assert np.linalg.norm(g32 - g64) / np.linalg.norm(g64) < 1e-5


def test_n0f8_conversion_is_correctly_rounded(orc):
    raw = np.arange(256, dtype=np.uint8).reshape(1, 16, 16, 1, order="F")
    f = orc.to_compute(raw, np.float32)
    exact = np.arange(256, dtype=np.float64) / 255.0
    np.testing.assert_array_equal(f.ravel(order="F"), exact.astype(np.float32))

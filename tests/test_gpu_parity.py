"""Parity of the CUDA path (through the C ABI) with the CPU oracle on seeded inputs.

Tolerances (the parity bar): per-image (D)SSIM within 1e-5 absolute; the
gradient within 1e-4 relative L2, against the single-precision oracle (the
reference's operation order) and against the float64 oracle.
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


def _run(pkg, x, y, *, mode, dssim=False, div2=False, grad_dtype=torch.float32):
    """mode: 'fwd' (ssim!/dssim!), 'both' (*_with_gradient!), 'grad' (*_gradient!)."""
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    C, H, W, N = x.shape
    vals = grad = None
    if mode == "fwd":
        out = torch.empty(N, dtype=torch.float32, device="cuda")
        if dssim:
            pkg.dssim_(out, xt, yt, True, div2)
        else:
            pkg.ssim_(out, xt, yt)
        vals = out
    else:
        g = pkg.jl_empty((C, H, W, N), grad_dtype)
        if mode == "both":
            out = torch.empty(N, dtype=torch.float32, device="cuda")
            if dssim:
                pkg.dssim_with_gradient_(out, g, xt, yt, None, True, div2)
            else:
                pkg.ssim_with_gradient_(out, g, xt, yt, None, True)
            vals = out
        else:
            if dssim:
                pkg.dssim_gradient_(g, xt, yt, None, div2)
            else:
                pkg.ssim_gradient_(g, xt, yt, None)
        grad = g
    torch.cuda.synchronize()
    v = None if vals is None else vals.cpu().numpy().astype(np.float64)
    gr = None if grad is None else pkg.jl_to_numpy(grad).astype(np.float64)
    return v, gr


def _flags(orc, dssim, div2):
    return (orc.USE_DSSIM if dssim else 0) | (orc.DIVIDE_BY_TWO if (dssim and div2) else 0)


SHAPES = [
    ("fullhd_1ch_crop", (1, 135, 240, 1), 0.1),
    ("fullhd_3ch_crop", (3, 135, 240, 1), 0.05),
    ("batch_3x256x256", (3, 256, 256, 3), None),
    ("odd_3x1023x767", (3, 1023, 767, 1), 0.1),
    ("odd_1x37x5", (1, 37, 5, 1), None),
    ("single_px", (1, 1, 1, 2), None),
    ("c2_odd", (2, 57, 33, 3), 0.1),
    ("c4_rgba", (4, 40, 129, 2), 0.1),
    ("c5_general", (5, 31, 20, 1), None),
    ("tall_narrow", (1, 600, 12, 1), 0.2),
    ("short_wide", (1, 9, 700, 1), 0.2),
    ("h512", (3, 512, 200, 1), 0.1),
]


@pytest.mark.parametrize("name,shape,noise", SHAPES, ids=[s[0] for s in SHAPES])
def test_fused_ssim_and_gradient_vs_oracle(pkg, orc, name, shape, noise):
    x, y = _syn(pkg).host_pair(17, shape, noise)
    v, g = _run(pkg, x, y, mode="both")
    rv, rg = orc.ssim(x, y, precision="f32")
    dv, dg = orc.ssim(x, y, precision="f64")
    assert np.max(np.abs(v - rv)) <= SSIM_ATOL, (v, rv)
    assert np.max(np.abs(v - dv)) <= SSIM_ATOL, (v, dv)
    assert _rel_l2(g, rg) <= GRAD_RTOL_L2
    assert _rel_l2(g, dg) <= GRAD_RTOL_L2


@pytest.mark.parametrize("name,shape,noise", SHAPES, ids=[s[0] for s in SHAPES])
def test_forward_only_vs_oracle(pkg, orc, name, shape, noise):
    x, y = _syn(pkg).host_pair(23, shape, noise)
    v, _ = _run(pkg, x, y, mode="fwd")
    rv, _ = orc.ssim(x, y, flags=orc.SKIP_BACKWARD, precision="f64")
    assert np.max(np.abs(v - rv)) <= SSIM_ATOL, (v, rv)


@pytest.mark.parametrize("dssim,div2", [(False, False), (True, False), (True, True)])
@pytest.mark.parametrize("mode", ["fwd", "both", "grad"])
def test_flag_combinations(pkg, orc, dssim, div2, mode):
    x, y = _syn(pkg).host_pair(5, (3, 70, 90, 2), 0.1)
    v, g = _run(pkg, x, y, mode=mode, dssim=dssim, div2=div2)
    rv, rg = orc.ssim(x, y, flags=_flags(orc, dssim, div2), precision="f64")
    if v is not None:
        assert np.max(np.abs(v - rv)) <= SSIM_ATOL
    if g is not None:
        assert _rel_l2(g, rg) <= GRAD_RTOL_L2


@pytest.mark.parametrize("xdt,ydt", [(np.uint8, np.uint8), (np.float16, np.float16), (np.uint8, np.float32),
                                     (np.float32, np.float16), (np.float16, np.uint8)])
def test_input_dtypes_converted_in_kernel(pkg, orc, xdt, ydt):
    """Config-4 style inputs: N0f8 and Float16 converted in-kernel, accumulated in Float32."""
    syn = _syn(pkg)
    shape = (3, 160, 150, 2)
    x8, y8 = syn.host_pair(41, shape, 0.1, dtype=np.uint8)
    xf, yf = syn.host_pair(41, shape, 0.1)
    x = x8 if xdt == np.uint8 else xf.astype(xdt)
    y = y8 if ydt == np.uint8 else yf.astype(ydt)
    x, y = np.asfortranarray(x), np.asfortranarray(y)
    v, g = _run(pkg, x, y, mode="both")
    rv, rg = orc.ssim(x, y, precision="f32")
    assert np.max(np.abs(v - rv)) <= SSIM_ATOL
    assert _rel_l2(g, rg) <= GRAD_RTOL_L2


@pytest.mark.parametrize("dt", ["n0f8", "f16"])
@pytest.mark.parametrize("shape,mode", [((3, 64, 48, 2), "fwd"), ((3, 64, 48, 2), "both"),
                                        ((3, 700, 700, 3), "fwd")], ids=["tiles", "fused", "streaming"])
def test_converted_inputs_equal_their_float32_values_bitwise(pkg, shape, mode, dt):
    """An N0f8 byte r stands for the correctly rounded Float32 r/255 (FixedPointNumbers), and
    a Float16 value converts to Float32 exactly.  The kernels convert in the loader and then
    run the same arithmetic as on Float32 inputs, so converted images must give bitwise the
    results of the Float32 images holding those values, on the tile, fused and streaming
    (above 4 Mi elements) paths.  For N0f8 every byte value occurs in the images, so a
    conversion that is off by one ulp for any byte fails here."""
    syn = _syn(pkg)
    if dt == "n0f8":
        x, y = syn.host_pair(53, shape, 0.1, dtype=np.uint8)
        x.reshape(-1, order="F")[:256] = np.arange(256, dtype=np.uint8)
        y.reshape(-1, order="F")[256:512] = np.arange(256, dtype=np.uint8)
        x32 = np.asfortranarray((x.astype(np.float64) / 255).astype(np.float32))   # correctly rounded
        y32 = np.asfortranarray((y.astype(np.float64) / 255).astype(np.float32))
    else:
        xf, yf = syn.host_pair(53, shape, 0.1)
        x, y = np.asfortranarray(xf.astype(np.float16)), np.asfortranarray(yf.astype(np.float16))
        x32, y32 = np.asfortranarray(x.astype(np.float32)), np.asfortranarray(y.astype(np.float32))
    vc, gc = _run(pkg, x, y, mode=mode)
    v32, g32 = _run(pkg, x32, y32, mode=mode)
    np.testing.assert_array_equal(vc, v32)
    if mode == "both":
        np.testing.assert_array_equal(gc, g32)


def test_float16_gradient_output(pkg, orc):
    """test/eltypes.jl:28-36: a Float16 gradient buffer is within 1e-3 of Float32."""
    x, y = _syn(pkg).host_pair(9, (3, 128, 96, 1), 0.1)
    _, g16 = _run(pkg, x, y, mode="grad", dssim=True, grad_dtype=torch.float16)
    _, g32 = _run(pkg, x, y, mode="grad", dssim=True)
    assert np.max(np.abs(g16 - g32)) < 1e-3
    _, rg = orc.ssim(x, y, flags=orc.USE_DSSIM)
    assert np.max(np.abs(g16 - rg)) < 1e-3


@pytest.mark.parametrize("sdt", [torch.float64, torch.float16])
def test_output_vector_dtypes(pkg, orc, sdt):
    x, y = _syn(pkg).host_pair(10, (1, 50, 60, 3), 0.1)
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    out = torch.zeros(3, dtype=sdt, device="cuda")
    pkg.ssim_(out, xt, yt)
    rv, _ = orc.ssim(x, y, flags=orc.SKIP_BACKWARD, precision="f64")
    tol = SSIM_ATOL if sdt == torch.float64 else 1e-3
    assert np.max(np.abs(out.cpu().double().numpy() - rv)) <= tol


def test_should_zero_false_accumulates(pkg, orc):
    """src/core.jl:919-922: without zeroing, the previous contents join the sum."""
    x, y = _syn(pkg).host_pair(12, (2, 40, 30, 2), 0.1)
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    npx = 2 * 40 * 30
    pre = torch.tensor([3.0, -5.0], dtype=torch.float64, device="cuda")
    out = pre.clone()
    pkg.ssim_(out, xt, yt, False)
    rv, _ = orc.ssim(x, y, flags=orc.SKIP_BACKWARD, precision="f64")
    np.testing.assert_allclose(out.cpu().numpy(), pre.cpu().numpy() / npx + rv, atol=SSIM_ATOL)


def test_bitwise_deterministic(pkg):
    x, y = _syn(pkg).host_pair(13, (3, 200, 170, 4), 0.1)
    a = _run(pkg, x, y, mode="both")
    b = _run(pkg, x, y, mode="both")
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])


def test_golden_scipy_cases(pkg, golden):
    _, cases = golden
    for name, c in cases.items():
        flags = int(c["flags"])
        dssim, div2 = bool(flags & 4), bool(flags & 8)
        v, g = _run(pkg, c["x"], c["y"], mode="both", dssim=dssim, div2=div2)
        assert np.max(np.abs(v - c["vals"])) <= SSIM_ATOL, name
        # smooth ramps: the Float32 algorithm itself sits ~8e-5 from float64 there
        tol = 2e-4 if name.startswith("ramps") else GRAD_RTOL_L2
        assert _rel_l2(g, c["grad"]) <= tol, (name, _rel_l2(g, c["grad"]))


@pytest.mark.parametrize("xdt,ydt", [(np.float64, np.float64), (np.float32, np.float64), (np.float64, np.uint8)])
@pytest.mark.parametrize("shape", [(3, 53, 41, 2), (1, 37, 5, 1), (2, 128, 96, 1)])
def test_float64_inputs_compute_in_double(pkg, orc, xdt, ydt, shape):
    """Float64 on either input: the whole computation runs in double precision, and
    the allocated outputs are Float64 (promote_type(T1, T2, Float32), src/core.jl:953-954;
    test/eltypes.jl:13,24-25)."""
    syn = _syn(pkg)
    x, y = syn.host_pair(61, shape, 0.1, dtype=np.float64)
    x8, y8 = syn.host_pair(61, shape, 0.1, dtype=np.uint8)
    x = x8 if xdt == np.uint8 else np.asfortranarray(x.astype(xdt))
    y = y8 if ydt == np.uint8 else np.asfortranarray(y.astype(ydt))
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    for dssim, div2 in ((False, False), (True, True)):
        if dssim:
            v, g = pkg.dssim_with_gradient(xt, yt, div2)
        else:
            v, g = pkg.ssim_with_gradient(xt, yt)
        assert v.dtype == torch.float64 and g.dtype == torch.float64
        rv, rg = orc.ssim(x, y, flags=_flags(orc, dssim, div2), precision="f64")
        assert np.max(np.abs(v.cpu().numpy() - rv)) <= 1e-10
        assert _rel_l2(pkg.jl_to_numpy(g), rg) <= 1e-9
        fv = pkg.dssim(xt, yt, div2) if dssim else pkg.ssim(xt, yt)
        assert np.max(np.abs(fv.cpu().numpy() - rv)) <= 1e-10


@pytest.mark.parametrize("shape", [(3, 65, 33, 3), (1, 32, 97, 2)])
def test_float64_gradient_only_and_narrow_gradient_outputs(pkg, orc, shape):
    """Float64 inputs through the gradient-only entry points (no values computed), into
    Float64, Float32 and Float16 gradient buffers; tiles with one row or one column
    inside the image sit on the right and bottom edges."""
    syn = _syn(pkg)
    x, y = syn.host_pair(67, shape, 0.1, dtype=np.float64)
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    for dssim in (False, True):
        _, rg = orc.ssim(x, y, flags=orc.USE_DSSIM if dssim else 0, precision="f64")
        g = pkg.dssim_gradient(xt, yt) if dssim else pkg.ssim_gradient(xt, yt)
        assert g.dtype == torch.float64
        assert _rel_l2(pkg.jl_to_numpy(g), rg) <= 1e-9
        # computed in double and rounded once: within one unit in the last place of the
        # oracle's value rounded to the buffer's dtype (Float16 values here are subnormal)
        for gdt, npdt in ((torch.float32, np.float32), (torch.float16, np.float16)):
            gb = pkg.jl_empty(shape, gdt)
            if dssim:
                pkg.dssim_gradient_(gb, xt, yt, None)
            else:
                pkg.ssim_gradient_(gb, xt, yt, None)
            want = rg.astype(npdt)
            ulp = np.spacing(np.abs(want)).astype(np.float64)
            err = np.abs(pkg.jl_to_numpy(gb).astype(np.float64) - want.astype(np.float64))
            assert np.all(err <= ulp), (gdt, float(np.max(err / ulp)))


def test_float64_gradient_output_from_float32_inputs(pkg, orc):
    x, y = _syn(pkg).host_pair(62, (3, 64, 48, 2), 0.1)
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    g = pkg.jl_empty((3, 64, 48, 2), torch.float64)
    pkg.ssim_gradient_(g, xt, yt, None)
    _, rg = orc.ssim(x, y, precision="f32")
    assert _rel_l2(pkg.jl_to_numpy(g), rg) <= GRAD_RTOL_L2


@pytest.mark.parametrize("shape", [(3, 1100, 1400, 1), (1, 600, 800, 10), (3, 256, 256, 16)],
                         ids=["3x1100x1400", "10x1x600x800", "16x3x256x256"])
def test_forward_streaming_kernel_vs_oracle(pkg, orc, shape):
    """Float32 forward calls above 4 Mi elements (several channels: from 3 Mi) take the streaming
    kernel (smaller ones run as tiles): the same tolerance against the float64 oracle."""
    x, y = _syn(pkg).host_pair(29, shape, 0.1)
    v, _ = _run(pkg, x, y, mode="fwd")
    rv, _ = orc.ssim(x, y, flags=orc.SKIP_BACKWARD, precision="f64")
    assert np.max(np.abs(v - rv)) <= SSIM_ATOL, (v, rv)
    v, _ = _run(pkg, x, y, mode="fwd", dssim=True, div2=True)
    assert np.max(np.abs(v - (1.0 - rv) / 2)) <= SSIM_ATOL


def test_forward_tile_and_streaming_kernels_agree_across_the_threshold(pkg):
    """A batch just above the tile threshold (streaming) and its images computed one at a
    time (tiles) give the same per-image values within the tolerance."""
    x, y = _syn(pkg).host_pair(31, (3, 700, 700, 3), 0.1)        # 4.41 Mi elements: streaming
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    whole = torch.empty(3, dtype=torch.float32, device="cuda")
    pkg.ssim_(whole, xt, yt)
    single = torch.empty(1, dtype=torch.float32, device="cuda")
    for i in range(3):                                               # 1.47 Mi elements each: tiles
        pkg.ssim_(single, xt[..., i:i + 1], yt[..., i:i + 1])
        assert abs(float(single[0]) - float(whole[i])) <= SSIM_ATOL


def test_forward_on_an_image_of_more_than_2_31_elements(pkg, orc):
    """1 x 46341 x 46341 (2^31 + 4633 elements) runs the 64-bit streaming kernel.  x = y gives
    SSIM 1; zeroing y's last column changes only the map near it.  The oracle on a crop of the
    last 22 columns (whose left half is unchanged, so it adds s = 1 exactly) gives the expected
    shift of the full-image mean; the rounding of the unchanged pixels cancels in the shift."""
    n = 46341
    if torch.cuda.get_device_properties(0).total_memory < 40 * 2**30:
        pytest.skip("needs 2 x 8.6 GB of device memory")
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    x = pkg.jl_empty((1, n, n, 1), torch.float32)
    x.uniform_(0.0, 1.0, generator=g)
    y = x.clone()
    same = torch.empty(1, dtype=torch.float64, device="cuda")
    pkg.ssim_(same, x, y)
    y[0, :, n - 1, 0] = 0.0
    changed = torch.empty(1, dtype=torch.float64, device="cuda")
    pkg.ssim_(changed, x, y)
    k = 22
    xc, yc = pkg.jl_to_numpy(x[:, :, n - k:, :]), pkg.jl_to_numpy(y[:, :, n - k:, :])
    del x, y
    torch.cuda.empty_cache()
    rc, _ = orc.ssim(xc, yc, flags=orc.SKIP_BACKWARD, precision="f64")
    shift = (float(rc[0]) - 1.0) * (n * k) / (n * n)
    assert abs(float(same[0]) - 1.0) <= 1e-6
    assert shift < -1e-5                                   # the change is visible at this size
    assert abs((float(changed[0]) - float(same[0])) - shift) <= 1e-9 + 1e-4 * abs(shift)


@pytest.mark.parametrize("dt", ["u8", "f16"])
def test_forward_converted_inputs_on_the_streaming_path(pkg, orc, dt):
    """N0f8 and Float16 forward calls above 4 Mi elements stream (converted in group A's loader)."""
    shape = (3, 1100, 1400, 1)
    syn = _syn(pkg)
    if dt == "u8":
        x, y = syn.host_pair(37, shape, 0.1, dtype=np.uint8)
    else:
        x, y = syn.host_pair(37, shape, 0.1)
        x, y = np.asfortranarray(x.astype(np.float16)), np.asfortranarray(y.astype(np.float16))
    v, _ = _run(pkg, x, y, mode="fwd")
    rv, _ = orc.ssim(x, y, flags=orc.SKIP_BACKWARD, precision="f32")
    assert np.max(np.abs(v - rv)) <= SSIM_ATOL, (v, rv)


@pytest.mark.parametrize("mode", ["both", "fwd"])
def test_many_channels(pkg, orc, mode):
    """C = 16 (a multispectral stack): channels are independent planes averaged per image."""
    x, y = _syn(pkg).host_pair(43, (16, 45, 38, 2), 0.1)
    v, g = _run(pkg, x, y, mode=mode)
    rv, rg = orc.ssim(x, y, flags=0 if mode == "both" else orc.SKIP_BACKWARD, precision="f64")
    assert np.max(np.abs(v - rv)) <= SSIM_ATOL
    if g is not None:
        assert _rel_l2(g, rg) <= GRAD_RTOL_L2


@pytest.mark.parametrize("mode", ["both", "fwd"])
def test_many_tiny_images(pkg, orc, mode):
    """5000 images of 1 x 9 x 13: one CTA per image, so every image's counter and
    last-CTA reduction run, thousands at once."""
    x, y = _syn(pkg).host_pair(47, (1, 9, 13, 5000), 0.2)
    v, g = _run(pkg, x, y, mode=mode)
    rv, rg = orc.ssim(x, y, flags=0 if mode == "both" else orc.SKIP_BACKWARD, precision="f64")
    assert np.max(np.abs(v - rv)) <= SSIM_ATOL
    if g is not None:
        assert _rel_l2(g, rg) <= GRAD_RTOL_L2
    # the workspace is left zeroed: a second call gives the same values
    v2, _ = _run(pkg, x, y, mode=mode)
    np.testing.assert_array_equal(v, v2)


def test_workspace_reuse_from_few_to_many_images(pkg, orc):
    """The workspace is shared by the calls on a stream.  A call with few large images writes
    many per-CTA partial sums just after its counters; a later call with more images places its
    counters over them.  Every call must leave the workspace zeroed for that to work."""
    syn = _syn(pkg)
    xb, yb = syn.host_pair(51, (3, 300, 400, 2), 0.1)          # 2 images, dozens of CTAs each
    _run(pkg, xb, yb, mode="both")
    xs, ys = syn.host_pair(53, (1, 20, 20, 200), 0.1)         # 200 counters: bytes 0..799
    for mode in ("both", "fwd"):
        v, _ = _run(pkg, xs, ys, mode=mode)
        rv, _ = orc.ssim(xs, ys, flags=0 if mode == "both" else orc.SKIP_BACKWARD, precision="f64")
        assert np.max(np.abs(v - rv)) <= SSIM_ATOL, np.argmax(np.abs(v - rv))
        _run(pkg, xb, yb, mode=mode)


MANY_CTA_CASES = [
    ("tiles_fwd", (3, 700, 500, 2), "fwd", np.float32),       # 22 x 10 tiles x 3 channels: 660 per image
    ("tiles_u8", (3, 400, 600, 3), "fwd", np.uint8),          # converted inputs, 390 tiles per image
    ("stream_fwd", (3, 1500, 1000, 1), "fwd", np.float32),    # streaming forward, above 4 Mi elements
    ("fused", (3, 1200, 900, 2), "both", np.float32),         # fused: 14 bands x 3 channels x segments
]


@pytest.mark.parametrize("name,shape,mode,dt", MANY_CTA_CASES, ids=[c[0] for c in MANY_CTA_CASES])
def test_images_of_many_ctas_leave_the_workspace_zeroed(pkg, orc, name, shape, mode, dt):
    """Images of hundreds of CTAs (tiles, streaming forward, fused): values against the
    oracle, bitwise equal on a second call, and every counter and partial sum of the
    workspace zero again after each call (the next call relies on it)."""
    core = __import__(pkg.__name__ + ".core", fromlist=["x"])
    syn = _syn(pkg)
    x, y = syn.host_pair(61, shape, 0.1, dtype=dt)
    x, y = np.asfortranarray(x), np.asfortranarray(y)
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    C, H, W, N = shape
    outs = []
    for _ in range(2):
        s = torch.empty(N, dtype=torch.float32, device="cuda")
        g = pkg.jl_empty(shape, torch.float32) if mode == "both" else None
        if g is None:
            pkg.ssim_(s, xt, yt)
        else:
            pkg.ssim_with_gradient_(s, g, xt, yt, None, True)
        torch.cuda.synchronize()
        for ws in core._workspaces.values():
            assert int(torch.count_nonzero(ws)) == 0
        outs.append((s.cpu().numpy().astype(np.float64), None if g is None else pkg.jl_to_numpy(g)))
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    rv, rg = orc.ssim(x, y, flags=0 if mode == "both" else orc.SKIP_BACKWARD, precision="f64")
    assert np.max(np.abs(outs[0][0] - rv)) <= SSIM_ATOL
    if mode == "both":
        np.testing.assert_array_equal(outs[0][1], outs[1][1])
        assert _rel_l2(outs[0][1], rg) <= GRAD_RTOL_L2


TMA_TILE_SHAPES = [(1, 1080, 1920, 1), (1, 4, 5, 3), (1, 8, 64, 2), (1, 28, 54, 1), (1, 32, 55, 2),
                   (1, 100, 300, 4), (1, 512, 512, 3)]


@pytest.mark.parametrize("shape", TMA_TILE_SHAPES, ids=["x".join(map(str, s)) for s in TMA_TILE_SHAPES])
def test_tma_tiles_vs_oracle(pkg, orc, shape):
    """One-channel Float32 forward calls with a height divisible by 4 load their tiles with
    TMA (tile rows shifted by 3, boxes zero-filled outside the image).  Against the oracle,
    bitwise equal on a second call; a view one element off 16-byte alignment takes the plain
    loads and must agree within the tolerance."""
    syn = _syn(pkg)
    x, y = syn.host_pair(67, shape, 0.1)
    v, _ = _run(pkg, x, y, mode="fwd")
    v2, _ = _run(pkg, x, y, mode="fwd")
    rv, _ = orc.ssim(x, y, flags=orc.SKIP_BACKWARD, precision="f64")
    assert np.max(np.abs(v - rv)) <= SSIM_ATOL, (v, rv)
    np.testing.assert_array_equal(v, v2)
    # the same images, one element into a larger buffer: not 16-byte aligned
    C, H, W, N = shape
    n_el = C * H * W * N
    bx = torch.empty(n_el + 1, dtype=torch.float32, device="cuda")
    by = torch.empty(n_el + 1, dtype=torch.float32, device="cuda")
    bx[1:] = torch.from_numpy(np.asfortranarray(x).reshape(-1, order="F")).cuda()
    by[1:] = torch.from_numpy(np.asfortranarray(y).reshape(-1, order="F")).cuda()
    xv = bx[1:].as_strided((C, H, W, N), (1, C, C * H, C * H * W))
    yv = by[1:].as_strided((C, H, W, N), (1, C, C * H, C * H * W))
    out = torch.empty(N, dtype=torch.float32, device="cuda")
    pkg.ssim_(out, xv, yv)
    torch.cuda.synchronize()
    assert np.max(np.abs(out.cpu().numpy().astype(np.float64) - rv)) <= SSIM_ATOL


def test_gradient_into_the_first_input_buffer(pkg, orc):
    """`ssim_gradient!(imgs1, imgs1, imgs2, nothing)` works in the reference (its backward
    launch reads x only at the pixel it writes).  The fused kernel reads neighbouring rows
    late, so the driver copies the aliased input; the C ABI refuses the overlap itself."""
    x, y = _syn(pkg).host_pair(57, (3, 150, 120, 2), 0.1)
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    buf = xt.data_ptr()
    g = pkg.ssim_gradient_(xt, xt, yt, None)
    torch.cuda.synchronize()
    assert g.data_ptr() == buf
    _, rg = orc.ssim(x, y, precision="f64")
    assert _rel_l2(pkg.jl_to_numpy(xt), rg) <= GRAD_RTOL_L2
    # the same with DSSIM/2 and the gradient written into imgs2's buffer
    x2, y2 = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    pkg.dssim_gradient_(y2, x2, y2, None, True)
    torch.cuda.synchronize()
    _, rg2 = orc.ssim(x, y, flags=orc.USE_DSSIM | orc.DIVIDE_BY_TWO, precision="f64")
    assert _rel_l2(pkg.jl_to_numpy(y2), rg2) <= GRAD_RTOL_L2


MANY_ROWS_SHAPES = [("1x300x40x600", (1, 300, 40, 600)), ("3x120x60x400", (3, 120, 60, 400))]


@pytest.mark.parametrize("name,shape", MANY_ROWS_SHAPES, ids=[s[0] for s in MANY_ROWS_SHAPES])
@pytest.mark.parametrize("mode,dssim,div2", [("both", False, False), ("both", True, True), ("grad", False, False)])
def test_many_narrow_band_rows_vs_oracle(pkg, orc, name, shape, mode, dssim, div2):
    """Thousands of narrow band rows (3600 CTAs, several waves): SSIM, DSSIM/2 and the gradient
    alone, and bitwise determinism."""
    x, y = _syn(pkg).host_pair(59, shape, 0.1)
    v, g = _run(pkg, x, y, mode=mode, dssim=dssim, div2=div2)
    rv, rg = orc.ssim(x, y, flags=_flags(orc, dssim, div2), precision="f64")
    if v is not None:
        assert np.max(np.abs(v - rv)) <= SSIM_ATOL, np.argmax(np.abs(v - rv))
    assert _rel_l2(g, rg) <= GRAD_RTOL_L2
    if mode == "both":                      # bitwise deterministic here too
        v2, g2 = _run(pkg, x, y, mode=mode, dssim=dssim, div2=div2)
        np.testing.assert_array_equal(v, v2)
        np.testing.assert_array_equal(g, g2)


def test_many_narrow_band_rows_with_gradient_factor(pkg, orc):
    shape = (1, 300, 40, 600)
    x, y = _syn(pkg).host_pair(61, shape, 0.1)
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    scale = torch.linspace(-2.0, 2.0, shape[3], device="cuda")
    _, g = pkg.ssim_fwd_bwd(None, None, xt, yt, None, False, True, False, False, False, grad_scale=scale)
    torch.cuda.synchronize()
    _, rg = orc.ssim(x, y, precision="f64")
    want = rg * scale.double().cpu().numpy().reshape(1, 1, 1, -1)
    assert _rel_l2(pkg.jl_to_numpy(g), want) <= GRAD_RTOL_L2

"""The reference's test suite (FastCUDASSIM.jl test/*.jl), restated against this engine.

Each test names the reference test it follows.  test/correctness.jl and the
TestImages inputs of test/eltypes.jl are not available; eltype rules are
checked on seeded synthetic images instead.
"""
import json
import math
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
RTOL = math.sqrt(np.finfo(np.float32).eps)
HERE = os.path.dirname(os.path.abspath(__file__))


def approx(a, b, rtol=RTOL, atol=0.0):
    a = np.asarray(a.cpu() if isinstance(a, torch.Tensor) else a, np.float64)
    b = np.asarray(b.cpu() if isinstance(b, torch.Tensor) else b, np.float64)
    # Julia's isapprox on arrays: norm(a - b) <= max(atol, rtol * max(norm(a), norm(b)))
    return np.linalg.norm(a - b) <= max(atol, rtol * max(np.linalg.norm(a), np.linalg.norm(b)))


def ramp_rows(pkg, *shape, axis):
    """range(0, 1, length=n) laid along Julia axis `axis` of a column-major array."""
    n = shape[axis]
    r = np.linspace(0, 1, n, dtype=np.float64).astype(np.float32)
    idx = [None] * len(shape)
    idx[axis] = slice(None)
    a = np.broadcast_to(r[tuple(idx)], shape)
    return pkg.jl_from_numpy(np.asfortranarray(a))


def test_sanity_checks(pkg):
    """test/sanity_checks.jl:2-16."""
    C1 = 0.01 ** 2
    img0 = pkg.jl_zeros((200, 300))
    img1 = pkg.jl_zeros((200, 300)).fill_(1.0)
    assert pkg.ssim(img0, img0) == pytest.approx(1, rel=RTOL)
    assert pkg.ssim(img1, img1) == pytest.approx(1, rel=RTOL)
    assert abs(pkg.ssim(img0, img1) - C1 / (1 + C1)) <= 1e-5
    assert abs(pkg.ssim(img0, img1) - C1 / (1 + C1)) <= 1e-4
    assert pkg.dssim(img0, img1) == pytest.approx(1, rel=RTOL)
    assert pkg.dssim(img0, img1, True) == pytest.approx(0.5, rel=RTOL)


@pytest.mark.parametrize("i", [0, 1, 2])
def test_single_pixel(pkg, i):
    """test/single_pixel.jl:42-56: closed-form SSIM and gradient of a 1x1x1x1 image."""
    with open(os.path.join(HERE, "golden", "known_answers.json")) as f:
        case = json.load(f)["single_pixel"][i]
    a = pkg.jl_zeros((1, 1, 1, 1)).fill_(np.float32(case["a"]))
    b = pkg.jl_zeros((1, 1, 1, 1)).fill_(np.float32(case["b"]))
    s, g = pkg.ssim_with_gradient(a, b)
    es, eg = case["f32"]
    assert float(s[0]) == pytest.approx(es, rel=RTOL)
    assert float(g.reshape(-1)[0]) == pytest.approx(eg, rel=RTOL)


def test_method_forwarding(pkg):
    """test/forwarding.jl:4-28: all variants agree."""
    c, h, w, b = 3, 200, 300, 1
    imgs1 = ramp_rows(pkg, c, h, w, b, axis=1)
    imgs2 = ramp_rows(pkg, c, h, w, b, axis=2)
    ssims = torch.zeros(b, device="cuda")
    dL = pkg.jl_empty((c, h, w, b))
    pkg.ssim_with_gradient_(ssims, dL, imgs1, imgs2, None, False)
    assert approx(ssims, pkg.ssim(imgs1, imgs2))
    assert approx(dL, pkg.ssim_gradient(imgs1, imgs2))
    assert approx(ssims, pkg.ssim_with_gradient(imgs1, imgs2)[0])
    assert approx(dL, pkg.ssim_with_gradient(imgs1, imgs2)[1])
    ssims_b = torch.empty_like(ssims)
    pkg.ssim_(ssims_b, imgs1, imgs2)
    assert approx(ssims, ssims_b)
    dL_b = pkg.jl_empty((c, h, w, b))
    pkg.ssim_gradient_(dL_b, imgs1, imgs2, None)
    assert approx(dL, dL_b)


def test_dssim(pkg):
    """test/dssim.jl:2-13."""
    imgs1 = ramp_rows(pkg, 3, 200, 300, 1, axis=1)
    imgs2 = ramp_rows(pkg, 3, 200, 300, 1, axis=2)
    assert approx(pkg.dssim(imgs1, imgs2), 1 - pkg.ssim(imgs1, imgs2))
    assert approx(pkg.dssim(imgs1, imgs2, True), (1 - pkg.ssim(imgs1, imgs2)) / 2)
    assert approx(pkg.dssim_gradient(imgs1, imgs2), -pkg.ssim_gradient(imgs1, imgs2))
    assert approx(pkg.dssim_gradient(imgs1, imgs2, True), -pkg.ssim_gradient(imgs1, imgs2) / 2)


def test_sizes(pkg):
    """test/sizes.jl:3-80 (the Colorant variants are Julia-side views of these arrays)."""
    h, w = 200, 300
    img1_nn = ramp_rows(pkg, h, w, axis=0)
    img2_nn = ramp_rows(pkg, h, w, axis=1)
    s_nn, g_nn = pkg.ssim_with_gradient(img1_nn, img2_nn)
    assert isinstance(s_nn, float)
    assert tuple(g_nn.shape) == (h, w)
    img1_cn = ramp_rows(pkg, 1, h, w, axis=1)
    img2_cn = ramp_rows(pkg, 1, h, w, axis=2)
    s_cn, g_cn = pkg.ssim_with_gradient(img1_cn, img2_cn)
    assert isinstance(s_cn, float) and tuple(g_cn.shape) == (1, h, w)
    img1_cb = ramp_rows(pkg, 1, h, w, 1, axis=1)
    img2_cb = ramp_rows(pkg, 1, h, w, 1, axis=2)
    s_cb, g_cb = pkg.ssim_with_gradient(img1_cb, img2_cb)
    assert isinstance(s_cb, torch.Tensor) and tuple(s_cb.shape) == (1,) and s_cb.dtype == torch.float32
    assert tuple(g_cb.shape) == (1, h, w, 1)
    # three identical channels average to the grayscale value
    img1_rn = ramp_rows(pkg, 3, h, w, axis=1)
    img2_rn = ramp_rows(pkg, 3, h, w, axis=2)
    s_rn, g_rn = pkg.ssim_with_gradient(img1_rn, img2_rn)
    assert s_nn == pytest.approx(s_cn, rel=RTOL) and s_nn == pytest.approx(float(s_cb[0]), rel=RTOL)
    assert s_nn == pytest.approx(s_rn, rel=RTOL)
    # in-place call with inconsistent but canonically equal formats (test/sizes.jl:70-80)
    ssims = torch.zeros(1, device="cuda")
    dL_cn = pkg.jl_empty((1, h, w))
    qmp_nn = pkg.jl_empty((h, 3, w))
    s_ip, g_ip = pkg.ssim_with_gradient_(ssims, dL_cn, img1_nn, img2_cb, qmp_nn)
    assert s_ip is ssims and g_ip is dL_cn
    assert approx(s_ip, s_cb) and approx(g_ip, g_cn)


def test_batch_order(pkg):
    """test/batch_order.jl:2-22."""
    c, h, w = 1, 200, 300
    a = np.broadcast_to(np.linspace(0, 1, h, dtype=np.float64).astype(np.float32)[None, :, None], (c, h, w))
    b = np.broadcast_to(np.linspace(0, 1, w, dtype=np.float64).astype(np.float32)[None, None, :], (c, h, w))
    imgs1 = pkg.jl_from_numpy(np.asfortranarray(np.stack([a, b, a, b], axis=3)))
    imgs2 = pkg.jl_from_numpy(np.asfortranarray(np.stack([b, a, b, a], axis=3)))
    ssims, grads = pkg.ssim_with_gradient(imgs1, imgs2)
    assert all(approx(s, ssims[0]) for s in ssims)
    assert approx(grads[..., 0], grads[..., 2]) and approx(grads[..., 1], grads[..., 3])


def test_eltype_promotion_synthetic(pkg):
    """test/eltypes.jl:12-26 rules on synthetic images (the TestImages inputs are unavailable)."""
    syn = __import__(pkg.__name__ + ".synthetic", fromlist=["x"])
    x8, y8 = syn.host_pair(77, (3, 96, 96), 0.2, dtype=np.uint8)
    x32 = (x8.astype(np.float64) / 255).astype(np.float32)
    y32 = (y8.astype(np.float64) / 255).astype(np.float32)
    s8 = pkg.ssim(pkg.jl_from_numpy(np.asfortranarray(x8)), pkg.jl_from_numpy(np.asfortranarray(y8)))
    s32 = pkg.ssim(pkg.jl_from_numpy(np.asfortranarray(x32)), pkg.jl_from_numpy(np.asfortranarray(y32)))
    assert isinstance(s8, float) and s8 == pytest.approx(s32, rel=RTOL)
    g8 = pkg.ssim_gradient(pkg.jl_from_numpy(np.asfortranarray(x8)), pkg.jl_from_numpy(np.asfortranarray(y8)))
    assert g8.dtype == torch.float32
    x16 = pkg.jl_from_numpy(np.asfortranarray(x32.astype(np.float16)))
    y16 = pkg.jl_from_numpy(np.asfortranarray(y32.astype(np.float16)))
    assert isinstance(pkg.ssim(x16, y16), float)
    # Float32 with Float64 -> Float64 (test/eltypes.jl:13); N0f8 == Float32 == Float64 values (:16-18)
    x64 = pkg.jl_from_numpy(np.asfortranarray(x32.astype(np.float64)))
    y64 = pkg.jl_from_numpy(np.asfortranarray(y32.astype(np.float64)))
    s64 = pkg.ssim(x64, y64)
    assert isinstance(s64, float) and s64 == pytest.approx(s32, rel=RTOL) and s64 == pytest.approx(s8, rel=RTOL)
    xb = pkg.jl_reshape(pkg.jl_from_numpy(np.asfortranarray(x32)), (3, 96, 96, 1))
    yb = pkg.jl_reshape(y64, (3, 96, 96, 1))
    sb = pkg.ssim(xb, yb)
    assert sb.dtype == torch.float64
    # the gradient follows the first image's format, promoted (test/eltypes.jl:24-25)
    assert pkg.ssim_gradient(x64, pkg.jl_from_numpy(np.asfortranarray(x8))).dtype == torch.float64
    assert pkg.ssim_gradient(pkg.jl_from_numpy(np.asfortranarray(x8)), x64).dtype == torch.float64


def test_autodiff(pkg):
    """test/autodiff.jl:1-27 through the torch counterpart of the rrule."""
    h, w = 200, 300
    img1 = ramp_rows(pkg, h, w, axis=0).requires_grad_(True)
    img2 = ramp_rows(pkg, h, w, axis=1)
    zs = pkg.ssim_autograd(img1, img2)
    zs.backward()
    fs, fg = pkg.ssim_with_gradient(img1.detach(), img2)
    assert float(zs) == pytest.approx(fs, rel=RTOL)
    assert approx(img1.grad, fg)
    imgs1 = ramp_rows(pkg, 1, h, w, 1, axis=1).requires_grad_(True)
    imgs2 = ramp_rows(pkg, 1, h, w, 1, axis=2)
    zd = pkg.dssim_autograd(imgs1, imgs2, True)
    zd.sum().backward()
    fd, fg = pkg.dssim_with_gradient(imgs1.detach(), imgs2, True)
    assert float(zd.sum()) == pytest.approx(float(fd.sum()), rel=RTOL)
    assert approx(imgs1.grad, fg)
    # batch cotangent scales each image's gradient (ext/...:35)
    imgs1.grad = None
    cot = torch.tensor([3.0], device="cuda")
    pkg.dssim_autograd(imgs1, imgs2).backward(cot)
    assert approx(imgs1.grad, 3 * pkg.dssim_gradient(imgs1.detach(), imgs2))

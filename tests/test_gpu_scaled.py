"""Per-image gradient factor (``fssim_fwd_bwd_scaled``) and the deferred autograd rule.

The scaled call must give grad_scale[i] times the unscaled gradient of image i
(checked against the oracle's gradient times the same factor, relative L2
1e-4) and leave the (D)SSIM values unscaled (1e-5 absolute).  The deferred rule
must match the eager rule of ext/FastCUDASSIMChainRulesCoreExt.jl.
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


def _inputs(pkg, shape, xdt, ydt, seed):
    syn = _syn(pkg)
    x8, y8 = syn.host_pair(seed, shape, 0.1, dtype=np.uint8)
    xf, yf = syn.host_pair(seed, shape, 0.1, dtype=np.float64)
    x = x8 if xdt == np.uint8 else np.asfortranarray(xf.astype(xdt))
    y = y8 if ydt == np.uint8 else np.asfortranarray(yf.astype(ydt))
    return x, y


@pytest.mark.parametrize("xdt,ydt", [(np.float32, np.float32), (np.uint8, np.uint8), (np.float16, np.float16),
                                     (np.uint8, np.float32), (np.float64, np.float64)])
@pytest.mark.parametrize("sdt", [torch.float32, torch.float64, torch.float16])
def test_scaled_gradient_vs_oracle(pkg, orc, xdt, ydt, sdt):
    shape = (3, 75, 66, 4)
    x, y = _inputs(pkg, shape, xdt, ydt, 71)
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    scale = torch.tensor([2.5, -0.75, 0.0, 1.0], dtype=sdt, device="cuda")
    f64 = np.float64 in (xdt, ydt)
    prec = "f64" if f64 else "f32"
    for dssim, div2 in ((False, False), (True, False), (True, True)):
        flags = (orc.USE_DSSIM if dssim else 0) | (orc.DIVIDE_BY_TWO if div2 else 0)
        v, g = pkg.ssim_fwd_bwd(None, None, xt, yt, None, False, False, False, dssim, div2, grad_scale=scale)
        torch.cuda.synchronize()
        rv, rg = orc.ssim(x, y, flags=flags, precision=prec)
        want = rg * scale.double().cpu().numpy().reshape(1, 1, 1, -1)
        got = pkg.jl_to_numpy(g).astype(np.float64)
        assert np.max(np.abs(v.double().cpu().numpy() - rv)) <= (1e-10 if f64 else SSIM_ATOL)
        assert _rel_l2(got, want) <= (1e-9 if f64 else GRAD_RTOL_L2)
        assert np.all(got[..., 2] == 0.0)          # a zero factor gives an exactly zero gradient
        # gradient only (skip_ssim), as the deferred pullback calls it
        _, g2 = pkg.ssim_fwd_bwd(None, None, xt, yt, None, False, True, False, dssim, div2, grad_scale=scale)
        torch.cuda.synchronize()
        assert _rel_l2(pkg.jl_to_numpy(g2), want) <= (1e-9 if f64 else GRAD_RTOL_L2)


def test_scaled_by_one_is_bitwise_unscaled(pkg):
    x, y = _syn(pkg).host_pair(72, (3, 140, 90, 3), 0.1)
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    _, g0 = pkg.ssim_with_gradient(xt, yt)
    _, g1 = pkg.ssim_fwd_bwd(None, None, xt, yt, None, False, False, False, False, False,
                             grad_scale=torch.ones(3, device="cuda"))
    torch.cuda.synchronize()
    assert torch.equal(g0, g1)


def test_scale_length_is_checked(pkg):
    x, y = _syn(pkg).host_pair(73, (1, 20, 20, 3), 0.1)
    xt, yt = pkg.jl_from_numpy(x), pkg.jl_from_numpy(y)
    with pytest.raises(pkg.DimensionMismatch):
        pkg.ssim_fwd_bwd(None, None, xt, yt, None, False, False, False, False, False,
                         grad_scale=torch.ones(2, device="cuda"))


@pytest.mark.parametrize("use_dssim,div2", [(False, False), (True, True)])
def test_deferred_autograd_matches_eager(pkg, use_dssim, div2):
    x, y = _syn(pkg).host_pair(74, (3, 96, 80, 3), 0.1)
    cot = torch.tensor([0.5, -2.0, 3.0], device="cuda")
    grads, vals = [], []
    for defer in (False, True):
        xt = pkg.jl_from_numpy(x).requires_grad_(True)
        yt = pkg.jl_from_numpy(y)
        z = (pkg.dssim_autograd(xt, yt, div2, defer_gradient=defer) if use_dssim
             else pkg.ssim_autograd(xt, yt, defer_gradient=defer))
        z.backward(cot)
        vals.append(z.detach())
        grads.append(xt.grad)
    assert torch.allclose(vals[0], vals[1], atol=SSIM_ATOL, rtol=0)
    a, b = grads[0].double().cpu().numpy(), grads[1].double().cpu().numpy()
    assert _rel_l2(b, a) <= GRAD_RTOL_L2


def test_deferred_autograd_without_batch_axis(pkg):
    x, y = _syn(pkg).host_pair(75, (1, 64, 48, 1), 0.1)
    xt = pkg.jl_reshape(pkg.jl_from_numpy(x), (64, 48)).requires_grad_(True)
    yt = pkg.jl_reshape(pkg.jl_from_numpy(y), (64, 48))
    z = pkg.ssim_autograd(xt, yt, defer_gradient=True)
    assert z.ndim == 0
    (2 * z).backward()
    ref = pkg.ssim_gradient(xt.detach(), yt)
    assert tuple(xt.grad.shape) == (64, 48)
    assert _rel_l2(xt.grad.double().cpu().numpy(), 2 * ref.double().cpu().numpy()) <= GRAD_RTOL_L2

"""Reverse-mode rules: the torch counterpart of ext/FastCUDASSIMChainRulesCoreExt.jl.

``ssim_autograd(imgs1, imgs2)`` / ``dssim_autograd(imgs1, imgs2, divide_by_two)``
return the (D)SSIM values as a tensor (0-d for an input without a batch axis)
and differentiate with respect to ``imgs1``; ``imgs2`` and the flag get no
gradient.  As in the reference rrule (ext/...:19-44, :54-73) the forward pass
computes values and gradient in one call, and the pullback scales the stored
gradient IN PLACE by the cotangent, broadcast over the batch axis.

``defer_gradient=True`` is an alternative with no counterpart in the
reference: the forward pass computes only the values (the forward-only
kernel) and keeps the inputs; the pullback computes the gradient with the
cotangent folded into the kernel as a per-image factor
(``fssim_fwd_bwd_scaled``).  No gradient array lives between the two passes
and no broadcast pass runs, at the price of reading the inputs twice.
"""
from __future__ import annotations

import torch

from .core import ssim_fwd_bwd
from .interface import dssim, dssim_with_gradient, ssim, ssim_with_gradient


class _SSIMRule(torch.autograd.Function):
    @staticmethod
    def forward(ctx, imgs1, imgs2, use_dssim: bool, divide_by_two: bool):
        if use_dssim:
            vals, grad = dssim_with_gradient(imgs1.detach(), imgs2.detach(), divide_by_two)
        else:
            vals, grad = ssim_with_gradient(imgs1.detach(), imgs2.detach())
        scalar = not isinstance(vals, torch.Tensor)
        if scalar:
            vals = torch.tensor(vals, dtype=grad.dtype, device=grad.device)
        ctx.grad_imgs1 = grad
        ctx.scalar = scalar
        return vals

    @staticmethod
    def backward(ctx, cot):
        g = ctx.grad_imgs1
        ctx.grad_imgs1 = None
        if ctx.scalar:
            g.mul_(cot.to(g.dtype))
        else:
            # reshape(dL_dssims, 1, ..., 1, :): the batch axis is the last Julia axis
            g.mul_(cot.to(g.dtype).reshape((1,) * (g.ndim - 1) + (-1,)))
        return g, None, None, None


class _DeferredSSIMRule(torch.autograd.Function):
    @staticmethod
    def forward(ctx, imgs1, imgs2, use_dssim: bool, divide_by_two: bool):
        x, y = imgs1.detach(), imgs2.detach()
        vals = dssim(x, y, divide_by_two) if use_dssim else ssim(x, y)
        if not isinstance(vals, torch.Tensor):
            vals = torch.tensor(vals, dtype=torch.float64 if torch.float64 in (x.dtype, y.dtype) else torch.float32,
                                device=x.device)
        ctx.inputs = (x, y)
        ctx.use_dssim = use_dssim
        ctx.divide_by_two = divide_by_two
        return vals

    @staticmethod
    def backward(ctx, cot):
        x, y = ctx.inputs
        ctx.inputs = None
        _, g = ssim_fwd_bwd(None, None, x, y, None, False, True, False, ctx.use_dssim, ctx.divide_by_two,
                            grad_scale=cot.detach().reshape(-1))
        return g, None, None, None


def ssim_autograd(imgs1, imgs2, defer_gradient: bool = False):
    """Differentiable ``ssim`` (ext/FastCUDASSIMChainRulesCoreExt.jl:15-45)."""
    rule = _DeferredSSIMRule if defer_gradient else _SSIMRule
    return rule.apply(imgs1, imgs2, False, False)


def dssim_autograd(imgs1, imgs2, divide_by_two_in_dssim=False, defer_gradient: bool = False):
    """Differentiable ``dssim`` (ext/FastCUDASSIMChainRulesCoreExt.jl:54-74)."""
    rule = _DeferredSSIMRule if defer_gradient else _SSIMRule
    return rule.apply(imgs1, imgs2, True, bool(divide_by_two_in_dssim))

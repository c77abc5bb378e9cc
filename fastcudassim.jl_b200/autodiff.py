"""Reverse-mode rules: the torch counterpart of ext/FastCUDASSIMChainRulesCoreExt.jl.

``ssim_autograd(imgs1, imgs2)`` / ``dssim_autograd(imgs1, imgs2, divide_by_two)``
return the (D)SSIM values as a tensor (0-d for an input without a batch axis)
and differentiate with respect to ``imgs1``; ``imgs2`` and the flag get no
gradient.  As in the reference rrule (ext/...:19-44, :54-73) the forward pass
computes values and gradient in one call, and the pullback scales the stored
gradient IN PLACE by the cotangent, broadcast over the batch axis.
"""
from __future__ import annotations

import torch

from .interface import dssim_with_gradient, ssim_with_gradient


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


def ssim_autograd(imgs1, imgs2):
    """Differentiable ``ssim`` (ext/FastCUDASSIMChainRulesCoreExt.jl:15-45)."""
    return _SSIMRule.apply(imgs1, imgs2, False, False)


def dssim_autograd(imgs1, imgs2, divide_by_two_in_dssim=False):
    """Differentiable ``dssim`` (ext/FastCUDASSIMChainRulesCoreExt.jl:54-74)."""
    return _SSIMRule.apply(imgs1, imgs2, True, bool(divide_by_two_in_dssim))

"""fastcudassim.jl_b200: B200-native SSIM / DSSIM engine behind FastCUDASSIM.jl's API.

The compute path is ``lib/libfastssim.so`` (hand-written CUDA for sm_100a, C ABI
in ``include/fastssim.h``).  This package is its host-side mirror of the
reference's Julia API, used by the tests and the benchmark:

  interface   the twelve exported functions (``ssim``, ``ssim_``, ``dssim_with_gradient_``, ...)
  core        the driver ``ssim_fwd_bwd`` (reference ``_ssim_fwd_bwd!``)
  conversions Julia-layout arrays on torch and the canonical-format rules
  autodiff    the ChainRulesCore ``rrule`` as a torch.autograd.Function
  sharded     batch sharding over GPUs with an all-gather of the scores
  synthetic   seeded benchmark inputs
"""
from . import _native
from ._native import DimensionMismatch, FastSSIMError
from .autodiff import dssim_autograd, ssim_autograd
from .conversions import jl_empty, jl_from_numpy, jl_reshape, jl_to_numpy, jl_zeros
from .core import ssim_fwd_bwd
from .interface import (dssim, dssim_, dssim_gradient, dssim_gradient_, dssim_with_gradient,
                        dssim_with_gradient_, ssim, ssim_, ssim_gradient, ssim_gradient_,
                        ssim_with_gradient, ssim_with_gradient_)

__all__ = [
    "ssim", "ssim_gradient", "ssim_with_gradient",
    "ssim_", "ssim_gradient_", "ssim_with_gradient_",
    "dssim", "dssim_gradient", "dssim_with_gradient",
    "dssim_", "dssim_gradient_", "dssim_with_gradient_",
    "ssim_autograd", "dssim_autograd", "ssim_fwd_bwd",
    "jl_empty", "jl_zeros", "jl_from_numpy", "jl_to_numpy", "jl_reshape",
    "DimensionMismatch", "FastSSIMError",
]


def version() -> str:
    return _native.version()

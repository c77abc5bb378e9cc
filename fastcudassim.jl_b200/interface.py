"""Public API: the twelve exported functions of FastCUDASSIM.jl (src/interface.jl:1-338).

Julia's mutating ``name!`` becomes ``name_`` here (Python identifiers cannot
contain ``!``); arguments, defaults, flag mapping and return values follow the
reference.  As in the reference code (not its docstring at src/interface.jl:54),
``divide_by_two_in_dssim`` defaults to ``False`` everywhere.
"""
from __future__ import annotations

from .core import ssim_fwd_bwd


def ssim_with_gradient_(ssims, dL_dimgs1, imgs1, imgs2, N_dssims_dQMP, should_zero=True):
    """src/interface.jl:31-45 -> ``(ssims, dL_dimgs1)``."""
    return ssim_fwd_bwd(ssims, dL_dimgs1, imgs1, imgs2, N_dssims_dQMP, should_zero,
                        False, False, False, False)


def dssim_with_gradient_(dssims, dL_dimgs1, imgs1, imgs2, N_dssims_dQMP, should_zero=True,
                         divide_by_two_in_dssim=False):
    """src/interface.jl:64-79 -> ``(dssims, dL_dimgs1)``."""
    return ssim_fwd_bwd(dssims, dL_dimgs1, imgs1, imgs2, N_dssims_dQMP, should_zero,
                        False, False, True, divide_by_two_in_dssim)


def ssim_gradient_(dL_dimgs1, imgs1, imgs2, N_dssims_dQMP):
    """src/interface.jl:94-107 -> ``dL_dimgs1``."""
    return ssim_fwd_bwd(None, dL_dimgs1, imgs1, imgs2, N_dssims_dQMP, False,
                        True, False, False, False)[1]


def dssim_gradient_(dL_dimgs1, imgs1, imgs2, N_dssims_dQMP, divide_by_two_in_dssim=False):
    """src/interface.jl:125-139 -> ``dL_dimgs1``."""
    return ssim_fwd_bwd(None, dL_dimgs1, imgs1, imgs2, N_dssims_dQMP, False,
                        True, False, True, divide_by_two_in_dssim)[1]


def ssim_with_gradient(imgs1, imgs2):
    """src/interface.jl:162-171 -> ``(ssims, dL_dimgs1)``, both allocated."""
    return ssim_with_gradient_(None, None, imgs1, imgs2, None, False)


def dssim_with_gradient(imgs1, imgs2, divide_by_two_in_dssim=False):
    """src/interface.jl:187-196."""
    return dssim_with_gradient_(None, None, imgs1, imgs2, None, False, divide_by_two_in_dssim)


def ssim_gradient(imgs1, imgs2):
    """src/interface.jl:209-217."""
    return ssim_gradient_(None, imgs1, imgs2, None)


def dssim_gradient(imgs1, imgs2, divide_by_two_in_dssim=False):
    """src/interface.jl:235-244."""
    return dssim_gradient_(None, imgs1, imgs2, None, divide_by_two_in_dssim)


def ssim_(ssims, imgs1, imgs2, should_zero=True):
    """src/interface.jl:260-273 -> ``ssims``."""
    return ssim_fwd_bwd(ssims, None, imgs1, imgs2, None, should_zero, False, True, False, False)[0]


def dssim_(dssims, imgs1, imgs2, should_zero=True, divide_by_two_in_dssim=False):
    """src/interface.jl:292-306 -> ``dssims``."""
    return ssim_fwd_bwd(dssims, None, imgs1, imgs2, None, should_zero, False, True, True,
                        divide_by_two_in_dssim)[0]


def ssim(imgs1, imgs2):
    """src/interface.jl:319-321: SSIM values (a Python float for an input without a batch axis)."""
    return ssim_(None, imgs1, imgs2, False)


def dssim(imgs1, imgs2, divide_by_two_in_dssim=False):
    """src/interface.jl:336-338."""
    return dssim_(None, imgs1, imgs2, False, divide_by_two_in_dssim)

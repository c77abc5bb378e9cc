"""Julia-layout arrays on torch, and the format rules of FastCUDASSIM.jl's src/conversions.jl.

A *Julia array* here is a ``torch.Tensor`` whose ``shape`` is the Julia ``size``
and whose memory is column-major (first index fastest), exactly like a
``CuArray``.  ``jl_empty``/``jl_zeros``/``jl_from_numpy`` create them;
``jl_reshape`` is Julia's ``reshape`` (a view, never a copy).

Julia's ``Colorant`` element types (``Gray``, ``RGB``) are zero-copy views over
such arrays (``channelview``); on this side of the boundary the caller passes
the channel view itself, e.g. an RGB ``h x w`` image is a ``(3, h, w)`` array.
"""
from __future__ import annotations

import numpy as np
import torch


def is_column_major(t: torch.Tensor) -> bool:
    """True if ``t`` is laid out like a Julia array of size ``t.shape`` (dimensions of
    size 1 may have any stride)."""
    expect = 1
    for size, stride in zip(t.shape, t.stride()):
        if size != 1 and stride != expect:
            return False
        expect *= size
    return True


def jl_empty(shape, dtype=torch.float32, device="cuda") -> torch.Tensor:
    shape = tuple(int(s) for s in shape)
    t = torch.empty(tuple(reversed(shape)), dtype=dtype, device=device)
    return t.permute(*reversed(range(len(shape))))


def jl_zeros(shape, dtype=torch.float32, device="cuda") -> torch.Tensor:
    return jl_empty(shape, dtype, device).zero_()


def jl_from_numpy(a: np.ndarray, device="cuda") -> torch.Tensor:
    """Copy a numpy array (any order) into a Julia-layout tensor of the same shape."""
    a = np.asarray(a)
    t = jl_empty(a.shape, torch.from_numpy(np.zeros(0, dtype=a.dtype)).dtype, device)
    t.copy_(torch.from_numpy(np.ascontiguousarray(a)))
    return t


def jl_to_numpy(t: torch.Tensor) -> np.ndarray:
    """Fortran-ordered numpy copy of a Julia-layout tensor (same shape)."""
    return np.asfortranarray(t.detach().cpu().numpy())


def jl_reshape(t: torch.Tensor, shape) -> torch.Tensor:
    """Julia ``reshape``: same column-major memory, new size.  Never copies."""
    shape = tuple(int(s) for s in shape)
    if not is_column_major(t):
        raise ValueError("jl_reshape needs a column-major (Julia-layout) tensor")
    n = 1
    for s in shape:
        n *= s
    if n != t.numel():
        raise ValueError(f"cannot reshape an array of {t.numel()} elements to size {shape}")
    strides, acc = [], 1
    for s in shape:
        strides.append(acc)
        acc *= s
    return t.as_strided(shape, tuple(strides))


def canonicalize_image(img: torch.Tensor) -> torch.Tensor:
    """``_canonicalize_image`` (src/conversions.jl:20-36): (h,w) -> (1,h,w,1),
    (c,h,w) -> (c,h,w,1), (c,h,w,n) unchanged.  A 3-D array is one c-channel
    image, never a grayscale batch (src/conversions.jl:14-18)."""
    if img.ndim == 2:
        return jl_reshape(img, (1,) + tuple(img.shape) + (1,))
    if img.ndim == 3:
        return jl_reshape(img, tuple(img.shape) + (1,))
    if img.ndim == 4:
        return img
    raise ValueError(f"cannot interpret a {img.ndim}-dimensional array as an image batch (c, h, w, n)")


def canonicalize_gradient_buffer(gb: torch.Tensor) -> torch.Tensor:
    """``_canonicalize_gradient_buffer`` (src/conversions.jl:46-54): (h,3,w) ->
    (h,3,1,w,1), (h,3,c,w) -> (h,3,c,w,1), 5-D unchanged."""
    if gb.ndim == 3:
        return jl_reshape(gb, (gb.shape[0], gb.shape[1], 1, gb.shape[2], 1))
    if gb.ndim == 4:
        return jl_reshape(gb, tuple(gb.shape) + (1,))
    return gb


def decanonicalize_gradient_image(dl: torch.Tensor, img: torch.Tensor) -> torch.Tensor:
    """``_decanonicalize_gradient_image`` (src/conversions.jl:66-89): back to ``size(img)``."""
    return jl_reshape(dl, tuple(img.shape))


def should_unpack(vals: torch.Tensor, img: torch.Tensor) -> bool:
    """``_should_unpack_and_free`` (src/conversions.jl:114-120): a singleton result
    for an input without a batch axis is returned as a scalar."""
    return img.ndim <= 3 and tuple(vals.shape) == (1,)

"""Host driver: the Python mirror of ``_ssim_fwd_bwd!`` (FastCUDASSIM.jl src/core.jl:933-1107).

Canonicalisation, shape checks (``DimensionMismatch``), allocation of missing
outputs and the scalar unpack stay on the host, as in the reference.  The device
work - which the reference split over a memset, two kernels and a broadcast - is
one call into ``libfastssim.so`` (``fssim_fwd_bwd``), which launches one kernel.
"""
from __future__ import annotations

import threading

import torch

from . import _native as nat
from .conversions import (canonicalize_gradient_buffer, canonicalize_image,
                          decanonicalize_gradient_image, is_column_major, jl_empty, should_unpack)

_DTYPE_CODE = {torch.float32: nat.FLOAT32, torch.float16: nat.FLOAT16, torch.uint8: nat.N0F8,
               torch.float64: nat.FLOAT64}
_CODE_DTYPE = {v: k for k, v in _DTYPE_CODE.items()}

# Zero-filled scratch for the per-image reductions, one per (device, stream).
# Every call leaves its workspace zero-filled again, so it is reused as is.
_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


# fssim_workspace_size results per (sizes, flags, device): the value depends only
# on those, and computing it configures every kernel variant.
_ws_sizes: dict[tuple[int, int, int, int, int, int], int] = {}


def _workspace_size(c: int, h: int, w: int, n: int, flags: int, device_index: int) -> int:
    key = (c, h, w, n, flags, device_index)
    nbytes = _ws_sizes.get(key)
    if nbytes is None:
        nbytes = nat.workspace_size(c, h, w, n, flags)
        if len(_ws_sizes) > 4096:
            _ws_sizes.clear()
        _ws_sizes[key] = nbytes
    return nbytes


def _current_stream_handle(device_index: int) -> int:
    """The raw cudaStream_t of the current stream of a device (without building a
    torch Stream object on every call)."""
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return int(raw(device_index))
    return torch.cuda.current_stream(device_index).cuda_stream


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    key = (device.index, stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
            _workspaces[key] = ws
        return ws


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError:
        raise nat.FastSSIMError(nat.ERR_UNSUPPORTED_DTYPE, f"unsupported element type {t.dtype}") from None


def promote_dtype(t1: torch.dtype, t2: torch.dtype) -> torch.dtype:
    """``promote_type(T1, T2, Float32)`` for the element types this engine accepts
    (src/core.jl:953-954): Float64 if either is Float64, else Float32 (N0f8 and
    Float16 promote to Float32)."""
    return torch.float64 if torch.float64 in (t1, t2) else torch.float32


def _span(t: torch.Tensor) -> tuple[int, int]:
    return t.data_ptr(), t.data_ptr() + t.numel() * t.element_size()


def _overlap(a: torch.Tensor, b: torch.Tensor) -> bool:
    (a0, a1), (b0, b1) = _span(a), _span(b)
    return a.device == b.device and a0 < b1 and b0 < a1


def _jl_copy(t: torch.Tensor) -> torch.Tensor:
    out = jl_empty(tuple(t.shape), t.dtype, t.device)
    out.copy_(t)
    return out


def _require_device_array(name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor in Julia (column-major) layout")
    if not t.is_cuda:
        raise ValueError(f"{name} must live on a CUDA device (got {t.device}); CPU arrays are not uploaded")
    if not is_column_major(t):
        raise ValueError(f"{name} must be column-major (Julia layout); use conversions.jl_empty/jl_reshape")


def ssim_fwd_bwd(ssims, dL_dimgs1, imgs1, imgs2, N_dssims_dQMP, should_zero: bool,
                 skip_ssim: bool, skip_backward: bool, use_dssim: bool, divide_by_two_in_dssim: bool,
                 grad_scale: torch.Tensor | None = None):
    """``_ssim_fwd_bwd!`` (src/core.jl:933-1107).  Returns ``(ssims, dL_dimgs1)``.

    Arguments that are ``None`` are allocated (outputs) or not needed (the
    intermediate buffer: the fused kernel keeps the partial gradients on chip).
    An allocated ``ssims`` for an input without a batch axis comes back as a
    Python float (src/conversions.jl:98-106).

    ``grad_scale`` (no counterpart in the reference driver) is an optional
    device vector with one factor per image: the gradient of image i comes out
    multiplied by it, which is the rrule's ``dL_dimgs1 .*= reshape(dL_dssims, 1,
    1, 1, :)`` (ext/FastCUDASSIMChainRulesCoreExt.jl:28-36) done inside the
    kernel (``fssim_fwd_bwd_scaled``)."""
    # Shape rules first, as in the reference (src/core.jl:942-984); the device
    # check comes after them, where the reference would fail on a CPU array.
    cimgs1 = canonicalize_image(imgs1)
    cimgs2 = canonicalize_image(imgs2)
    if tuple(cimgs1.shape) != tuple(cimgs2.shape):
        raise nat.DimensionMismatch(
            "The two image batches should have the same dimensions! "
            f"Received (canonical) sizes {tuple(cimgs1.shape)} and {tuple(cimgs2.shape)}.")
    c, h, w, b = (int(s) for s in cimgs1.shape)
    T = promote_dtype(cimgs1.dtype, cimgs2.dtype)
    device = cimgs1.device
    flags = 0
    allocated_ssims = False
    if not skip_ssim:
        if ssims is None:
            ssims = torch.empty(b, dtype=T, device=device)
            allocated_ssims = True
            flags |= nat.SHOULD_ZERO
        else:
            if tuple(ssims.shape) != (b,):
                raise nat.DimensionMismatch(
                    f"Expected the (d)ssims to be a CuVector of length the batch size {b}! "
                    f"Received size {tuple(ssims.shape)}.")
            if should_zero:
                flags |= nat.SHOULD_ZERO
    else:
        flags |= nat.SKIP_SSIM
    if not skip_backward and N_dssims_dQMP is not None:
        gb = canonicalize_gradient_buffer(N_dssims_dQMP)
        if tuple(gb.shape) != (h, 3, c, w, b):
            raise nat.DimensionMismatch(
                f"Given images in canonical size {(c, h, w, b)}, expected the intermediate gradients buffer "
                f"N_dssims_dQMP to have size {(h, 3, c, w, b)}, but received {tuple(gb.shape)}!")
    allocated_grad = False
    if skip_backward:
        flags |= nat.SKIP_BACKWARD
        dl_c = None
    else:
        if dL_dimgs1 is None:
            dl_c = jl_empty((c, h, w, b), T, device)
            allocated_grad = True
        else:
            dl_c = canonicalize_image(dL_dimgs1)
            if tuple(dl_c.shape) != tuple(cimgs1.shape):
                raise nat.DimensionMismatch(
                    "Expected the output gradient dL_dimgs1 to have the same canonical size "
                    f"{tuple(cimgs1.shape)} as the first input image batch! Instead received (canonical) "
                    f"size {tuple(dl_c.shape)}.")
    if use_dssim:
        flags |= nat.USE_DSSIM
        if divide_by_two_in_dssim:
            flags |= nat.DIVIDE_BY_TWO
    if dl_c is not None:
        # The gradient may be asked for in an input's own buffer (the reference's separate
        # backward launch allows it); the fused kernel does not, so that input is copied.
        if _overlap(dl_c, cimgs1):
            cimgs1 = _jl_copy(cimgs1)
        if _overlap(dl_c, cimgs2):
            cimgs2 = _jl_copy(cimgs2)
    if grad_scale is not None and not skip_backward:
        if tuple(grad_scale.shape) not in ((b,), ()) or (grad_scale.ndim == 0 and b != 1):
            raise nat.DimensionMismatch(
                f"Expected the gradient scale to have one entry per image ({b}); "
                f"received size {tuple(grad_scale.shape)}.")
        grad_scale = grad_scale.reshape(b).contiguous()
    else:
        grad_scale = None
    for name, t in (("imgs1", imgs1), ("imgs2", imgs2), ("ssims", None if skip_ssim else ssims),
                    ("dL_dimgs1", dl_c), ("grad_scale", grad_scale)):
        if t is not None:
            _require_device_array(name, t)
            if t.device != device:
                raise ValueError(f"{name} is on {t.device}, expected {device}")

    # the library launches on the current device: switch only when it differs
    switch = device.index != torch.cuda.current_device()
    prev = torch.cuda.current_device() if switch else None
    if switch:
        torch.cuda.set_device(device)
    try:
        stream = _current_stream_handle(device.index)
        nbytes = _workspace_size(c, h, w, b, flags, device.index)
        ws = _workspace(device, stream, nbytes)
        out_args = (ssims.data_ptr() if not skip_ssim else 0, dtype_code(ssims) if not skip_ssim else nat.FLOAT32,
                    b if skip_ssim else int(ssims.shape[0]),
                    dl_c.data_ptr() if dl_c is not None else 0,
                    dtype_code(dl_c) if dl_c is not None else nat.FLOAT32,
                    cimgs1.data_ptr(), dtype_code(cimgs1), cimgs2.data_ptr(), dtype_code(cimgs2))
        ws_args = (ws.data_ptr() if ws is not None else 0, ws.numel() if ws is not None else 0, stream)
        if grad_scale is None:
            nat.fwd_bwd(*out_args, 0, c, h, w, b, flags, *ws_args)
        else:
            nat.fwd_bwd_scaled(*out_args, c, h, w, b, flags, grad_scale.data_ptr(), dtype_code(grad_scale),
                               *ws_args)
    finally:
        if switch:
            torch.cuda.set_device(prev)

    if not skip_ssim and allocated_ssims and should_unpack(ssims, imgs1):
        ssims = ssims.item()           # the reference's blocking scalar read
    if allocated_grad:
        dL_dimgs1 = decanonicalize_gradient_image(dl_c, imgs1)
    return (None if skip_ssim else ssims), dL_dimgs1

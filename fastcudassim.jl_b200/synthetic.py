"""Seeded synthetic image pairs with the shapes and value distributions of the
benchmark workloads (the reference's own benchmark images are not available).

Two generators:
  * ``host_uniform`` / ``host_normal``: counter-based (splitmix64) and fully
    reproducible on any machine - used for small parity cases, so the CPU oracle
    and the GPU see identical bytes;
  * ``device_pair``: torch's CUDA generator with a fixed seed - used for the
    multi-gigabyte benchmark batches, which are checked through properties,
    not element by element.
"""
from __future__ import annotations

import numpy as np
import torch

from .conversions import jl_empty

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _splitmix(seed: int, n: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + (np.arange(1, n + 1, dtype=np.uint64) * _GOLDEN)
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def host_uniform(seed: int, shape) -> np.ndarray:
    """Float32 values in [0, 1) (24 random bits each), Fortran order, Julia shape."""
    n = int(np.prod(shape))
    u = (_splitmix(seed, n) >> np.uint64(40)).astype(np.float32) * np.float32(2.0 ** -24)
    return np.asfortranarray(u.reshape(tuple(shape), order="F"))


def host_normal(seed: int, shape) -> np.ndarray:
    """Standard normal values (Box-Muller in float64), Fortran order, Julia shape."""
    n = int(np.prod(shape))
    z = _splitmix(seed ^ 0x5DEECE66D, n)
    u1 = ((z >> np.uint64(11)).astype(np.float64) + 1.0) * 2.0 ** -53
    u2 = (_splitmix(seed ^ 0x2545F4914F6CDD1D, n) >> np.uint64(11)).astype(np.float64) * 2.0 ** -53
    g = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return np.asfortranarray(g.reshape(tuple(shape), order="F"))


def host_pair(seed: int, shape, noise: float | None, dtype=np.float32):
    """x ~ U[0,1); y = clamp(x + N(0, noise^2), 0, 1), or an independent U[0,1)
    when ``noise`` is None.  ``dtype`` uint8 returns N0f8 raw bytes of the same
    distributions (round(255 v)); float16 rounds the Float32 values."""
    x = host_uniform(seed, shape)
    if noise is None:
        y = host_uniform(seed + 1, shape)
    else:
        y = np.clip(x + np.float32(noise) * host_normal(seed + 2, shape).astype(np.float32), 0, 1)
        y = np.asfortranarray(y.astype(np.float32))
    if dtype == np.uint8:
        return (np.asfortranarray(np.rint(x * 255).astype(np.uint8)),
                np.asfortranarray(np.rint(y * 255).astype(np.uint8)))
    return np.asfortranarray(x.astype(dtype)), np.asfortranarray(y.astype(dtype))


def device_pair(shape, noise: float | None, dtype=torch.float32, seed: int = 1234, device="cuda"):
    """Julia-layout pair generated on the device (same distributions as host_pair)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = jl_empty(shape, torch.float32, device)
    y = jl_empty(shape, torch.float32, device)
    x.uniform_(0.0, 1.0, generator=g)
    if noise is None:
        y.uniform_(0.0, 1.0, generator=g)
    else:
        y.normal_(0.0, float(noise), generator=g).add_(x).clamp_(0.0, 1.0)
    if dtype == torch.uint8:
        return x.mul_(255).round_().to(torch.uint8), y.mul_(255).round_().to(torch.uint8)
    if dtype != torch.float32:
        return x.to(dtype), y.to(dtype)
    return x, y

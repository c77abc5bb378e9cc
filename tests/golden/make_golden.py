"""Generates the golden fixtures under tests/golden/ (run: python tests/golden/make_golden.py).

FastCUDASSIM.jl cannot run here (no Julia), so the fixtures come from two
sources that do not share code with the C oracle:

  known_answers.json  the closed forms of the reference's own tests:
                      test/single_pixel.jl:7-27 (SSIM and its gradient for a 1x1
                      image with zero padding), test/sanity_checks.jl:2-16
                      (C1/(1+C1), 1, 0.5) - evaluated here in float64 and in
                      float32 arithmetic from the Float32 kernel weights;
  scipy_cases.npz     an independent float64 restatement of the SSIM map and
                      gradient with scipy.ndimage.correlate1d (zero padding), on
                      the reference's ramp fixtures (test/forwarding.jl:4-11)
                      and on small seeded random cases, including odd sizes.

Weights: src/core.jl:40-46 (Float32 exp(-0.5 (i/1.5)^2) normalised by the
Float32 sum); constants: src/core.jl:49-50.
"""
from __future__ import annotations

import json
import os

import numpy as np
from scipy.ndimage import correlate1d

HERE = os.path.dirname(os.path.abspath(__file__))


def weights_f32() -> np.ndarray:
    i = np.arange(-5, 6, dtype=np.int32)
    r = i.astype(np.float32) / np.float32(1.5)
    raw = np.exp((np.float32(-0.5) * (r * r)).astype(np.float64)).astype(np.float32)
    s = np.float32(0)
    for v in raw:
        s = np.float32(s + v)
    return (raw / s).astype(np.float32)


C1 = np.float32(0.01) * np.float32(0.01)
C2 = np.float32(0.03) * np.float32(0.03)


def single_pixel(a, b, K, dt):
    """test/single_pixel.jl:7-27 in arithmetic of type dt."""
    a, b = dt(a), dt(b)
    W = dt(K[5]) * dt(K[5])
    c1, c2 = dt(C1), dt(C2)
    x = dt(2) * a * b * W * W + c1
    y = dt(2) * a * b * (W - W * W) + c2
    z = (a * a + b * b) * W * W + c1
    t = (a * a + b * b) * (W - W * W) + c2
    s = x * y / (z * t)
    dx = dt(2) * b * W * W
    dy = dt(2) * b * (W - W * W)
    dz = dt(2) * a * W * W
    dtt = dt(2) * a * (W - W * W)
    ds = ((dx * y + x * dy) * z * t - x * y * (dz * t + z * dtt)) / ((z * t) * (z * t))
    return float(s), float(ds)


def ssim_f64(x, y, flags=0):
    """Independent float64 SSIM / gradient on canonical (C,H,W,N) arrays."""
    K = weights_f32().astype(np.float64)
    c1, c2 = float(C1), float(C2)
    C, H, W, N = x.shape
    conv = lambda a: correlate1d(correlate1d(a, K, axis=0, mode="constant"), K, axis=1, mode="constant")
    vals = np.zeros(N)
    grad = np.zeros(x.shape)
    use_dssim, div2 = bool(flags & 4), bool(flags & 8)
    for n in range(N):
        tot = 0.0
        for c in range(C):
            a = x[c, :, :, n].astype(np.float64)
            b = y[c, :, :, n].astype(np.float64)
            m, mr = conv(a), conv(b)
            q, qr, p = conv(a * a), conv(b * b), conv(a * b)
            X = 2 * m * mr + c1
            Y = 2 * (p - m * mr) + c2
            Z = m * m + mr * mr + c1
            T = (q - m * m) + (qr - mr * mr) + c2
            s = X * Y / (Z * T)
            tot += s.sum()
            dQ = -s / T
            dM = 2 / (Z * T) * ((Y - X) * mr + s * (Z - T) * m)
            dP = 2 * X / (Z * T)
            grad[c, :, :, n] = 2 * a * conv(dQ) + conv(dM) + b * conv(dP)
        vals[n] = tot / (C * H * W)
    grad /= C * H * W
    if use_dssim:
        vals = (1 - vals) / 2 if div2 else 1 - vals
        grad *= -0.5 if div2 else -1.0
    return vals, grad


def splitmix_uniform(seed, shape):
    n = int(np.prod(shape))
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + np.arange(1, n + 1, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    u = (z >> np.uint64(40)).astype(np.float32) * np.float32(2.0 ** -24)
    return np.asfortranarray(u.reshape(shape, order="F"))


def ramps(c, h, w, b):
    """test/forwarding.jl:4-11: imgs1 constant along rows, imgs2 along columns."""
    x = np.empty((c, h, w, b), np.float32, order="F")
    y = np.empty((c, h, w, b), np.float32, order="F")
    x[...] = np.linspace(0, 1, h, dtype=np.float64).astype(np.float32)[None, :, None, None]
    y[...] = np.linspace(0, 1, w, dtype=np.float64).astype(np.float32)[None, None, :, None]
    return x, y


def main():
    K = weights_f32()
    pts = [(0.0, 0.1), (0.2, 0.5), (float(np.float32(1 / np.pi)), float(np.float32(1 / np.e)))]
    ka = {
        "weights_f32": [float(v) for v in K],
        "C1": float(C1), "C2": float(C2),
        "single_pixel": [
            {"a": a, "b": b,
             "f64": single_pixel(a, b, K, np.float64),
             "f32": single_pixel(a, b, K, np.float32)} for a, b in pts],
        "sanity": {"ssim_00": 1.0, "ssim_11": 1.0, "ssim_01": float(C1 / (1 + C1)),
                   "dssim_01": 1.0, "dssim_01_div2": 0.5, "size": [200, 300]},
    }
    with open(os.path.join(HERE, "known_answers.json"), "w") as f:
        json.dump(ka, f, indent=1)

    cases = {}
    x, y = ramps(3, 64, 96, 1)
    cases["ramps_3x64x96"] = (x, y, 0)
    x, y = ramps(1, 37, 5, 1)
    cases["ramps_1x37x5"] = (x, y, 0)
    for seed, (name, shape, flags) in enumerate([
            ("rand_1x37x5x1", (1, 37, 5, 1), 0), ("rand_3x23x17x2", (3, 23, 17, 2), 4),
            ("rand_2x64x40x1", (2, 64, 40, 1), 4 | 8), ("rand_1x1x1x3", (1, 1, 1, 3), 0),
            ("rand_4x70x9x1", (4, 70, 9, 1), 0)], start=101):
        cases[name] = (splitmix_uniform(seed, shape), splitmix_uniform(seed + 1, shape), flags)
    out = {}
    for name, (x, y, flags) in cases.items():
        v, g = ssim_f64(x, y, flags)
        out[name + "/x"] = x
        out[name + "/y"] = y
        out[name + "/flags"] = np.array(flags)
        out[name + "/vals"] = v
        out[name + "/grad"] = g.astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "scipy_cases.npz"), **out)


if __name__ == "__main__":
    main()

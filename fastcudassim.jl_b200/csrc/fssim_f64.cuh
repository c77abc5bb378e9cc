// Float64 inputs: the double-precision tile kernel (f64_kernel).
#pragma once

#include "fssim_common.cuh"

namespace fssim {

// ---------------------------------------------------------------------------
// Float64 path: inputs of any supported dtype of which at least one is Float64
// are computed in double precision, as the reference does when either input is
// Float64 (promote_type(T1, T2, Float32), src/core.jl:159 and :953-954).
//
// A CTA computes one TO x TO output tile of one channel of one image (two CTAs
// per SM).  Five phases, each split evenly over the CTA's threads, with a
// barrier between them:
//   1  load the (TO + 4R)^2 input tile (zero outside the image)
//   2  h-direction pass of the four moment images x, y, x^2+y^2, xy on the
//      TO + 2R partial rows (an item: 6 rows of one moment pair in one column)
//   3  w-direction pass, SSIM map and partials on the (TO + 2R)^2 partial tile
//      (an item: 7 columns of one row); the partials overwrite the input tile
//   4  h-direction pass of the three partials on the TO output rows (16 rows of
//      one partial in one column); overwrites the moments
//   5  w-direction pass and the combine on the own pixels (4 columns of one row;
//      x and y are read again from global memory)
// As in the Float32 kernels, E[x^2] and E[y^2] are convolved together.  The
// map's 1/(zt) is a hardware reciprocal estimate refined by two Newton-Raphson
// steps (r <- r + r (1 - zt r)), which give a double-precision result; 1/t and
// 1/z come from it by multiplication, as in the Float32 kernels.
// Shared memory rows have odd strides, so both access directions of every
// buffer are free of bank conflicts.
// ---------------------------------------------------------------------------
struct D64Geo {
    static constexpr int TO = 32;              // output tile edge
    static constexpr int TP = TO + 2 * RAD;    // partial-derivative tile edge (42)
    static constexpr int TI = TO + 4 * RAD;    // input tile edge (52)
    static constexpr int NT = 256;
    static constexpr int XS = TI + 1;          // row stride of the input and moment tiles
    static constexpr int QS = TP + 1;          // row stride of the partial tiles
    static constexpr int V1 = 6;               // phase 2: rows per item
    static constexpr int V2 = 7;               // phase 3: columns per item
    static constexpr int V3 = 16;              // phase 4: rows per item
    static constexpr int V4 = 4;               // phase 5: columns per item
    static constexpr int N2 = 2 * (TP / V1) * TI;      // phase 2 items (728)
    static constexpr int N3 = (TP / V2) * TP;          // phase 3 items (252)
    static constexpr int N4 = 3 * (TO / V3) * TP;      // phase 4 items (252)
    static constexpr int N5 = (TO / V4) * TO;          // phase 5 items (256)
    static constexpr int in_bytes = 2 * TI * XS * 8;   // x, y; then the partials
    static constexpr int h1_bytes = 4 * TP * XS * 8;   // moments; then the partials' h-pass
    static constexpr int red_bytes = (NT / 32 + 2) * 8;
    static constexpr int total = in_bytes + h1_bytes + red_bytes;
    static_assert(TP % V1 == 0 && TP % V2 == 0 && TO % V3 == 0 && TO % V4 == 0, "whole items");
    static_assert(N3 <= NT && N4 <= NT && N5 <= NT, "phases 3-5: one item per thread");
    static_assert(3 * TP * QS * 8 <= in_bytes && 3 * TO * QS * 8 <= h1_bytes, "the overlays fit");
};

__device__ __forceinline__ double ld_f64(const void* base, int dt, int64_t idx)
{
    if (dt == DT_F64) return __ldg(reinterpret_cast<const double*>(base) + idx);
    return static_cast<double>(cvt_raw(ld_raw(base, dt, idx), dt, nullptr));
}

// 1/v for v > 0 of normal magnitude: the hardware estimate plus two Newton-Raphson steps.
__device__ __forceinline__ double rcp_nr(double v)
{
    double r;
    asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(r) : "d"(v));
    r = fma(r, fma(-v, r, 1.0), r);
    return fma(r, fma(-v, r, 1.0), r);
}

template <bool FUSED, bool WANT_SSIM>
__global__ void __launch_bounds__(D64Geo::NT, 2) f64_kernel(const Params p)
{
    using G = D64Geo;
    constexpr int TO = G::TO, TP = G::TP, TI = G::TI, NT = G::NT, XS = G::XS, QS = G::QS;
    constexpr int V1 = G::V1, V2 = G::V2, V3 = G::V3, V4 = G::V4;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    double* xs = reinterpret_cast<double*>(smem_raw);   // [TI][XS]: row (h), column (w)
    double* ys = xs + TI * XS;
    double* h1 = ys + TI * XS;                          // [4][TP][XS]
    double* qm = xs;                                    // [3][TP][QS], over x and y after phase 2
    double* b1 = h1;                                    // [3][TO][QS], over the moments after phase 3
    double* red = reinterpret_cast<double*>(smem_raw + G::in_bytes + G::h1_bytes);

    const int tid = threadIdx.x;
    // block -> (channel, tile column, tile row, image); 32-bit divisions (grid < 2^31)
    const uint32_t b0 = blockIdx.x, b1q = b0 / static_cast<uint32_t>(p.C);
    const uint32_t b2q = b1q / static_cast<uint32_t>(p.nseg), b3q = b2q / static_cast<uint32_t>(p.nb);
    const int c = static_cast<int>(b0 - b1q * static_cast<uint32_t>(p.C));
    const int tw = static_cast<int>(b1q - b2q * static_cast<uint32_t>(p.nseg));   // tile column
    const int th = static_cast<int>(b2q - b3q * static_cast<uint32_t>(p.nb));     // tile row
    const int n = static_cast<int>(b3q);
    const int C = p.C, H = p.H, W = p.W;
    const int64_t CH = static_cast<int64_t>(C) * H;
    const int64_t ibase = static_cast<int64_t>(n) * p.img_elems + c;
    const int h0 = th * TO, w0 = tw * TO;
    double k[RAD + 1];   // the Float32 taps, exactly
#pragma unroll
    for (int i = 0; i <= RAD; ++i) k[i] = static_cast<double>(p.kh[i]);
#define FSSIM_KD(tap) k[(tap) <= RAD ? (tap) : 2 * RAD - (tap)]
    const double C1 = p.C1, C2 = p.C2;

    // ---- phase 1: input tile, rows h0-2R .., columns w0-2R ..; zero outside the image.
    // Every load of a thread is issued before the first store, so their latencies overlap.
    const bool f64in = p.xdt == DT_F64 && p.ydt == DT_F64;
    {
        constexpr int NL = (TI * TI + NT - 1) / NT;
        double xv[NL], yv[NL];
#pragma unroll
        for (int u = 0; u < NL; ++u) {
            const int e = tid + u * NT;
            const int r = e % TI, q = e / TI;
            const int hr = h0 - 2 * RAD + r, wc = w0 - 2 * RAD + q;
            const int64_t g = ibase + static_cast<int64_t>(C) * hr + CH * wc;
            const bool ok = e < TI * TI && hr >= 0 && hr < H && wc >= 0 && wc < W &&
                            FSSIM_IN_BOUNDS(g, p.total_elems, SITE_F64_LOAD);
            if (f64in) {
                xv[u] = ok ? __ldg(reinterpret_cast<const double*>(p.x) + g) : 0.0;
                yv[u] = ok ? __ldg(reinterpret_cast<const double*>(p.y) + g) : 0.0;
            } else {
                xv[u] = ok ? ld_f64(p.x, p.xdt, g) : 0.0;
                yv[u] = ok ? ld_f64(p.y, p.ydt, g) : 0.0;
            }
        }
#pragma unroll
        for (int u = 0; u < NL; ++u) {
            const int e = tid + u * NT;
            if (e < TI * TI) {
                const int r = e % TI, q = e / TI;
                xs[r * XS + q] = xv[u];
                ys[r * XS + q] = yv[u];
            }
        }
    }
    __syncthreads();
    // ---- phase 2: h-direction pass; item = (moment pair, row group, column)
    for (int it = tid; it < G::N2; it += NT) {
        const int q = it % TI;
        const int rg = (it / TI) % (TP / V1), pair = it / (TI * (TP / V1));
        double a0[V1], a1[V1];
#pragma unroll
        for (int o = 0; o < V1; ++o) a0[o] = a1[o] = 0.0;
        const double* xc = xs + rg * V1 * XS + q;
        const double* yc = ys + rg * V1 * XS + q;
        if (pair == 0) {   // x, y
#pragma unroll
            for (int i = 0; i < V1 + 2 * RAD; ++i) {
                const double u = xc[i * XS], v = yc[i * XS];
#pragma unroll
                for (int o = 0; o < V1; ++o) {
                    const int tap = i - o;
                    if (tap >= 0 && tap < TAPS) {
                        a0[o] = fma(FSSIM_KD(tap), u, a0[o]);
                        a1[o] = fma(FSSIM_KD(tap), v, a1[o]);
                    }
                }
            }
        } else {           // x^2 + y^2, xy
#pragma unroll
            for (int i = 0; i < V1 + 2 * RAD; ++i) {
                const double xv = xc[i * XS], yv = yc[i * XS];
                const double u = fma(xv, xv, yv * yv), v = xv * yv;
#pragma unroll
                for (int o = 0; o < V1; ++o) {
                    const int tap = i - o;
                    if (tap >= 0 && tap < TAPS) {
                        a0[o] = fma(FSSIM_KD(tap), u, a0[o]);
                        a1[o] = fma(FSSIM_KD(tap), v, a1[o]);
                    }
                }
            }
        }
        double* d0 = h1 + ((2 * pair) * TP + rg * V1) * XS + q;
        double* d1 = d0 + TP * XS;
#pragma unroll
        for (int o = 0; o < V1; ++o) {
            d0[o * XS] = a0[o];
            d1[o * XS] = a1[o];
        }
    }
    __syncthreads();
    // ---- phase 3: w-direction pass, SSIM map (own pixels), partials on the TP x TP tile
    double tsum = 0.0;
    if (tid < G::N3) {
        const int r = tid % TP, cg = tid / TP;   // partial row r <-> image row h0-R+r
        double m[4][V2];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int o = 0; o < V2; ++o) m[j][o] = 0.0;
#pragma unroll
        for (int i = 0; i < V2 + 2 * RAD; ++i) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const double v = h1[(j * TP + r) * XS + cg * V2 + i];
#pragma unroll
                for (int o = 0; o < V2; ++o) {
                    const int tap = i - o;
                    if (tap >= 0 && tap < TAPS) m[j][o] = fma(FSSIM_KD(tap), v, m[j][o]);
                }
            }
        }
        const double gscale = (p.use_dssim ? -1.0 : 1.0) * ((p.use_dssim && p.div2) ? 0.5 : 1.0) / p.npx *
                              (p.img_scale ? ld_out(p.img_scale, p.isdt, n) : 1.0);
        const int hr = h0 - RAD + r;
        const bool row_in = hr >= 0 && hr < H;
#pragma unroll
        for (int o = 0; o < V2; ++o) {
            const int q = cg * V2 + o;              // partial column q <-> image column w0-R+q
            const int wc = w0 - RAD + q;
            const double mx = m[0][o], my = m[1][o], qs = m[2][o], pxy = m[3][o];
            const double mxy = mx * my;
            const double sumsq = fma(mx, mx, my * my);
            const double z = sumsq + C1;                   // mx^2 + my^2 + C1
            const double t = (qs - sumsq) + C2;            // vx + vy + C2
            const double ax = fma(2.0, mxy, C1);           // 2 mx my + C1
            const double by = fma(2.0, pxy - mxy, C2);     // 2 cov + C2
            const double inv = rcp_nr(z * t);
            const double s = (ax * by) * inv;
            const bool in_img = row_in && wc >= 0 && wc < W;
            if (WANT_SSIM && in_img && r >= RAD && r < RAD + TO && q >= RAD && q < RAD + TO) tsum += s;
            if (FUSED) {
                // dS/dQ = -s/t (stored doubled), dS/dM, dS/dP (src/core.jl:384-388), times the scale
                const double inv2 = in_img ? 2.0 * gscale * inv : 0.0;
                qm[(0 * TP + r) * QS + q] = -(s * z) * inv2;
                qm[(1 * TP + r) * QS + q] = inv2 * fma(by - ax, my, (s * (z - t)) * mx);
                qm[(2 * TP + r) * QS + q] = ax * inv2;
            }
        }
    }
    if (FUSED) {
        __syncthreads();
        // ---- phase 4: h-direction pass of the partials; item = (partial, row group, column)
        if (tid < G::N4) {
            const int q = tid % TP;
            const int rg = (tid / TP) % (TO / V3), j = tid / (TP * (TO / V3));
            double a[V3];
#pragma unroll
            for (int o = 0; o < V3; ++o) a[o] = 0.0;
            const double* src = qm + (j * TP + rg * V3) * QS + q;
#pragma unroll
            for (int i = 0; i < V3 + 2 * RAD; ++i) {
                const double v = src[i * QS];
#pragma unroll
                for (int o = 0; o < V3; ++o) {
                    const int tap = i - o;
                    if (tap >= 0 && tap < TAPS) a[o] = fma(FSSIM_KD(tap), v, a[o]);
                }
            }
            double* dst = b1 + (j * TO + rg * V3) * QS + q;
#pragma unroll
            for (int o = 0; o < V3; ++o) dst[o * QS] = a[o];
        }
        __syncthreads();
        // ---- phase 5: w-direction pass and the combine on the own pixels
        {
            const int r = tid % TO, cg = tid / TO;
            const int hg = h0 + r;
            double xo[V4], yo[V4];   // x and y of the own pixels, loaded before the arithmetic
#pragma unroll
            for (int o = 0; o < V4; ++o) {
                const int wg = w0 + cg * V4 + o;
                const int64_t g = ibase + static_cast<int64_t>(C) * hg + CH * wg;
                const bool ok = hg < H && wg < W && FSSIM_IN_BOUNDS(g, p.total_elems, SITE_F64_GRAD);
                if (f64in) {
                    xo[o] = ok ? __ldg(reinterpret_cast<const double*>(p.x) + g) : 0.0;
                    yo[o] = ok ? __ldg(reinterpret_cast<const double*>(p.y) + g) : 0.0;
                } else {
                    xo[o] = ok ? ld_f64(p.x, p.xdt, g) : 0.0;
                    yo[o] = ok ? ld_f64(p.y, p.ydt, g) : 0.0;
                }
            }
            double a[3][V4];
#pragma unroll
            for (int j = 0; j < 3; ++j)
#pragma unroll
                for (int o = 0; o < V4; ++o) a[j][o] = 0.0;
#pragma unroll
            for (int i = 0; i < V4 + 2 * RAD; ++i) {
#pragma unroll
                for (int j = 0; j < 3; ++j) {
                    const double v = b1[(j * TO + r) * QS + cg * V4 + i];
#pragma unroll
                    for (int o = 0; o < V4; ++o) {
                        const int tap = i - o;
                        if (tap >= 0 && tap < TAPS) a[j][o] = fma(FSSIM_KD(tap), v, a[j][o]);
                    }
                }
            }
#pragma unroll
            for (int o = 0; o < V4; ++o) {
                const int wg = w0 + cg * V4 + o;
                if (hg < H && wg < W) {
                    const int64_t g = ibase + static_cast<int64_t>(C) * hg + CH * wg;
                    if (FSSIM_IN_BOUNDS(g, p.total_elems, SITE_F64_GRAD)) {
                        // src/core.jl:773-782: 2 x K(dQ) + K(dM) + y K(dP), 2 dQ stored doubled
                        const double gv = fma(xo[o], a[0][o], fma(yo[o], a[2][o], a[1][o]));
                        if (p.gdt == DT_F64) reinterpret_cast<double*>(p.grad)[g] = gv;
                        else st_grad(p.grad, p.gdt, g, static_cast<float>(gv));
                    }
                }
            }
        }
    }
#undef FSSIM_KD
    if (WANT_SSIM) {
        const int local_cta = (th * p.nseg + tw) * p.C + c;
        finish_image<NT>(p, n, local_cta, tsum, red);
    }
}

}  // namespace fssim

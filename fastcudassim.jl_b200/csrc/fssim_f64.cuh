// Float64 inputs: the double-precision tile kernel (f64_kernel).
#pragma once

#include "fssim_common.cuh"

namespace fssim {

// ---------------------------------------------------------------------------
// Float64 path: inputs of any supported dtype of which at least one is Float64
// are computed in double precision, as the reference does when either input is
// Float64 (promote_type(T1, T2, Float32), src/core.jl:159 and :953-954).  The
// reference's own five moments are convolved (E[x^2] and E[y^2] separately).
//
// A CTA computes one 16 x 16 output tile of one channel of one image from a
// (16 + 4R)^2 input tile held in shared memory: moments on the tile plus a
// 5-pixel halo (the backward correlation needs partials there), the SSIM map,
// the partials, then the two backward passes.  Plain, not streamed: this path
// exists for numerical parity, not speed.
// ---------------------------------------------------------------------------
struct D64Geo {
    static constexpr int TO = 16;              // output tile edge
    static constexpr int TP = TO + 2 * RAD;    // partial-derivative tile edge (26)
    static constexpr int TI = TO + 4 * RAD;    // input tile edge (36)
    static constexpr int NT = 256;
    static constexpr int in_bytes = 2 * TI * TI * 8;        // x, y
    static constexpr int h1_bytes = 5 * TP * TI * 8;        // h-pass moments: TP rows x TI cols
    static constexpr int qmp_bytes = 3 * TP * TP * 8;       // partials
    static constexpr int b1_bytes = 3 * TO * TP * 8;        // h-pass of the partials: TO rows x TP cols
    static constexpr int red_bytes = (NT / 32 + 2) * 8;
    static constexpr int total = in_bytes + h1_bytes + qmp_bytes + b1_bytes + red_bytes;
};

__device__ __forceinline__ double ld_f64(const void* base, int dt, int64_t idx)
{
    if (dt == DT_F64) return __ldg(reinterpret_cast<const double*>(base) + idx);
    return static_cast<double>(cvt_raw(ld_raw(base, dt, idx), dt, nullptr));
}

template <bool FUSED, bool WANT_SSIM>
__global__ void __launch_bounds__(D64Geo::NT) f64_kernel(const Params p)
{
    using G = D64Geo;
    constexpr int TO = G::TO, TP = G::TP, TI = G::TI, NT = G::NT;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    double* xs = reinterpret_cast<double*>(smem_raw);          // [TI][TI] (row h, col w)
    double* ys = xs + TI * TI;
    double* h1 = ys + TI * TI;                                  // [5][TP][TI]
    double* qm = h1 + 5 * TP * TI;                              // [3][TP][TP]
    double* b1 = qm + 3 * TP * TP;                              // [3][TO][TP]
    double* red = reinterpret_cast<double*>(smem_raw + G::total - G::red_bytes);

    const int tid = threadIdx.x;
    int64_t blk = blockIdx.x;
    const int c = static_cast<int>(blk % p.C);
    blk /= p.C;
    const int tw = static_cast<int>(blk % p.nseg);   // tile column
    blk /= p.nseg;
    const int th = static_cast<int>(blk % p.nb);     // tile row
    const int n = static_cast<int>(blk / p.nb);
    const int C = p.C, H = p.H, W = p.W;
    const int64_t CH = static_cast<int64_t>(C) * H;
    const int64_t ibase = static_cast<int64_t>(n) * p.img_elems + c;
    const int h0 = th * TO, w0 = tw * TO;
    double k[TAPS];
#pragma unroll
    for (int i = 0; i < TAPS; ++i) k[i] = static_cast<double>(p.kh[i <= RAD ? i : 2 * RAD - i]);
    const double C1 = p.C1, C2 = p.C2;

    // input tile: rows h0-2R .. h0+TO+2R, cols w0-2R .. ; zero outside the image
    for (int e = tid; e < TI * TI; e += NT) {
        const int r = e % TI, q = e / TI;
        const int hr = h0 - 2 * RAD + r, wc = w0 - 2 * RAD + q;
        double xv = 0.0, yv = 0.0;
        if (hr >= 0 && hr < H && wc >= 0 && wc < W) {
            const int64_t g = ibase + static_cast<int64_t>(C) * hr + CH * wc;
            if (FSSIM_IN_BOUNDS(g, p.total_elems, SITE_F64_LOAD)) {
                xv = ld_f64(p.x, p.xdt, g);
                yv = ld_f64(p.y, p.ydt, g);
            }
        }
        xs[r * TI + q] = xv;
        ys[r * TI + q] = yv;
    }
    __syncthreads();
    // h-direction pass of the five moment images on the TP partial rows
    for (int e = tid; e < TP * TI; e += NT) {
        const int r = e / TI, q = e % TI;   // output row r <-> input row r + R
        double a1 = 0, a2 = 0, a3 = 0, a4 = 0, a5 = 0;
#pragma unroll
        for (int i = 0; i < TAPS; ++i) {
            const double xv = xs[(r + i) * TI + q], yv = ys[(r + i) * TI + q];
            const double xk = xv * k[i], yk = yv * k[i];
            a1 += xk; a2 += xv * xk; a3 += yk; a4 += yv * yk; a5 += xv * yk;
        }
        h1[(0 * TP + r) * TI + q] = a1;
        h1[(1 * TP + r) * TI + q] = a2;
        h1[(2 * TP + r) * TI + q] = a3;
        h1[(3 * TP + r) * TI + q] = a4;
        h1[(4 * TP + r) * TI + q] = a5;
    }
    __syncthreads();
    // w-direction pass, SSIM map (own pixels), partials on the TP x TP tile
    const double gscale = static_cast<double>(p.use_dssim ? -1.0 : 1.0) *
                          ((p.use_dssim && p.div2) ? 0.5 : 1.0) / p.npx *
                          (p.img_scale ? ld_out(p.img_scale, p.isdt, n) : 1.0);
    double tsum = 0.0;
    for (int e = tid; e < TP * TP; e += NT) {
        const int r = e % TP, q = e / TP;        // partial pixel (r, q) <-> image (h0-R+r, w0-R+q)
        double mom[5];
#pragma unroll
        for (int j = 0; j < 5; ++j) {
            double acc = h1[(j * TP + r) * TI + q + RAD] * k[RAD];
#pragma unroll
            for (int i = 0; i < RAD; ++i)
                acc += (h1[(j * TP + r) * TI + q + i] + h1[(j * TP + r) * TI + q + 2 * RAD - i]) * k[i];
            mom[j] = acc;
        }
        const double m = mom[0], qq = mom[1], mR = mom[2], qR = mom[3], pp = mom[4];
        const double x = 2 * m * mR + C1;
        const double y = 2 * (pp - m * mR) + C2;
        const double z = m * m + mR * mR + C1;
        const double t = (qq - m * m) + (qR - mR * mR) + C2;
        const double zt_inv = 1.0 / (z * t);
        const double s = x * y * zt_inv;
        const int hr = h0 - RAD + r, wc = w0 - RAD + q;
        const bool in_img = hr >= 0 && hr < H && wc >= 0 && wc < W;
        if (WANT_SSIM && in_img && r >= RAD && r < RAD + TO && q >= RAD && q < RAD + TO) tsum += s;
        if (FUSED) {
            const double sc = in_img ? gscale : 0.0;
            qm[(0 * TP + r) * TP + q] = sc * 2.0 * (-s / t);
            qm[(1 * TP + r) * TP + q] = sc * (2 * zt_inv * ((y - x) * mR + s * (z - t) * m));
            qm[(2 * TP + r) * TP + q] = sc * (2 * x * zt_inv);
        }
    }
    if (FUSED) {
        __syncthreads();
        // h-direction pass of the partials: TO output rows x TP columns
        for (int e = tid; e < TO * TP; e += NT) {
            const int r = e % TO, q = e / TO;
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                double acc = qm[(j * TP + r + RAD) * TP + q] * k[RAD];
#pragma unroll
                for (int i = 0; i < RAD; ++i)
                    acc += (qm[(j * TP + r + i) * TP + q] + qm[(j * TP + r + 2 * RAD - i) * TP + q]) * k[i];
                b1[(j * TO + r) * TP + q] = acc;
            }
        }
        __syncthreads();
        // w-direction pass and the combine on the own TO x TO pixels
        for (int e = tid; e < TO * TO; e += NT) {
            const int r = e % TO, q = e / TO;
            const int hg = h0 + r, wg = w0 + q;
            if (hg >= H || wg >= W) continue;
            double cv[3];
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                double acc = b1[(j * TO + r) * TP + q + RAD] * k[RAD];
#pragma unroll
                for (int i = 0; i < RAD; ++i)
                    acc += (b1[(j * TO + r) * TP + q + i] + b1[(j * TO + r) * TP + q + 2 * RAD - i]) * k[i];
                cv[j] = acc;
            }
            const double xv = xs[(r + 2 * RAD) * TI + q + 2 * RAD], yv = ys[(r + 2 * RAD) * TI + q + 2 * RAD];
            const double gv = xv * cv[0] + cv[1] + yv * cv[2];     // 2 dQ is stored doubled
            const int64_t g = ibase + static_cast<int64_t>(C) * hg + CH * wg;
            if (!FSSIM_IN_BOUNDS(g, p.total_elems, SITE_F64_GRAD)) continue;
            if (p.gdt == DT_F64) reinterpret_cast<double*>(p.grad)[g] = gv;
            else st_grad(p.grad, p.gdt, g, static_cast<float>(gv));
        }
    }
    if (WANT_SSIM) {
        const int local_cta = (th * p.nseg + tw) * p.C + c;
        finish_image<NT>(p, n, local_cta, tsum, red);
    }
}

}  // namespace fssim

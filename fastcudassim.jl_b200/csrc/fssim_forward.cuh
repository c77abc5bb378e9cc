// Forward-only kernels: the two-group pipeline (fwd_pipe_kernel), the tile kernel
// (tile_fwd_kernel) and the single-group streaming kernel with 64-bit offsets (band_kernel).
#pragma once

#include <cuda.h>   // CUtensorMap

#include "fssim_common.cuh"

namespace fssim {

// Geometry and shared-memory footprint of one CTA of the forward streaming
// kernel (host and device agree on it).
template <int NT>
struct Geo {
    static constexpr int S = 8;                            // columns per step
    static constexpr int R1 = NT;                          // moment rows = output rows of a band
    static constexpr int T = NT;
    static constexpr int R2 = R1 + 2 * RAD;                // input rows
    static constexpr int LAG = RAD;                        // input column offset of the stream
    static constexpr int SP = S + 1;                       // staging row stride (float2), odd
    static constexpr int FC = S + 1;                       // float4 row stride, odd: conflict-free
    static constexpr int NRUN1 = R1 / V;                   // F1 runs per column
    static constexpr int IT1 = S * NRUN1 / NT;             // F1 items per thread
    static constexpr int LROWS = (R2 + NT - 1) / NT;       // staging rows per thread
    static constexpr int stage_one = R2 * SP * 8;
    static constexpr int stage_bytes = 2 * stage_one;
    static constexpr int f1_bytes = R1 * FC * 16;
    static constexpr int red_bytes = (NT / 32 + 2) * 8;
    static constexpr int total = stage_bytes + f1_bytes + red_bytes;
    static_assert(R1 % V == 0 && NT % 32 == 0, "band geometry");
    static_assert((S * NRUN1) % NT == 0, "F1 items must divide evenly over the CTA");
    static_assert(stage_one % 16 == 0, "staging must keep 16-byte alignment");
};

// Forward-only streaming kernel for Float32 inputs (SSIM values, no gradient).
// Loads go straight to shared memory with cp.async, double-buffered two steps
// ahead; two barriers per step (after F1, after F2).  The launch bound keeps
// 16 warps per SM resident (at most 128 registers a thread, no spills).
template <int NT>
__global__ void __launch_bounds__(NT, 512 / NT) band_kernel(const Params p)
{
    using G = Geo<NT>;
    constexpr int S = G::S, T = G::T, R2 = G::R2, LAG = G::LAG;
    constexpr int SP = G::SP, FC = G::FC;

    extern __shared__ __align__(16) unsigned char smem_raw[];
    float2* stage = reinterpret_cast<float2*>(smem_raw);
    float4* f1buf = reinterpret_cast<float4*>(smem_raw + G::stage_bytes);
    double* red = reinterpret_cast<double*>(smem_raw + G::total - G::red_bytes);

    const int tid = threadIdx.x;
    const BandIndex bi = band_index(p);
    const int c = bi.c, seg = bi.seg, band = bi.band, n = bi.n;
    const int C = p.C, H = p.H, W = p.W;
    const int64_t CH = static_cast<int64_t>(C) * H;   // element stride of one column
    const int h0 = band * T;
    const int w0 = seg * p.L;
    const int wend = min(w0 + p.L, W);
    const int Lc = wend - w0;
    const int64_t ibase = static_cast<int64_t>(n) * p.img_elems + c;
    // Steps: the last owned output column must come out of the final step:
    // ns = ceil((Lc + 2*LAG - S) / S) + 1.
    const int ns = (Lc + 2 * LAG - 1) / S + 1;

    // Gaussian weights as (k, k) pairs for the packed FMAs.
    float2 KP[RAD + 1];
#pragma unroll
    for (int i = 0; i <= RAD; ++i) KP[i] = make_float2(p.kh[i], p.kh[i]);
#define FSSIM_K2(tap) KP[(tap) <= RAD ? (tap) : 2 * RAD - (tap)]

    // ---------------- loader: one step = S columns x R2 rows ----------------
    // thread `tid` owns staging rows tid, tid+NT, ... and walks the S columns of
    // the step; lanes cover consecutive rows.
    int64_t lrow_base[G::LROWS];
    bool lrow_ok[G::LROWS];
#pragma unroll
    for (int r = 0; r < G::LROWS; ++r) {
        const int i = tid + NT * r;
        const int hr = h0 - LAG + i;
        lrow_ok[r] = i < R2 && hr >= 0 && hr < H;
        lrow_base[r] = ibase + static_cast<int64_t>(C) * hr;
    }
    auto issue_async = [&](int k, float2* buf) {
        const int cb = w0 - LAG + k * S;   // image column of staging column 0
#pragma unroll
        for (int r = 0; r < G::LROWS; ++r) {
            const int i = tid + NT * r;
            if (i < R2) {
#pragma unroll
                for (int j = 0; j < S; ++j) {
                    const int wc = cb + j;
                    bool ok = lrow_ok[r] && k < ns && static_cast<unsigned>(wc) < static_cast<unsigned>(W);
                    ok = ok && FSSIM_IN_BOUNDS(lrow_base[r] + CH * wc, p.total_elems, SITE_BAND_LOAD);
                    const int64_t g = ok ? lrow_base[r] + CH * wc : 0;
                    float2* d = buf + i * SP + j;
                    cp_async4(&d->x, reinterpret_cast<const float*>(p.x) + g, ok);
                    cp_async4(&d->y, reinterpret_cast<const float*>(p.y) + g, ok);
                }
            }
        }
        cp_async_commit();
    };

    issue_async(0, stage);
    issue_async(1, stage + R2 * SP);
    cp_async_wait<1>();
    __syncthreads();

    // F2 role: row `tid` of the band
    const int hr2 = h0 + tid;                           // image row of the F2 row
    const bool row_owned = hr2 < H;

    float2 hA[HIST], hB[HIST];          // (mx, my), (E[x^2+y^2], E[xy]) history of F1 columns
#pragma unroll
    for (int m = 0; m < HIST; ++m) {
        hA[m] = make_float2(0.f, 0.f);
        hB[m] = make_float2(0.f, 0.f);
    }
    double tsum = 0.0;

#pragma unroll 1
    for (int k = 0; k < ns; ++k) {
        // ---------------- F1: h-direction pass of the 4 moment images ----------------
        {
            const float2* st = stage + (k & 1) * (R2 * SP);
#pragma unroll 1
            for (int it = 0; it < G::IT1; ++it) {
                const int item = tid + NT * it;
                const int j1 = item % S, q1 = item / S;
                float2 aA[V], aB[V];
#pragma unroll
                for (int o = 0; o < V; ++o) {
                    aA[o] = make_float2(0.f, 0.f);
                    aB[o] = make_float2(0.f, 0.f);
                }
#pragma unroll
                for (int i = 0; i < V + 2 * RAD; ++i) {
                    const float2 xy = st[(V * q1 + i) * SP + j1];
                    const float2 pr = __fmul2_rn(make_float2(xy.x, xy.x), xy);   // (x^2, xy)
                    const float2 sb = make_float2(fmaf(xy.y, xy.y, pr.x), pr.y); // (x^2+y^2, xy)
#pragma unroll
                    for (int o = 0; o < V; ++o) {
                        const int tap = i - o;
                        if (tap >= 0 && tap < TAPS) {
                            aA[o] = __ffma2_rn(xy, FSSIM_K2(tap), aA[o]);
                            aB[o] = __ffma2_rn(sb, FSSIM_K2(tap), aB[o]);
                        }
                    }
                }
#pragma unroll
                for (int o = 0; o < V; ++o)
                    f1buf[(V * q1 + o) * FC + j1] = make_float4(aA[o].x, aA[o].y, aB[o].x, aB[o].y);
            }
        }
        __syncthreads();

        // ---------------- F2: w-direction pass and the SSIM map ----------------
        {
            // the staging buffer F1 just read is free: refill it two steps ahead
            issue_async(k + 2, stage + (k & 1) * (R2 * SP));

            const int wcb = w0 - LAG + k * S - RAD;   // image column of output o = 0
            float2 nA[S], nB[S];
            float ssum = 0.f;
#pragma unroll
            for (int o = 0; o < S; ++o) {
                {   // column o of this step enters the window just before its first use
                    const float4 v = f1buf[tid * FC + o];
                    nA[o] = make_float2(v.x, v.y);
                    nB[o] = make_float2(v.z, v.w);
                }
                float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
#pragma unroll
                for (int tap = 0; tap < TAPS; ++tap) {
                    const int m = o + tap;
                    const float2 wa = (m < HIST) ? hA[m] : nA[m - HIST];
                    const float2 wb = (m < HIST) ? hB[m] : nB[m - HIST];
                    a = __ffma2_rn(wa, FSSIM_K2(tap), a);
                    b = __ffma2_rn(wb, FSSIM_K2(tap), b);
                }
                const float mx = a.x, my = a.y, qs = b.x, pxy = b.y;
                const float2 sq = __fmul2_rn(a, a);                  // (mx^2, my^2)
                const float mxy = mx * my;
                const float sumsq = sq.x + sq.y;
                const float z = sumsq + p.C1;                        // mx^2 + my^2 + C1
                const float t = (qs - sumsq) + p.C2;                 // vx + vy + C2
                const float2 ab = __ffma2_rn(make_float2(2.f, 2.f), make_float2(mxy, pxy - mxy),
                                             make_float2(p.C1, p.C2));   // (2 mx my + C1, 2 cov + C2)
                const float s = (ab.x * ab.y) * rcp_approx(z * t);
                const int wc = wcb + o;                              // image column of this pixel
                if (row_owned && static_cast<unsigned>(wc - w0) < static_cast<unsigned>(Lc)) ssum += s;
            }
            tsum += static_cast<double>(ssum);
#pragma unroll
            for (int m = 0; m < HIST; ++m) {
                const int src = m + S;
                hA[m] = (src < HIST) ? hA[src] : nA[src - HIST];
                hB[m] = (src < HIST) ? hB[src] : nB[src - HIST];
            }
            cp_async_wait<1>();   // step k+1 has landed (k+2 may still fly)
        }
        __syncthreads();
    }
#undef FSSIM_K2

    const int local_cta = (band * p.nseg + seg) * p.C + c;
    finish_image<NT>(p, n, local_cta, tsum, red);
}


// ---------------------------------------------------------------------------
// Two-group pipelined forward kernel (SSIM only): the forward half of
// pipe_kernel.  Group A loads step t+1 and runs F1(t); group B runs F2(t-1)
// and the SSIM map.  One barrier per slot; the F1 output and the staging tile
// are double-buffered by slot parity; group B keeps the F1 history of its row
// as two 8-column blocks used in turn.  IOM 0: Float32 inputs through
// cp.async; otherwise (an InMode) group A loads raw elements into registers a
// slot ahead and converts them when it stores them.  In-image offsets are
// 32-bit (the host routes images of 2^31 elements or more elsewhere).
// ---------------------------------------------------------------------------
template <int NT>
struct FPGeo {
    static constexpr int S = 8;
    static constexpr int R1 = NT, T = NT, R2 = NT + 2 * RAD, LAG = RAD;
    static constexpr int SP = S + 1, FC = S + 1;
    static constexpr int LROWS = (R2 + NT - 1) / NT;
    static constexpr int stage_one = R2 * SP * 8;
    static constexpr int f1_one = R1 * FC * 16;
    static constexpr int red_bytes = (2 * NT / 32 + 2) * 8;
    static constexpr int off_stage = 0;
    static constexpr int off_f1 = off_stage + 2 * stage_one;
    static constexpr int off_red = off_f1 + 2 * f1_one;
    static constexpr int total = off_red + red_bytes;
    static_assert(R1 % V == 0 && NT % 32 == 0 && S * (R1 / V) == NT, "F1 items = one per thread");
    static_assert(stage_one % 16 == 0 && f1_one % 16 == 0, "16-byte alignment of the buffers");
};

template <int NT, int IOM>
__global__ void __launch_bounds__(2 * NT, 512 / (2 * NT)) fwd_pipe_kernel(const Params p)
{
    constexpr bool F32IO = IOM == 0;
    using G = FPGeo<NT>;
    constexpr int S = G::S, R1 = G::R1, T = G::T, R2 = G::R2, LAG = G::LAG;
    constexpr int SP = G::SP, FC = G::FC;
    constexpr int STG = R2 * SP, F1N = R1 * FC;

    extern __shared__ __align__(16) unsigned char smem_raw[];
    float2* stage = reinterpret_cast<float2*>(smem_raw + G::off_stage);
    float4* f1buf = reinterpret_cast<float4*>(smem_raw + G::off_f1);
    double* red = reinterpret_cast<double*>(smem_raw + G::off_red);

    const int tid = threadIdx.x;
    const BandIndex bi = band_index(p);
    const int c = bi.c, seg = bi.seg, band = bi.band, n = bi.n;
    const int C = p.C, H = p.H, W = p.W;
    const int h0 = band * T;
    const int w0 = seg * p.L;
    const int wend = min(w0 + p.L, W);
    const int Lc = wend - w0;
    const int64_t ibase = static_cast<int64_t>(n) * p.img_elems + c;
    const float* __restrict__ xg = reinterpret_cast<const float*>(p.x) + ibase;
    const float* __restrict__ yg = reinterpret_cast<const float*>(p.y) + ibase;
    const uint32_t CH32 = static_cast<uint32_t>(C) * static_cast<uint32_t>(H);
    const int ns = (Lc + 2 * LAG - 1) / S + 1;       // steps of the stream
    const int nslot = (ns + 2) & ~1;                 // F2 lags one slot; even for the 2-slot loop

    float2 KP[RAD + 1];
#pragma unroll
    for (int i = 0; i <= RAD; ++i) KP[i] = make_float2(p.kh[i], p.kh[i]);
#define FSSIM_K2(tap) KP[(tap) <= RAD ? (tap) : 2 * RAD - (tap)]

    // group B's first slot reads F1 output that does not exist yet: zeros
    for (int e = tid; e < 2 * F1N; e += 2 * NT) f1buf[e] = make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();
    double tsum = 0.0;

    if (tid < NT) {
        // ================= group A: loads, F1 =================
        const int ta = tid;
        const int j1 = ta & (S - 1), q1 = ta >> 3;
        uint32_t lrow_off[G::LROWS];
        bool lrow_ok[G::LROWS];
#pragma unroll
        for (int r = 0; r < G::LROWS; ++r) {
            const int i = ta + NT * r;
            const int hr = h0 - LAG + i;
            lrow_ok[r] = i < R2 && hr >= 0 && hr < H;
            lrow_off[r] = static_cast<uint32_t>(C) * static_cast<uint32_t>(lrow_ok[r] ? hr : 0);
        }
        // Float32 stage copies: thread ta copies row ta (and row ta + NT while that is below
        // R2) of each column of the step.  The row sizes are per-thread constants (4, or 0
        // outside the image: a zero-size copy fills zeros and does not read its source, so a
        // masked row's address may lie outside the image); a column costs one address per input.
        static_assert(G::LROWS <= 2 && R2 - NT <= NT, "at most one extra stage row per thread");
        const int rsz0 = lrow_ok[0] ? 4 : 0;
        const int rsz1 = G::LROWS > 1 && lrow_ok[G::LROWS - 1] ? 4 : 0;
        const float* xr0 = xg + static_cast<int64_t>(C) * (h0 - LAG + ta);
        const float* yr0 = yg + static_cast<int64_t>(C) * (h0 - LAG + ta);
        const float* xr1 = xr0 + static_cast<int64_t>(C) * NT;
        const float* yr1 = yr0 + static_cast<int64_t>(C) * NT;
        auto issue_stage = [&](int k, float2* buf) {   // stage <- input columns of step k
            const int cb = w0 - LAG + k * S;
            const unsigned sd = smem_addr(buf + ta * SP);
            static_for<0, S>([&](auto jj) {
                constexpr int j = decltype(jj)::value;
                const int wc = cb + j;
                const bool colok = static_cast<unsigned>(wc) < static_cast<unsigned>(W);
                const uint32_t coff = CH32 * static_cast<uint32_t>(colok ? wc : 0);
                int sz = colok ? rsz0 : 0;
#ifdef FSSIM_DEBUG_BOUNDS
                if (sz && !FSSIM_IN_BOUNDS(ibase + lrow_off[0] + coff, p.total_elems, SITE_FPIPE_STAGE)) sz = 0;
#endif
                cp_async4_at<j * 8>(sd, xr0 + coff, sz);
                cp_async4_at<j * 8 + 4>(sd, yr0 + coff, sz);
            });
            if (G::LROWS > 1 && ta < R2 - NT) {
                static_for<0, S>([&](auto jj) {
                    constexpr int j = decltype(jj)::value;
                    const int wc = cb + j;
                    const bool colok = static_cast<unsigned>(wc) < static_cast<unsigned>(W);
                    const uint32_t coff = CH32 * static_cast<uint32_t>(colok ? wc : 0);
                    int sz = colok ? rsz1 : 0;
#ifdef FSSIM_DEBUG_BOUNDS
                    if (sz && !FSSIM_IN_BOUNDS(ibase + lrow_off[G::LROWS - 1] + coff, p.total_elems,
                                               SITE_FPIPE_STAGE))
                        sz = 0;
#endif
                    cp_async4_at<NT * SP * 8 + j * 8>(sd, xr1 + coff, sz);
                    cp_async4_at<NT * SP * 8 + j * 8 + 4>(sd, yr1 + coff, sz);
                });
            }
        };
        // converting loader: raw bits of step k in registers, stored converted by store_raw
        uint32_t rsx[F32IO ? 1 : G::LROWS * S], rsy[F32IO ? 1 : G::LROWS * S];
        auto load_raw = [&](int k) {
            const int cb = w0 - LAG + k * S;
#pragma unroll
            for (int j = 0; j < (F32IO ? 0 : S); ++j) {
                const int wc = cb + j;
                const bool colok = static_cast<unsigned>(wc) < static_cast<unsigned>(W);
#pragma unroll
                for (int r = 0; r < G::LROWS; ++r) {
                    const int64_t g = ibase + (lrow_off[r] + CH32 * static_cast<uint32_t>(colok ? wc : 0));
                    const bool ok = lrow_ok[r] && colok && FSSIM_IN_BOUNDS(g, p.total_elems, SITE_FPIPE_RAW);
                    rsx[r * S + j] = ok ? ld_in<F32IO ? IN_ANY : IOM>(p.x, p.xdt, g) : 0u;
                    rsy[r * S + j] = ok ? ld_in<F32IO ? IN_ANY : IOM>(p.y, p.ydt, g) : 0u;
                }
            }
        };
        auto store_raw = [&](float2* buf) {
#pragma unroll
            for (int j = 0; j < (F32IO ? 0 : S); ++j) {
#pragma unroll
                for (int r = 0; r < G::LROWS; ++r) {
                    const int i = ta + NT * r;
                    if (G::LROWS == 1 || i < R2)
                        buf[i * SP + j] = make_float2(cvt_in<F32IO ? IN_ANY : IOM>(rsx[r * S + j], p.xdt),
                                                      cvt_in<F32IO ? IN_ANY : IOM>(rsy[r * S + j], p.ydt));
                }
            }
        };
        if (F32IO) {
            issue_stage(0, stage);
            cp_async_commit();
            cp_async_wait<0>();
        } else {
            load_raw(0);
            store_raw(stage);
        }
        named_barrier_sync(BAR_SLOT, 2 * NT);
#pragma unroll 1
        for (int t = 0; t < nslot; ++t) {
            if (F32IO) {
                if (t + 1 < ns) issue_stage(t + 1, stage + ((t + 1) & 1) * STG);
                cp_async_commit();
            } else if (t + 1 < ns) {
                load_raw(t + 1);
            }
            if (t < ns) {   // -------- F1(t): h-direction pass of the 4 moment images --------
                const float2* st = stage + (t & 1) * STG;
                float4* f1 = f1buf + (t & 1) * F1N;
                float2 aA[V], aB[V];
#pragma unroll
                for (int o = 0; o < V; ++o) {
                    aA[o] = make_float2(0.f, 0.f);
                    aB[o] = make_float2(0.f, 0.f);
                }
#pragma unroll
                for (int i = 0; i < V + 2 * RAD; ++i) {
                    const float2 xy = st[(V * q1 + i) * SP + j1];
                    const float2 sq = __fmul2_rn(xy, xy);                     // (x^2, y^2)
                    const float2 sb = make_float2(sq.x + sq.y, xy.x * xy.y);  // (x^2+y^2, xy)
#pragma unroll
                    for (int o = 0; o < V; ++o) {
                        const int tap = i - o;
                        if (tap >= 0 && tap < TAPS) {
                            aA[o] = __ffma2_rn(xy, FSSIM_K2(tap), aA[o]);
                            aB[o] = __ffma2_rn(sb, FSSIM_K2(tap), aB[o]);
                        }
                    }
                }
#pragma unroll
                for (int o = 0; o < V; ++o)
                    f1[(V * q1 + o) * FC + j1] = make_float4(aA[o].x, aA[o].y, aB[o].x, aB[o].y);
            }
            if (F32IO) cp_async_wait<0>();
            else if (t + 1 < ns) store_raw(stage + ((t + 1) & 1) * STG);
            named_barrier_sync(BAR_SLOT, 2 * NT);
        }
    } else {
        // ================= group B: F2 + SSIM map =================
        const int tb = tid - NT;
        const bool row_owned = h0 + tb < H;
        static_assert(HIST == S + 2, "window = 2 saved columns + previous block + current block");
        float2 A0[S], A1[S], B0[S], B1[S], TA[2], TB[2];
#pragma unroll
        for (int m = 0; m < S; ++m) A0[m] = A1[m] = B0[m] = B1[m] = make_float2(0.f, 0.f);
        TA[0] = TA[1] = TB[0] = TB[1] = make_float2(0.f, 0.f);
        auto bslot = [&](int t, float2(&Acur)[S], float2(&Aprv)[S], float2(&Bcur)[S], float2(&Bprv)[S]) {
            const int k = t - 1;   // F2 of step k (k = -1 reads the zeroed buffer)
            const float4* f1 = f1buf + (k & 1) * F1N;
            const int wcb = w0 - LAG + k * S - RAD;   // image column of output o = 0
            float ssum = 0.f;
#define FSSIM_WA(m) ((m) < 2 ? TA[(m)] : ((m) < HIST ? Aprv[(m) - 2] : Acur[(m) - HIST]))
#define FSSIM_WB(m) ((m) < 2 ? TB[(m)] : ((m) < HIST ? Bprv[(m) - 2] : Bcur[(m) - HIST]))
#pragma unroll
            for (int o = 0; o < S; ++o) {
                {   // column o of this step enters the window just before its first use
                    const float4 v = f1[tb * FC + o];
                    Acur[o] = make_float2(v.x, v.y);
                    Bcur[o] = make_float2(v.z, v.w);
                }
                float2 a = __fmul2_rn(FSSIM_WA(o + RAD), KP[RAD]);
                float2 b = __fmul2_rn(FSSIM_WB(o + RAD), KP[RAD]);
#pragma unroll
                for (int tap = 0; tap < RAD; ++tap) {
                    a = __ffma2_rn(__fadd2_rn(FSSIM_WA(o + tap), FSSIM_WA(o + 2 * RAD - tap)), KP[tap], a);
                    b = __ffma2_rn(__fadd2_rn(FSSIM_WB(o + tap), FSSIM_WB(o + 2 * RAD - tap)), KP[tap], b);
                }
                const float mx = a.x, my = a.y, qs = b.x, pxy = b.y;
                const float2 sq = __fmul2_rn(a, a);
                const float mxy = mx * my;
                const float sumsq = sq.x + sq.y;
                const float z = sumsq + p.C1;                    // mx^2 + my^2 + C1
                const float tt = (qs - sumsq) + p.C2;            // vx + vy + C2
                const float ax = fmaf(2.f, mxy, p.C1);           // 2 mx my + C1
                const float by = fmaf(2.f, pxy - mxy, p.C2);     // 2 cov + C2
                const float s = (ax * by) * rcp_approx(z * tt);
                const int wc = wcb + o;
                if (row_owned && static_cast<unsigned>(wc - w0) < static_cast<unsigned>(Lc)) ssum += s;
            }
#undef FSSIM_WA
#undef FSSIM_WB
            tsum += static_cast<double>(ssum);
            TA[0] = Aprv[S - 2];
            TA[1] = Aprv[S - 1];
            TB[0] = Bprv[S - 2];
            TB[1] = Bprv[S - 1];
            named_barrier_sync(BAR_SLOT, 2 * NT);
        };
        named_barrier_sync(BAR_SLOT, 2 * NT);
#pragma unroll 1
        for (int t = 0; t < nslot; t += 2) {
            bslot(t, A0, A1, B0, B1);
            bslot(t + 1, A1, A0, B1, B0);
        }
    }
#undef FSSIM_K2

    const int local_cta = (band * p.nseg + seg) * p.C + c;
    finish_image<2 * NT>(p, n, local_cta, tsum, red);
}


// ---------------------------------------------------------------------------
// Tile kernel for small forward-only calls (a single image, a few images).
//
// The streaming kernels cut a lone full-HD image into many short segments, each
// of which streams 10 halo columns and waits on two barriers per step, with two
// warps per CTA.  Here a CTA of 256 threads computes the SSIM map of one
// TH x TW output tile of one channel in three phases, with the whole input
// tile loaded at once:
//   load  (TH+10) x (TW+10) inputs of x and y (converted to Float32) -> stage
//   F1    h-direction 11-tap pass of the 4 moment images, all TW+10 columns
//   F2    w-direction pass, SSIM map and the tile's sum
// Shared-memory strides are odd (in 8- and 16-byte units), so the column reads
// of F1 and the row reads of F2 are conflict-free.
// ---------------------------------------------------------------------------
struct TGeo {
    static constexpr int TH = 32, TW = 54;           // output tile: rows (h) x columns (w)
    static constexpr int NT = 256;
    static constexpr int IR = TH + 2 * RAD;          // input rows
    static constexpr int IC = TW + 2 * RAD;          // input columns = F1 output columns
    static constexpr int RS = IR + 1;                // stage column stride (float2), odd
    static constexpr int NG = (TW + V - 1) / V;      // F2 column groups of V outputs per row
    static constexpr int FS = NG * V + 2 * RAD + 1;  // F1 row stride (float4), odd, covers the last group
    static constexpr int NE = IR * IC;               // staged elements
    static constexpr int stage_one = IC * RS * 8;
    static constexpr int f1_bytes = TH * FS * 16;
    static constexpr int red_bytes = (NT / 32 + 2) * 8;
    static constexpr int total = stage_one + f1_bytes + red_bytes;
    static_assert(IC * (TH / V) == NT, "one F1 item per thread");
    static_assert(TH * NG <= NT, "one F2 item per thread");
    static_assert(RS % 2 == 1 && FS % 2 == 1, "odd strides");
    static_assert(stage_one % 16 == 0, "f1 stays 16-byte aligned");
};

// IM: 0 = Float32 inputs, otherwise an InMode (N0f8 / Float16 / any, converted).
// CTA t computes tile t; the loop over t (stride gridDim.x) also serves grids
// smaller than the tile count.  A resident CTA's next tile streaming in behind
// the current one was measured slower: it halves the CTAs per SM.
template <int IM>
__global__ void __launch_bounds__(TGeo::NT, 4) tile_fwd_kernel(const Params p)
{
    using G = TGeo;
    constexpr int TH = G::TH, TW = G::TW, IR = G::IR, IC = G::IC, RS = G::RS, FS = G::FS;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float2* stage = reinterpret_cast<float2*>(smem_raw);                  // [IC][RS], (x, y)
    float4* f1 = reinterpret_cast<float4*>(smem_raw + G::stage_one);      // [TH][FS]
    double* red = reinterpret_cast<double*>(smem_raw + G::stage_one + G::f1_bytes);

    const int tid = threadIdx.x;
    const int C = p.C, H = p.H, W = p.W;
    const int64_t CH = static_cast<int64_t>(C) * H;
    const int64_t ntiles = static_cast<int64_t>(p.N) * p.cpi;
    struct Tile {
        int n, th, tw, c;
        int64_t ibase;
    };
    // tile index -> (channel, tile column, tile row, image); 32-bit divisions, as the
    // host keeps the tile count below 2^31
    auto tile_of = [&](int64_t t64) {
        Tile u;
        uint32_t t = static_cast<uint32_t>(t64);
        const uint32_t tc = t / static_cast<uint32_t>(C);
        u.c = static_cast<int>(t - tc * static_cast<uint32_t>(C));
        const uint32_t ts = tc / static_cast<uint32_t>(p.nseg);
        u.tw = static_cast<int>(tc - ts * static_cast<uint32_t>(p.nseg));
        const uint32_t tb = ts / static_cast<uint32_t>(p.nb);
        u.th = static_cast<int>(ts - tb * static_cast<uint32_t>(p.nb));
        u.n = static_cast<int>(tb);
        u.ibase = static_cast<int64_t>(u.n) * p.img_elems + u.c;
        return u;
    };
    // Stage element (row r, column q) of a tile.  Thread tid < LG * IR loads row
    // r = tid % IR of columns q = tid / IR + LG j (a warp reads consecutive rows of a
    // column), so its row test is made once and each column costs one test and one
    // pointer step; zero outside the image.  All loads of the tile are issued before the
    // first store.
    constexpr int LG = G::NT / IR;                 // column phases
    constexpr int NJ = (IC + LG - 1) / LG;         // columns per thread
    auto load_convert = [&](const Tile& u, float2* buf) {
        const int r = tid % IR, q0 = tid / IR;
        const int hr = u.th * TH - RAD + r, wc0 = u.tw * TW - RAD + q0;
        const bool row_ok = tid < LG * IR && hr >= 0 && hr < H;
        // element index of (row r, column q0); a masked load never uses it
        const int64_t g0 = u.ibase + static_cast<int64_t>(C) * hr + CH * wc0;
        const int64_t gstep = CH * LG;
        uint32_t rx[NJ], ry[NJ];
        const unsigned int* px = reinterpret_cast<const unsigned int*>(p.x) + g0;
        const unsigned int* py = reinterpret_cast<const unsigned int*>(p.y) + g0;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            const int wc = wc0 + LG * j;
            const int64_t g = g0 + gstep * j;
            const bool ok = row_ok && (j < NJ - 1 || q0 + LG * j < IC) &&
                            static_cast<unsigned>(wc) < static_cast<unsigned>(W) &&
                            FSSIM_IN_BOUNDS(g, p.total_elems, SITE_TILE_LOAD);
            if (IM == 0) {
                rx[j] = ok ? __ldg(px) : 0u;
                ry[j] = ok ? __ldg(py) : 0u;
                px += gstep;
                py += gstep;
            } else {
                rx[j] = ok ? ld_in<IM>(p.x, p.xdt, g) : 0u;
                ry[j] = ok ? ld_in<IM>(p.y, p.ydt, g) : 0u;
            }
        }
        if (tid < LG * IR) {
            float2* d = buf + q0 * RS + r;
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                if (j < NJ - 1 || q0 + LG * j < IC)
                    d[LG * j * RS] = IM == 0 ? make_float2(__uint_as_float(rx[j]), __uint_as_float(ry[j]))
                                             : make_float2(cvt_in<IM>(rx[j], p.xdt), cvt_in<IM>(ry[j], p.ydt));
            }
        }
    };

    // F1 columns past IC feed only outputs outside the tile: keep them finite
    for (int e = tid; e < TH * (FS - IC); e += G::NT)
        f1[(e / (FS - IC)) * FS + IC + e % (FS - IC)] = make_float4(0.f, 0.f, 0.f, 0.f);
    float2 KP[RAD + 1];
#pragma unroll
    for (int i = 0; i <= RAD; ++i) KP[i] = make_float2(p.kh[i], p.kh[i]);
#define FSSIM_K2(tap) KP[(tap) <= RAD ? (tap) : 2 * RAD - (tap)]

#pragma unroll 1
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
        float2* st = stage;
        const Tile u = tile_of(t);
        load_convert(u, st);
        __syncthreads();   // the stage is complete; the previous tile's F2 is done with f1

        // ---- F1: rows V*q1 .. V*q1+V-1 of column q (stage rows V*q1 .. V*q1+V+2R-1)
        {
            const int q = tid % IC, q1 = tid / IC;
            float2 aA[V], aB[V];
#pragma unroll
            for (int o = 0; o < V; ++o) {
                aA[o] = make_float2(0.f, 0.f);
                aB[o] = make_float2(0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < V + 2 * RAD; ++i) {
                const float2 xy = st[q * RS + V * q1 + i];
                const float2 sq = __fmul2_rn(xy, xy);
                const float2 sb = make_float2(sq.x + sq.y, xy.x * xy.y);     // (x^2+y^2, xy)
#pragma unroll
                for (int o = 0; o < V; ++o) {
                    const int tap = i - o;
                    if (tap >= 0 && tap < TAPS) {
                        aA[o] = __ffma2_rn(xy, FSSIM_K2(tap), aA[o]);
                        aB[o] = __ffma2_rn(sb, FSSIM_K2(tap), aB[o]);
                    }
                }
            }
#pragma unroll
            for (int o = 0; o < V; ++o)
                f1[(V * q1 + o) * FS + q] = make_float4(aA[o].x, aA[o].y, aB[o].x, aB[o].y);
        }
        __syncthreads();

        // ---- F2 + map: row r, output columns V*g .. V*g+V-1 of the tile
        double tsum = 0.0;
        {
            const int r = tid % TH, g = tid / TH;
            if (g < G::NG) {
                float2 a[V], b[V];
#pragma unroll
                for (int o = 0; o < V; ++o) {
                    a[o] = make_float2(0.f, 0.f);
                    b[o] = make_float2(0.f, 0.f);
                }
#pragma unroll
                for (int m = 0; m < V + 2 * RAD; ++m) {
                    const float4 v = f1[r * FS + V * g + m];
                    const float2 va = make_float2(v.x, v.y), vb = make_float2(v.z, v.w);
#pragma unroll
                    for (int o = 0; o < V; ++o) {
                        const int tap = m - o;
                        if (tap >= 0 && tap < TAPS) {
                            a[o] = __ffma2_rn(va, FSSIM_K2(tap), a[o]);
                            b[o] = __ffma2_rn(vb, FSSIM_K2(tap), b[o]);
                        }
                    }
                }
                const int hr = u.th * TH + r, w0 = u.tw * TW;
                float ssum = 0.f;
#pragma unroll
                for (int o = 0; o < V; ++o) {
                    const float mx = a[o].x, my = a[o].y, qs = b[o].x, pxy = b[o].y;
                    const float2 sq = __fmul2_rn(a[o], a[o]);
                    const float mxy = mx * my;
                    const float sumsq = sq.x + sq.y;
                    const float z = sumsq + p.C1;
                    const float tt = (qs - sumsq) + p.C2;
                    const float ax = fmaf(2.f, mxy, p.C1);
                    const float by = fmaf(2.f, pxy - mxy, p.C2);
                    const float sv = (ax * by) * rcp_approx(z * tt);
                    const int col = V * g + o;
                    if (hr < H && col < TW && w0 + col < W) ssum += sv;
                }
                tsum = static_cast<double>(ssum);
            }
        }
        finish_image<G::NT>(p, u.n, (u.th * p.nseg + u.tw) * C + u.c, tsum, red);
    }
#undef FSSIM_K2
}

// ---------------------------------------------------------------------------
// Tile kernel with TMA loads: one-channel Float32 images whose height is a
// multiple of 4.  The same three phases as tile_fwd_kernel, but the input tile
// arrives as two tensor-memory-access boxes (x and y), issued by one thread and
// completed on an mbarrier, so the CTA spends no instructions on the loads.
//
// A TMA box must start at a 16-byte boundary of the contiguous (height) axis.
// Tile rows therefore start at 32*th - 3, so that each box starts at image row
// 32*th - 8, a multiple of 4.  The box is 44 rows by 64 columns and lands in
// shared memory as [column][row]: its 44-float columns are 11 16-byte chunks, an
// odd number, so the h-pass reads four rows per 16-byte load without bank
// conflicts.  Rows and columns outside the image are filled with zeros by the
// copy itself.  The wait on the mbarrier is bounded; were it ever to run out,
// the tile's sum becomes NaN, so the image's value shows it.
// ---------------------------------------------------------------------------
struct TTGeo {
    static constexpr int TH = 32, TW = 54;           // output tile: rows (h) x columns (w)
    static constexpr int NT = 256;
    static constexpr int SHIFT = 3;                  // tile th covers rows 32*th - 3 .. 32*th + 28
    static constexpr int BR = 44;                    // box rows: 32*th - 8 .. 32*th + 35
    static constexpr int IC = TW + 2 * RAD;          // box columns = F1 output columns (64)
    static constexpr int NG = (TW + V - 1) / V;      // F2 column groups of V outputs per row
    static constexpr int FS = NG * V + 2 * RAD + 1;  // F1 row stride (float4), odd
    static constexpr int plane_bytes = IC * BR * 4;  // one input's box
    static constexpr int f1_bytes = TH * FS * 16;
    static constexpr int red_bytes = (NT / 32 + 2) * 8;
    static constexpr int off_x = 0, off_y = plane_bytes, off_f1 = 2 * plane_bytes;
    static constexpr int off_red = off_f1 + f1_bytes, off_bar = off_red + red_bytes;
    static constexpr int total = off_bar + 8;
    static constexpr unsigned tx_bytes = 2u * plane_bytes;
    static_assert(BR % 4 == 0 && (BR / 4) % 2 == 1, "box columns: an odd number of whole 16-byte chunks");
    static_assert((SHIFT + RAD) % 4 == 0 && TH % 4 == 0, "every box starts at a multiple of 4 rows");
    static_assert(TH + 2 * RAD <= BR, "the box covers the tile's rows and their halo");
    static_assert(V * (TH / V - 1) + 4 * ((V + 2 * RAD + 3) / 4) <= BR, "the h-pass reads whole chunks inside the box");
    static_assert(IC * (TH / V) == NT && TH * NG <= NT, "one F1 item and at most one F2 item per thread");
    static_assert(FS % 2 == 1 && plane_bytes % 128 == 0 && off_bar % 8 == 0, "strides and alignment");
};

__device__ __forceinline__ void tma_load_3d(unsigned dst, const CUtensorMap* tm, int x, int y, int z, unsigned bar)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];\n"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

// Waits for phase `phase` of the mbarrier at `bar`; false if it did not complete
// within the bound (each try_wait may itself suspend the thread for a while).
__device__ __forceinline__ bool mbar_wait_bounded(unsigned bar, unsigned phase)
{
    for (int i = 0; i < (1 << 20); ++i) {
        unsigned done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(bar), "r"(phase)
            : "memory");
        if (done) return true;
    }
    return false;
}

__global__ void __launch_bounds__(TTGeo::NT, 4)
    tile_tma_kernel(const Params p, const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmy)
{
    using G = TTGeo;
    constexpr int TH = G::TH, TW = G::TW, IC = G::IC, BR = G::BR, FS = G::FS;
    extern __shared__ __align__(128) unsigned char smem_tma[];
    float* sx = reinterpret_cast<float*>(smem_tma + G::off_x);       // [IC][BR]
    float* sy = reinterpret_cast<float*>(smem_tma + G::off_y);
    float4* f1 = reinterpret_cast<float4*>(smem_tma + G::off_f1);    // [TH][FS]
    double* red = reinterpret_cast<double*>(smem_tma + G::off_red);
    const unsigned bar = smem_addr(smem_tma + G::off_bar);

    const int tid = threadIdx.x;
    const int H = p.H, W = p.W;
    // block -> (tile column, tile row, image); one channel; 32-bit divisions (grid < 2^31)
    const uint32_t b0 = blockIdx.x, q1b = b0 / static_cast<uint32_t>(p.nseg), q2b = q1b / static_cast<uint32_t>(p.nb);
    const int tw = static_cast<int>(b0 - q1b * static_cast<uint32_t>(p.nseg));
    const int th = static_cast<int>(q1b - q2b * static_cast<uint32_t>(p.nb));
    const int n = static_cast<int>(q2b);

    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(bar) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    // F1 columns past IC feed only outputs outside the tile: keep them finite
    for (int e = tid; e < TH * (FS - IC); e += G::NT)
        f1[(e / (FS - IC)) * FS + IC + e % (FS - IC)] = make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();
    if (tid == 0) {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(G::tx_bytes)
                     : "memory");
        const int r0 = th * TH - G::SHIFT - RAD;   // 32*th - 8: 16-byte aligned
        const int c0 = tw * TW - RAD;
        tma_load_3d(smem_addr(sx), &tmx, r0, c0, n, bar);
        tma_load_3d(smem_addr(sy), &tmy, r0, c0, n, bar);
    }
    float2 KP[RAD + 1];
#pragma unroll
    for (int i = 0; i <= RAD; ++i) KP[i] = make_float2(p.kh[i], p.kh[i]);
#define FSSIM_K2(tap) KP[(tap) <= RAD ? (tap) : 2 * RAD - (tap)]
    const bool landed = mbar_wait_bounded(bar, 0u);

    // ---- F1: rows V*q1 .. V*q1+V-1 of column q (box rows V*q1 .. V*q1+V+2R-1)
    {
        const int q = tid % IC, q1 = tid / IC;
        const float4* cx = reinterpret_cast<const float4*>(sx + q * BR + V * q1);
        const float4* cy = reinterpret_cast<const float4*>(sy + q * BR + V * q1);
        float2 aA[V], aB[V];
#pragma unroll
        for (int o = 0; o < V; ++o) {
            aA[o] = make_float2(0.f, 0.f);
            aB[o] = make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int ch = 0; ch < (V + 2 * RAD + 3) / 4; ++ch) {
            const float4 x4 = cx[ch], y4 = cy[ch];
            const float xr[4] = {x4.x, x4.y, x4.z, x4.w}, yr[4] = {y4.x, y4.y, y4.z, y4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int i = 4 * ch + j;
                if (i < V + 2 * RAD) {
                    const float2 xy = make_float2(xr[j], yr[j]);
                    const float2 sq = __fmul2_rn(xy, xy);
                    const float2 sb = make_float2(sq.x + sq.y, xy.x * xy.y);   // (x^2+y^2, xy)
#pragma unroll
                    for (int o = 0; o < V; ++o) {
                        const int tap = i - o;
                        if (tap >= 0 && tap < TAPS) {
                            aA[o] = __ffma2_rn(xy, FSSIM_K2(tap), aA[o]);
                            aB[o] = __ffma2_rn(sb, FSSIM_K2(tap), aB[o]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int o = 0; o < V; ++o)
            f1[(V * q1 + o) * FS + q] = make_float4(aA[o].x, aA[o].y, aB[o].x, aB[o].y);
    }
    __syncthreads();
    // every thread is past the wait: the mbarrier's word goes back to plain shared memory
    if (tid == 0) asm volatile("mbarrier.inval.shared::cta.b64 [%0];\n" ::"r"(bar) : "memory");

    // ---- F2 + map: row r, output columns V*g .. V*g+V-1 of the tile
    double tsum = 0.0;
    {
        const int r = tid % TH, g = tid / TH;
        if (g < G::NG) {
            float2 a[V], b[V];
#pragma unroll
            for (int o = 0; o < V; ++o) {
                a[o] = make_float2(0.f, 0.f);
                b[o] = make_float2(0.f, 0.f);
            }
#pragma unroll
            for (int m = 0; m < V + 2 * RAD; ++m) {
                const float4 v = f1[r * FS + V * g + m];
                const float2 va = make_float2(v.x, v.y), vb = make_float2(v.z, v.w);
#pragma unroll
                for (int o = 0; o < V; ++o) {
                    const int tap = m - o;
                    if (tap >= 0 && tap < TAPS) {
                        a[o] = __ffma2_rn(va, FSSIM_K2(tap), a[o]);
                        b[o] = __ffma2_rn(vb, FSSIM_K2(tap), b[o]);
                    }
                }
            }
            const int hr = th * TH - G::SHIFT + r, w0 = tw * TW;
            float ssum = 0.f;
#pragma unroll
            for (int o = 0; o < V; ++o) {
                const float mx = a[o].x, my = a[o].y, qs = b[o].x, pxy = b[o].y;
                const float2 sq = __fmul2_rn(a[o], a[o]);
                const float mxy = mx * my;
                const float sumsq = sq.x + sq.y;
                const float z = sumsq + p.C1;
                const float tt = (qs - sumsq) + p.C2;
                const float ax = fmaf(2.f, mxy, p.C1);
                const float by = fmaf(2.f, pxy - mxy, p.C2);
                const float sv = (ax * by) * rcp_approx(z * tt);
                const int col = V * g + o;
                if (static_cast<unsigned>(hr) < static_cast<unsigned>(H) && col < TW && w0 + col < W) ssum += sv;
            }
            tsum = landed ? static_cast<double>(ssum) : __longlong_as_double(0x7ff8000000000000ll);
        }
    }
#undef FSSIM_K2
    finish_image<G::NT>(p, n, th * p.nseg + tw, tsum, red);
}

}  // namespace fssim

// Fused SSIM / DSSIM kernels for sm_100a.
//
// Replaces FastCUDASSIM.jl's two CUDA.jl kernels (src/core.jl:147-447 forward,
// src/core.jl:567-800 backward) and the divide-by-N broadcast
// (src/core.jl:1123-1157) with ONE launch per call.
//
// Decomposition.  A CTA owns one channel c of one image n, a band of T output
// rows [h0, h0+T) along the contiguous height axis, and a segment of output
// columns [w0, w0+L) along the width axis.  It streams along the width axis in
// steps of S columns:
//
//   loader  global (C,H,W,N) -> shared staging with cp.async (Float32 I/O), or
//           one step ahead through registers with an in-kernel conversion
//           (Float16, N0f8 inputs; Float16 / Float64 gradients)
//   F1      h-direction 11-tap Gaussian of the 4 moment images x, y, x^2+y^2, xy
//           (each thread: V = 8 consecutive rows of one column; taps from smem)
//   F2      w-direction 11-tap Gaussian (each thread: one row; the 10 previous
//           columns stay in registers, so no column is ever recomputed inside a
//           segment), then the SSIM map and, for gradients, the three partial
//           derivatives dS/dQ, dS/dM, dS/dP at that pixel (zero outside the image),
//           pre-scaled by +-1/N so the backward pass needs no final multiply
//   B1, B2  the same two passes over the partial-derivative images, then the
//           combine x*K(2 dQ) + K(dM) + y*K(dP)
//
// With gradients the forward stages run on the band plus a 5-row halo (the
// backward correlation needs partials there); the width halo costs nothing but
// the 10+10 warm-up columns of each segment.  Nothing but the inputs, the
// gradient and one double per CTA ever touches global memory.
//
// Kernels: pipe_kernel (SSIM + gradient, two warp groups); forward only:
// fwd_pipe_kernel (its forward half, calls above 4 Mi elements), tile_fwd_kernel
// (smaller calls, mixed input dtypes) and band_kernel (single group, 64-bit
// offsets: Float32 images of 2^31 elements or more); f64_kernel (any call with
// a Float64 input, in double precision).
//
// Only four moment images are convolved, not the reference's five: the SSIM map
// needs the two variances only through their sum, so E[x^2] and E[y^2] are
// convolved together as E[x^2 + y^2] (t = E[x^2+y^2] - mx^2 - my^2 + C2).
// Pairs of moments share one packed FP32x2 FMA (FFMA2) per tap.
//
// Per-image sums: each CTA writes one double to the workspace; the last CTA of
// an image (atomic counter) adds them in a fixed order, divides by N and applies
// the DSSIM transform, so results are bitwise reproducible.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fssim {

constexpr int RAD = 5;              // Gaussian radius (src/core.jl:41)
constexpr int TAPS = 2 * RAD + 1;   // 11
constexpr int V = 8;                // rows per thread in the h-direction passes
constexpr int HIST = 2 * RAD;       // columns of history kept in registers

enum DType { DT_F32 = 0, DT_F16 = 1, DT_U8 = 2, DT_F64 = 3 };

struct Params {
    const void* x;            // imgs1, canonical (C,H,W,N)
    const void* y;            // imgs2
    void* grad;               // dL/dimgs1 (fused kernels with a gradient)
    void* ssims;              // length-N output (kernels with WANT_SSIM)
    double* partials;         // workspace: N * cpi doubles
    unsigned int* counters;   // workspace: N counters, zero between calls
    int64_t img_elems;        // C*H*W
    int64_t total_elems;      // N*C*H*W (bounds of x, y and the gradient)
    int C, H, W, N;
    int nb, nseg, L;          // bands, segments, segment length (columns)
    int cpi;                  // CTAs per image = C * nb * nseg
    int xdt, ydt, gdt, sdt;   // dtypes of x, y, grad, ssims
    int should_zero, use_dssim, div2;
    float kh[RAD + 1];        // Gaussian weights k[0..5] (k[10-i] == k[i]; src/core.jl:40-46)
    float C1, C2;             // src/core.jl:49-50
    float gscale;             // +-1/N or +-0.5/N (src/core.jl:584-589, sign for DSSIM)
    double npx;               // N = C*H*W as a double
    const void* img_scale;    // optional per-image gradient factor (length N), dtype isdt
    int isdt;
};

__device__ __forceinline__ float rcp_approx(float v)
{
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}

// Opt-in bounds checking (built with -DFSSIM_DEBUG_BOUNDS, the library's stand-in
// for a memory checker): every global access first checks its element index
// against the array it addresses.  An index out of range is recorded (the first
// failing site and a count) and the access is skipped instead of made.
#ifdef FSSIM_DEBUG_BOUNDS
__device__ unsigned g_fssim_bounds_site;
__device__ unsigned long long g_fssim_bounds_count;
__device__ __forceinline__ bool in_bounds(int64_t idx, int64_t limit, unsigned site)
{
    if (idx >= 0 && idx < limit) return true;
    atomicCAS(&g_fssim_bounds_site, 0u, site);
    atomicAdd(&g_fssim_bounds_count, 1ull);
    return false;
}
#define FSSIM_IN_BOUNDS(idx, limit, site) ::fssim::in_bounds((idx), (limit), (site))
#else
#define FSSIM_IN_BOUNDS(idx, limit, site) true
#endif
// Site numbers reported by the bounds-checked build.
enum BoundsSite : unsigned {
    SITE_BAND_LOAD = 1, SITE_PIPE_STAGE, SITE_PIPE_XY, SITE_PIPE_STAGE_RAW, SITE_PIPE_XY_RAW,
    SITE_PIPE_GRAD, SITE_TILE_LOAD, SITE_F64_LOAD, SITE_F64_GRAD, SITE_PARTIALS, SITE_COUNTERS,
    SITE_FPIPE_STAGE, SITE_FPIPE_RAW
};

// Raw bits of one input element (zero-extended); converted at staging time so
// that the load's latency is not exposed at the point of issue.
__device__ __forceinline__ uint32_t ld_raw(const void* base, int dt, int64_t idx)
{
    if (dt == DT_F32) return __ldg(reinterpret_cast<const unsigned int*>(base) + idx);
    if (dt == DT_F16) return __ldg(reinterpret_cast<const unsigned short*>(base) + idx);
    return __ldg(reinterpret_cast<const unsigned char*>(base) + idx);
}

// N0f8 -> Float32: the correctly rounded value of raw/255.  q = raw * fl(1/255)
// is off by one ulp for about half of the 256 bytes; one Newton correction step
// for a constant divisor (residual e = raw - 255 q by FMA, then q + e * fl(1/255))
// gives the correctly rounded quotient for every byte (checked exhaustively, and
// against the division by a GPU test).
__device__ __forceinline__ float n0f8_to_f32(uint32_t r)
{
    const float inv = 1.0f / 255.0f;
    const float fr = static_cast<float>(r & 255u);
    const float q = fr * inv;
    const float e = fmaf(-q, 255.0f, fr);
    return fmaf(e, inv, q);
}

__device__ __forceinline__ float cvt_raw(uint32_t r, int dt, const float* /*unused*/)
{
    if (dt == DT_F32) return __uint_as_float(r);
    if (dt == DT_F16) return __half2float(__ushort_as_half(static_cast<unsigned short>(r)));
    return n0f8_to_f32(r);
}

// Input modes of the converting kernels: both inputs N0f8, both Float16, or any
// mix (dtype read at run time).
enum InMode { IN_U8 = 1, IN_F16 = 2, IN_ANY = 3 };

template <int IM>
__device__ __forceinline__ uint32_t ld_in(const void* base, int dt, int64_t idx)
{
    if (IM == IN_U8) return __ldg(reinterpret_cast<const unsigned char*>(base) + idx);
    if (IM == IN_F16) return __ldg(reinterpret_cast<const unsigned short*>(base) + idx);
    return ld_raw(base, dt, idx);
}

template <int IM>
__device__ __forceinline__ float cvt_in(uint32_t r, int dt)
{
    if (IM == IN_U8) return n0f8_to_f32(r);
    if (IM == IN_F16) return __half2float(__ushort_as_half(static_cast<unsigned short>(r)));
    return cvt_raw(r, dt, nullptr);
}

__device__ __forceinline__ void st_grad(void* base, int dt, int64_t idx, float v)
{
    if (dt == DT_F32) reinterpret_cast<float*>(base)[idx] = v;
    else if (dt == DT_F16) reinterpret_cast<__half*>(base)[idx] = __float2half_rn(v);
    else reinterpret_cast<double*>(base)[idx] = static_cast<double>(v);
}

__device__ __forceinline__ double ld_out(const void* base, int dt, int64_t i)
{
    if (dt == DT_F32) return reinterpret_cast<const float*>(base)[i];
    if (dt == DT_F16) return __half2float(reinterpret_cast<const __half*>(base)[i]);
    return reinterpret_cast<const double*>(base)[i];
}

__device__ __forceinline__ void st_out(void* base, int dt, int64_t i, double v)
{
    if (dt == DT_F32) reinterpret_cast<float*>(base)[i] = static_cast<float>(v);
    else if (dt == DT_F16) reinterpret_cast<__half*>(base)[i] = __double2half(v);
    else reinterpret_cast<double*>(base)[i] = v;
}

// 4-byte asynchronous global->shared copy; a false `valid` zero-fills the
// destination without reading global memory (src-size 0).
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc, bool valid)
{
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    const int sz = valid ? 4 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gsrc), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

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

// Reduce a per-thread double over the CTA in a fixed order; result valid in thread 0.
template <int NT>
__device__ __forceinline__ double block_sum(double v, double* red)
{
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    double tot = 0.0;
    if (threadIdx.x == 0) {
#pragma unroll
        for (int w = 0; w < NT / 32; ++w) tot += red[w];
    }
    return tot;
}

// Writes this CTA's map sum, and, in the last CTA of the image, the final value.
template <int NT>
__device__ __forceinline__ void finish_image(const Params& p, int n, int local_cta, double tsum,
                                             double* red)
{
    const double tot = block_sum<NT>(tsum, red);
    if (threadIdx.x == 0) {
        const int64_t slot = (int64_t)n * p.cpi + local_cta;
        const bool ok = FSSIM_IN_BOUNDS(slot, (int64_t)p.N * p.cpi, SITE_PARTIALS) &&
                        FSSIM_IN_BOUNDS(n, p.N, SITE_COUNTERS);
        unsigned prev = 0u;
        if (ok) {
            p.partials[slot] = tot;
            __threadfence();
            prev = atomicAdd(&p.counters[n], 1u);
        }
        red[NT / 32] = (ok && prev == static_cast<unsigned>(p.cpi - 1)) ? 1.0 : 0.0;
    }
    __syncthreads();
    if (red[NT / 32] != 0.0) {   // uniform over the CTA; no early return, so loops may call this
        __threadfence();
        double v = 0.0;
        for (int i = threadIdx.x; i < p.cpi; i += NT) {
            v += __ldcg(&p.partials[(int64_t)n * p.cpi + i]);
            // leave the workspace zeroed: a later call with more images places its
            // counters where these partial sums were
            p.partials[(int64_t)n * p.cpi + i] = 0.0;
        }
        __syncthreads();   // red[] is reused below
        const double sum = block_sum<NT>(v, red);
        if (threadIdx.x == 0) {
            double s = sum;
            if (!p.should_zero) s += ld_out(p.ssims, p.sdt, n);
            s = s / p.npx;                               // src/core.jl:1125-1157
            if (p.use_dssim) s = p.div2 ? (1.0 - s) * 0.5 : 1.0 - s;
            st_out(p.ssims, p.sdt, n, s);
            p.counters[n] = 0u;                          // leave the workspace zeroed
        }
    }
}

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
    int64_t blk = blockIdx.x;
    const int c = static_cast<int>(blk % p.C);
    blk /= p.C;
    const int seg = static_cast<int>(blk % p.nseg);
    blk /= p.nseg;
    const int band = static_cast<int>(blk % p.nb);
    const int n = static_cast<int>(blk / p.nb);
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

}  // namespace fssim

namespace fssim {

// ---------------------------------------------------------------------------
// Two-group pipelined kernel: SSIM + gradient (and gradient only), every input
// and gradient dtype but Float64.
//
// The streaming decomposition described at the top of this file, with the 5-row
// gradient halo (T = NT - 10); the CTA is split into two warp groups of NT
// threads that work on different steps at once:
//
//   group A (threads 0..NT-1):    cp.async loads (inputs, and the x/y values B2
//                                 needs), F1(t), B1(t-2)
//   group B (threads NT..2NT-1):  F2(t-1) + SSIM map + partials, B2(t-3)
//
// Every stage reads only what the other group wrote in the previous slot, so a
// single __syncthreads() per slot orders everything; the buffers passed between
// the groups are double-buffered by step parity.
//
// Group B keeps, per row, the last 10 columns of the F1 output and of the B1
// output in registers, as two 8-column blocks used in turn (its loop covers two
// slots per iteration, so only 2 carried columns are copied per slot).
// Unrolling further (5 slots, to index 40-column rings at compile time), or
// fusing F1 and B1 into one loop, was measured slower: the larger body misses
// the instruction cache.
// ---------------------------------------------------------------------------

template <int NT>
struct PGeo {
    static constexpr int S = 8;
    static constexpr int R1 = NT, T = NT - 2 * RAD, R2 = NT + 2 * RAD, LAG = 2 * RAD;
    static constexpr int SP = S + 1, FC = S + 1;
    static constexpr int NRUNB = (T + V - 1) / V;
    static constexpr int QROWS = NRUNB * V + 2 * RAD;
    static constexpr int LROWS = (R2 + NT - 1) / NT;
    static constexpr int LATENCY = 3;    // slots from F1(k) to B2(k)
    static constexpr int stage_one = R2 * SP * 8;
    static constexpr int f1_one = R1 * FC * 16;
    static constexpr int qmp_one = QROWS * FC * 16;
    static constexpr int b1_one = NT * FC * 16;
    static constexpr int xy_one = NT * SP * 8;
    static constexpr int red_bytes = (2 * NT / 32 + 2) * 8;
    static constexpr int off_stage = 0;
    static constexpr int off_f1 = off_stage + 2 * stage_one;
    static constexpr int off_qmp = off_f1 + 2 * f1_one;
    static constexpr int off_b1 = off_qmp + 2 * qmp_one;
    static constexpr int off_xy = off_b1 + 2 * b1_one;
    static constexpr int off_red = off_xy + 2 * xy_one;
    static constexpr int total = off_red + red_bytes;
    static_assert(R1 % V == 0 && NT % 32 == 0 && S * (R1 / V) == NT, "F1 items = one per thread");
    static_assert(S * NRUNB <= NT, "B1 items fit one round");
    static_assert(stage_one % 16 == 0 && xy_one % 16 == 0, "16-byte alignment of the buffers");
};

// IOM 0: Float32 inputs and gradient; inputs go to shared memory with cp.async.
// Otherwise (IOM = InMode) group A loads raw elements into registers one slot
// ahead, converts them (Float16 exactly, N0f8 as the correctly rounded raw/255)
// and stores them at the end of the slot; with IN_ANY the gradient is stored in
// its own dtype, the other modes write Float32.
template <int NT, bool WANT_SSIM, int IOM>
__global__ void __launch_bounds__(2 * NT, NT == 64 ? 3 : 2) pipe_kernel(const Params p)
{
    constexpr bool F32IO = IOM == 0;   // Float32 inputs and gradient (cp.async staging)
    using G = PGeo<NT>;
    constexpr int S = G::S, R1 = G::R1, T = G::T, R2 = G::R2, LAG = G::LAG;
    constexpr int SP = G::SP, FC = G::FC, NRUNB = G::NRUNB, QROWS = G::QROWS;

    extern __shared__ __align__(16) unsigned char smem_raw[];
    float2* stage = reinterpret_cast<float2*>(smem_raw + G::off_stage);
    float4* f1buf = reinterpret_cast<float4*>(smem_raw + G::off_f1);
    float4* qmp = reinterpret_cast<float4*>(smem_raw + G::off_qmp);
    float4* b1buf = reinterpret_cast<float4*>(smem_raw + G::off_b1);
    float2* xyb = reinterpret_cast<float2*>(smem_raw + G::off_xy);
    double* red = reinterpret_cast<double*>(smem_raw + G::off_red);
    constexpr int STG = R2 * SP, F1N = R1 * FC, QN = QROWS * FC, B1N = NT * FC, XYN = NT * SP;

    const int tid = threadIdx.x;
    const bool groupA = tid < NT;
    int64_t blk = blockIdx.x;
    const int c = static_cast<int>(blk % p.C);
    blk /= p.C;
    const int seg = static_cast<int>(blk % p.nseg);
    blk /= p.nseg;
    const int band = static_cast<int>(blk % p.nb);
    const int n = static_cast<int>(blk / p.nb);
    const int C = p.C, H = p.H, W = p.W;
    const int h0 = band * T;
    const int w0 = seg * p.L;
    const int wend = min(w0 + p.L, W);
    const int Lc = wend - w0;
    // In-image element offsets are 32-bit (the host guarantees C*H*W < 2^31), so
    // each address is one wide multiply-add from the image base.
    const int64_t ibase = static_cast<int64_t>(n) * p.img_elems + c;   // element index of (c, 0, 0, n)
    const float* __restrict__ xg = reinterpret_cast<const float*>(p.x) + ibase;   // (F32IO)
    const float* __restrict__ yg = reinterpret_cast<const float*>(p.y) + ibase;
    float* __restrict__ gg = reinterpret_cast<float*>(p.grad) + ibase;
    const uint32_t CH32 = static_cast<uint32_t>(C) * static_cast<uint32_t>(H);
    const int ns = (Lc + 2 * LAG - 1) / S + 1;
    const int nslot = (ns + G::LATENCY + 1) & ~1;   // even: group B runs two slots per iteration
    // +-1/N (or +-0.5/N), times the image's factor when one is given; doubled for inv2
    const float gscale2 =
        2.f * (p.img_scale ? static_cast<float>(p.gscale * ld_out(p.img_scale, p.isdt, n)) : p.gscale);

    float2 KP[RAD + 1];
#pragma unroll
    for (int i = 0; i <= RAD; ++i) KP[i] = make_float2(p.kh[i], p.kh[i]);
#define FSSIM_K2(tap) KP[(tap) <= RAD ? (tap) : 2 * RAD - (tap)]
#define FSSIM_K1(tap) p.kh[(tap) <= RAD ? (tap) : 2 * RAD - (tap)]

    // Zero the hand-off buffers once: the partial rows past R1 must read as zero,
    // and group B's first and last slots read these buffers before (after) the
    // stream has filled them.
    {
        float4* z4 = f1buf;
        const int n4 = (G::off_red - G::off_f1) / 16;   // f1buf, qmp, b1buf, xyb
        for (int e = tid; e < n4; e += 2 * NT) z4[e] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();
    double tsum = 0.0;

    if (groupA) {
        // ================= group A: loads, F1, B1 =================
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
        const bool xyrow_ok = ta < T && h0 + ta < H;
        const uint32_t xyrow_off = static_cast<uint32_t>(C) * static_cast<uint32_t>(xyrow_ok ? h0 + ta : 0);
        auto issue_stage = [&](int k, float2* buf) {   // stage <- input columns of step k
            const int cb = w0 - LAG + k * S;
#pragma unroll
            for (int j = 0; j < S; ++j) {
                const int wc = cb + j;
                const bool colok = static_cast<unsigned>(wc) < static_cast<unsigned>(W);
                const uint32_t coloff = CH32 * static_cast<uint32_t>(colok ? wc : 0);
#pragma unroll
                for (int r = 0; r < G::LROWS; ++r) {
                    const int i = ta + NT * r;
                    if (G::LROWS == 1 || i < R2) {
                        const uint32_t off = lrow_off[r] + coloff;
                        const bool ok = lrow_ok[r] && colok &&
                                        FSSIM_IN_BOUNDS(ibase + off, p.total_elems, SITE_PIPE_STAGE);
                        cp_async4(&buf[i * SP + j].x, xg + off, ok);
                        cp_async4(&buf[i * SP + j].y, yg + off, ok);
                    }
                }
            }
        };
        auto issue_xy = [&](int k, float2* buf) {      // xyb <- x, y at the gradient pixels of step k
            const int cb = w0 - LAG + k * S - 2 * RAD;
#pragma unroll
            for (int o = 0; o < S; ++o) {
                const int wc = cb + o;
                bool ok = xyrow_ok && static_cast<unsigned>(wc - w0) < static_cast<unsigned>(Lc);
                const uint32_t off = xyrow_off + CH32 * static_cast<uint32_t>(ok ? wc : 0);
                ok = ok && FSSIM_IN_BOUNDS(ibase + off, p.total_elems, SITE_PIPE_XY);
                cp_async4(&buf[ta * SP + o].x, xg + off, ok);
                cp_async4(&buf[ta * SP + o].y, yg + off, ok);
            }
        };

        // converting loaders: raw bits of step k (or of B2's pixels of step k) in
        // registers, converted and stored into shared memory by the store_* calls
        uint32_t rsx[F32IO ? 1 : G::LROWS * S], rsy[F32IO ? 1 : G::LROWS * S];
        uint32_t rxx[F32IO ? 1 : S], rxy[F32IO ? 1 : S];
        auto load_stage_raw = [&](int k) {
            const int cb = w0 - LAG + k * S;
#pragma unroll
            for (int j = 0; j < (F32IO ? 0 : S); ++j) {
                const int wc = cb + j;
                const bool colok = static_cast<unsigned>(wc) < static_cast<unsigned>(W);
#pragma unroll
                for (int r = 0; r < G::LROWS; ++r) {
                    const int64_t g = ibase + (lrow_off[r] + CH32 * static_cast<uint32_t>(colok ? wc : 0));
                    const bool ok = lrow_ok[r] && colok && FSSIM_IN_BOUNDS(g, p.total_elems, SITE_PIPE_STAGE_RAW);
                    rsx[r * S + j] = ok ? ld_in<IOM>(p.x, p.xdt, g) : 0u;
                    rsy[r * S + j] = ok ? ld_in<IOM>(p.y, p.ydt, g) : 0u;
                }
            }
        };
        auto store_stage_raw = [&](float2* buf) {
#pragma unroll
            for (int j = 0; j < (F32IO ? 0 : S); ++j) {
#pragma unroll
                for (int r = 0; r < G::LROWS; ++r) {
                    const int i = ta + NT * r;
                    if (G::LROWS == 1 || i < R2)
                        buf[i * SP + j] = make_float2(cvt_in<IOM>(rsx[r * S + j], p.xdt),
                                                      cvt_in<IOM>(rsy[r * S + j], p.ydt));
                }
            }
        };
        auto load_xy_raw = [&](int k) {
            const int cb = w0 - LAG + k * S - 2 * RAD;
#pragma unroll
            for (int o = 0; o < (F32IO ? 0 : S); ++o) {
                const int wc = cb + o;
                bool ok = xyrow_ok && static_cast<unsigned>(wc - w0) < static_cast<unsigned>(Lc);
                const int64_t g = ibase + (xyrow_off + CH32 * static_cast<uint32_t>(ok ? wc : 0));
                ok = ok && FSSIM_IN_BOUNDS(g, p.total_elems, SITE_PIPE_XY_RAW);
                rxx[o] = ok ? ld_in<IOM>(p.x, p.xdt, g) : 0u;
                rxy[o] = ok ? ld_in<IOM>(p.y, p.ydt, g) : 0u;
            }
        };
        auto store_xy_raw = [&](float2* buf) {
#pragma unroll
            for (int o = 0; o < (F32IO ? 0 : S); ++o)
                buf[ta * SP + o] = make_float2(cvt_in<IOM>(rxx[o], p.xdt), cvt_in<IOM>(rxy[o], p.ydt));
        };

        if (F32IO) {
            issue_stage(0, stage);
            cp_async_commit();
            cp_async_wait<0>();
        } else {
            load_stage_raw(0);
            store_stage_raw(stage);
        }
        __syncthreads();
#pragma unroll 1
        for (int t = 0; t < nslot; ++t) {
            const bool next_stage = t + 1 < ns;
            const bool next_xy = t >= 2 && t - 2 < ns;
            if (F32IO) {
                if (next_stage) issue_stage(t + 1, stage + ((t + 1) & 1) * STG);
                if (next_xy) issue_xy(t - 2, xyb + ((t + 1) & 1) * XYN);
                cp_async_commit();
            } else {
                if (next_stage) load_stage_raw(t + 1);
                if (next_xy) load_xy_raw(t - 2);
            }
            // -------- F1(t): h-direction pass of the 4 moment images --------
            if (t < ns) {
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
            // -------- B1(t-2): h-direction pass of the partials --------
            if (t >= 2 && t - 2 < ns && q1 < NRUNB) {
                const float4* qm = qmp + ((t - 2) & 1) * QN;
                float4* b1 = b1buf + ((t - 2) & 1) * B1N;
                float2 aQM[V];
                float aP[V];
#pragma unroll
                for (int o = 0; o < V; ++o) {
                    aQM[o] = make_float2(0.f, 0.f);
                    aP[o] = 0.f;
                }
#pragma unroll
                for (int i = 0; i < V + 2 * RAD; ++i) {
                    const float4 v = qm[(V * q1 + i) * FC + j1];
                    const float2 dqm = make_float2(v.x, v.y);
#pragma unroll
                    for (int o = 0; o < V; ++o) {
                        const int tap = i - o;
                        if (tap >= 0 && tap < TAPS) {
                            aQM[o] = __ffma2_rn(dqm, FSSIM_K2(tap), aQM[o]);
                            aP[o] = fmaf(v.z, FSSIM_K1(tap), aP[o]);
                        }
                    }
                }
#pragma unroll
                for (int o = 0; o < V; ++o)
                    b1[(V * q1 + o) * FC + j1] = make_float4(aQM[o].x, aQM[o].y, aP[o], 0.f);
            }
            if (F32IO) {
                cp_async_wait<0>();
            } else {
                if (next_stage) store_stage_raw(stage + ((t + 1) & 1) * STG);
                if (next_xy) store_xy_raw(xyb + ((t + 1) & 1) * XYN);
            }
            __syncthreads();
        }
    } else {
        // ================= group B: F2 + map, B2 =================
        const int tb = tid - NT;
        const int hr2 = h0 - LAG + RAD + tb;                 // image row of the F2 row
        const bool row_in = hr2 >= 0 && hr2 < H;
        const bool row_owned = row_in && tb >= RAD && tb < RAD + T;
        const bool grow_owned = tb < T && h0 + tb < H;
        const uint32_t grow_off = static_cast<uint32_t>(C) * static_cast<uint32_t>(grow_owned ? h0 + tb : 0);
        // Per-row histories as two S-column blocks used in turn: the block of step
        // k-1 ("prv"), and the block being filled by step k ("cur").  The window of
        // step k is [two saved columns of step k-2 | prv | cur]; after the step the
        // last two columns of prv are saved and the blocks swap roles.  The loop is
        // unrolled by two slots so the swap is a renaming, not a copy.
        static_assert(HIST == S + 2, "window = 2 saved columns + previous block + current block");
        float2 A0[S], A1[S], B0[S], B1[S], TA[2], TB[2];     // F1 output: (mx, my), (E[x^2+y^2], E[xy])
        float2 Q0[S], Q1[S], TQ[2];                         // B1 output: (2 dQ, dM)
        float P0[S], P1[S], TP[2];                          // B1 output: dP
#pragma unroll
        for (int m = 0; m < S; ++m) {
            A0[m] = A1[m] = B0[m] = B1[m] = Q0[m] = Q1[m] = make_float2(0.f, 0.f);
            P0[m] = P1[m] = 0.f;
        }
        TA[0] = TA[1] = TB[0] = TB[1] = TQ[0] = TQ[1] = make_float2(0.f, 0.f);
        TP[0] = TP[1] = 0.f;

        auto bslot = [&](int t, float2(&Acur)[S], float2(&Aprv)[S], float2(&Bcur)[S], float2(&Bprv)[S],
                         float2(&Qcur)[S], float2(&Qprv)[S], float(&Pcur)[S], float(&Pprv)[S]) {
            // Both stages run in every slot (so the history blocks are written
            // unconditionally and never held live twice); outside the stream they read
            // stale or zeroed buffers, and nothing they produce there is stored or owned.
            // -------- F2(t-1): w-direction pass, SSIM map, partials --------
            {
                const int k = t - 1;
                const float4* f1 = f1buf + (k & 1) * F1N;
                float4* qm = qmp + (k & 1) * QN;
                const int wcb = w0 - LAG + k * S - RAD;
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
                    // symmetric taps: k5 w5 + sum_t k_t (w_t + w_{10-t})
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
                    const float inv = rcp_approx(z * tt);
                    const float s = (ax * by) * inv;
                    const int wc = wcb + o;
                    if (WANT_SSIM) {
                        if (row_owned && static_cast<unsigned>(wc - w0) < static_cast<unsigned>(Lc)) ssum += s;
                    }
                    // dS/dQ = -s/t, dS/dM = 2/(zt) ((by-ax) my + s (z-t) mx), dS/dP = 2 ax/(zt)
                    // (src/core.jl:384-388), times +-1/N, zero outside the image, dQ doubled.
                    const bool in_img = row_in && static_cast<unsigned>(wc) < static_cast<unsigned>(W);
                    const float inv2 = in_img ? gscale2 * inv : 0.f;
                    const float dq2 = -(s * z) * inv2;
                    const float dm = inv2 * fmaf(by - ax, my, (s * (z - tt)) * mx);
                    const float dp = ax * inv2;
                    qm[tb * FC + o] = make_float4(dq2, dm, dp, 0.f);
                }
#undef FSSIM_WA
#undef FSSIM_WB
                if (WANT_SSIM) tsum += static_cast<double>(ssum);
                TA[0] = Aprv[S - 2];
                TA[1] = Aprv[S - 1];
                TB[0] = Bprv[S - 2];
                TB[1] = Bprv[S - 1];
            }
            // -------- B2(t-3): w-direction pass and the combine --------
            {
                const int k = t - G::LATENCY;
                const float4* b1 = b1buf + (k & 1) * B1N;
                const float2* xy = xyb + (t & 1) * XYN;
                const int wcg = w0 - LAG + k * S - 2 * RAD;
#define FSSIM_WQ(m) ((m) < 2 ? TQ[(m)] : ((m) < HIST ? Qprv[(m) - 2] : Qcur[(m) - HIST]))
#define FSSIM_WP(m) ((m) < 2 ? TP[(m)] : ((m) < HIST ? Pprv[(m) - 2] : Pcur[(m) - HIST]))
#pragma unroll
                for (int o = 0; o < S; ++o) {
                    {
                        const float4 v = b1[tb * FC + o];
                        Qcur[o] = make_float2(v.x, v.y);
                        Pcur[o] = v.z;
                    }
                    float2 a = __fmul2_rn(FSSIM_WQ(o + RAD), KP[RAD]);
                    float bp = FSSIM_WP(o + RAD) * p.kh[RAD];
#pragma unroll
                    for (int tap = 0; tap < RAD; ++tap) {
                        a = __ffma2_rn(__fadd2_rn(FSSIM_WQ(o + tap), FSSIM_WQ(o + 2 * RAD - tap)), KP[tap], a);
                        bp = fmaf(FSSIM_WP(o + tap) + FSSIM_WP(o + 2 * RAD - tap), p.kh[tap], bp);
                    }
                    const int wc = wcg + o;
                    const float2 v = xy[tb * SP + o];
                    // src/core.jl:773-782: (2 x K(dQ) + K(dM) + y K(dP)) * N_inv (N_inv folded upstream)
                    const float gv = fmaf(v.y, bp, fmaf(v.x, a.x, a.y));
                    if (grow_owned && static_cast<unsigned>(wc - w0) < static_cast<unsigned>(Lc)) {
                        const uint32_t off = grow_off + CH32 * static_cast<uint32_t>(wc);
                        if (FSSIM_IN_BOUNDS(ibase + off, p.total_elems, SITE_PIPE_GRAD)) {
                            if (IOM != IN_ANY) gg[off] = gv;
                            else st_grad(p.grad, p.gdt, ibase + off, gv);
                        }
                    }
                }
#undef FSSIM_WQ
#undef FSSIM_WP
                TQ[0] = Qprv[S - 2];
                TQ[1] = Qprv[S - 1];
                TP[0] = Pprv[S - 2];
                TP[1] = Pprv[S - 1];
            }
            __syncthreads();
        };

        __syncthreads();
#pragma unroll 1
        for (int t = 0; t < nslot; t += 2) {
            bslot(t, A0, A1, B0, B1, Q0, Q1, P0, P1);
            bslot(t + 1, A1, A0, B1, B0, Q1, Q0, P1, P0);
        }
    }
#undef FSSIM_K2
#undef FSSIM_K1

    if (WANT_SSIM) {
        const int local_cta = (band * p.nseg + seg) * p.C + c;
        finish_image<2 * NT>(p, n, local_cta, tsum, red);
    }
}

}  // namespace fssim

namespace fssim {

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
    int64_t blk = blockIdx.x;
    const int c = static_cast<int>(blk % p.C);
    blk /= p.C;
    const int seg = static_cast<int>(blk % p.nseg);
    blk /= p.nseg;
    const int band = static_cast<int>(blk % p.nb);
    const int n = static_cast<int>(blk / p.nb);
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
        auto issue_stage = [&](int k, float2* buf) {   // stage <- input columns of step k
            const int cb = w0 - LAG + k * S;
#pragma unroll
            for (int j = 0; j < S; ++j) {
                const int wc = cb + j;
                const bool colok = static_cast<unsigned>(wc) < static_cast<unsigned>(W);
                const uint32_t coloff = CH32 * static_cast<uint32_t>(colok ? wc : 0);
#pragma unroll
                for (int r = 0; r < G::LROWS; ++r) {
                    const int i = ta + NT * r;
                    if (G::LROWS == 1 || i < R2) {
                        const uint32_t off = lrow_off[r] + coloff;
                        const bool ok = lrow_ok[r] && colok &&
                                        FSSIM_IN_BOUNDS(ibase + off, p.total_elems, SITE_FPIPE_STAGE);
                        cp_async4(&buf[i * SP + j].x, xg + off, ok);
                        cp_async4(&buf[i * SP + j].y, yg + off, ok);
                    }
                }
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
        __syncthreads();
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
            __syncthreads();
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
            __syncthreads();
        };
        __syncthreads();
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

}  // namespace fssim

namespace fssim {

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
    static constexpr int NL = (NE + NT - 1) / NT;    // staged elements per thread
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
__global__ void __launch_bounds__(TGeo::NT, 3) tile_fwd_kernel(const Params p)
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
    auto tile_of = [&](int64_t t) {
        Tile u;
        u.c = static_cast<int>(t % C);
        t /= C;
        u.tw = static_cast<int>(t % p.nseg);
        t /= p.nseg;
        u.th = static_cast<int>(t % p.nb);
        u.n = static_cast<int>(t / p.nb);
        u.ibase = static_cast<int64_t>(u.n) * p.img_elems + u.c;
        return u;
    };
    // element e of a tile <-> stage row r = e % IR, column q = e / IR; zero outside the image;
    // all loads of the tile are issued before the first conversion
    auto load_convert = [&](int64_t t, float2* buf) {
        const Tile u = tile_of(t);
        uint32_t rx[G::NL], ry[G::NL];
#pragma unroll
        for (int k = 0; k < G::NL; ++k) {
            const int e = tid + G::NT * k;
            const int r = e % IR, q = e / IR;
            const int hr = u.th * TH - RAD + r, wc = u.tw * TW - RAD + q;
            bool ok = e < G::NE && hr >= 0 && hr < H && wc >= 0 && wc < W;
            const int64_t g = u.ibase + static_cast<int64_t>(C) * (ok ? hr : 0) + CH * (ok ? wc : 0);
            ok = ok && FSSIM_IN_BOUNDS(g, p.total_elems, SITE_TILE_LOAD);
            if (IM == 0) {
                rx[k] = ok ? __ldg(reinterpret_cast<const unsigned int*>(p.x) + g) : 0u;
                ry[k] = ok ? __ldg(reinterpret_cast<const unsigned int*>(p.y) + g) : 0u;
            } else {
                rx[k] = ok ? ld_in<IM>(p.x, p.xdt, g) : 0u;
                ry[k] = ok ? ld_in<IM>(p.y, p.ydt, g) : 0u;
            }
        }
#pragma unroll
        for (int k = 0; k < G::NL; ++k) {
            const int e = tid + G::NT * k;
            if (e < G::NE)
                buf[(e / IR) * RS + e % IR] =
                    IM == 0 ? make_float2(__uint_as_float(rx[k]), __uint_as_float(ry[k]))
                            : make_float2(cvt_in<IM>(rx[k], p.xdt), cvt_in<IM>(ry[k], p.ydt));
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
        load_convert(t, st);
        __syncthreads();   // the stage is complete; the previous tile's F2 is done with f1
        const Tile u = tile_of(t);

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

}  // namespace fssim

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

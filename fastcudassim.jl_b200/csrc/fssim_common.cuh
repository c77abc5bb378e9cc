// Fused SSIM / DSSIM kernels for sm_100a: shared definitions.
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
// fwd_pipe_kernel (its forward half, calls above 4 Mi elements, Float32 calls of several
// channels from 3 Mi), tile_fwd_kernel / tile_tma_kernel
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

#include <type_traits>

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
// for a memory-error tool): every global access first checks its element index
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

// Block index -> (channel, width segment, band, image) of the streaming kernels, whose
// grid is ordered channel fastest.  32-bit divisions: the host keeps grids below 2^31.
struct BandIndex {
    int c, seg, band, n;
};
__device__ __forceinline__ BandIndex band_index(const Params& p)
{
    const uint32_t b0 = blockIdx.x;
    const uint32_t q1 = b0 / static_cast<uint32_t>(p.C);
    const uint32_t q2 = q1 / static_cast<uint32_t>(p.nseg);
    const uint32_t q3 = q2 / static_cast<uint32_t>(p.nb);
    return BandIndex{static_cast<int>(b0 - q1 * static_cast<uint32_t>(p.C)),
                     static_cast<int>(q1 - q2 * static_cast<uint32_t>(p.nseg)),
                     static_cast<int>(q2 - q3 * static_cast<uint32_t>(p.nb)), static_cast<int>(q3)};
}

// Raw bits of one input element (zero-extended); converted at staging time so
// that the load's latency is not exposed at the point of issue.
__device__ __forceinline__ uint32_t ld_raw(const void* base, int dt, int64_t idx)
{
    if (dt == DT_F32) return __ldg(reinterpret_cast<const unsigned int*>(base) + idx);
    if (dt == DT_F16) return __ldg(reinterpret_cast<const unsigned short*>(base) + idx);
    return __ldg(reinterpret_cast<const unsigned char*>(base) + idx);
}

// N0f8 -> Float32: the correctly rounded value of raw/255.  1/255 is split into
// hi = fl(1/255) and lo = fl(1/255 - hi); fma(raw, hi, raw * lo) is within about
// 2^-47 (relative) of raw/255 before its single rounding, while raw/255 lies at
// least about 2^-32 (relative) from every rounding boundary, so the result is the
// correctly rounded quotient for every byte (checked exhaustively in exact rational
// arithmetic).  raw * fl(1/255) alone is off by one ulp for about half the bytes.
__device__ __forceinline__ float n0f8_to_f32(uint32_t r)
{
    const float hi = __uint_as_float(0x3b808081u);   // fl(1/255)
    const float lo = __uint_as_float(0xaf7efeffu);   // fl(1/255 - fl(1/255))
    const float fr = static_cast<float>(r & 255u);
    return fmaf(fr, hi, fr * lo);
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
// The same copy at a compile-time byte offset from a shared-memory address, with an
// explicit source size (4, or 0 to zero-fill without reading the source).
template <int DOFF>
__device__ __forceinline__ void cp_async4_at(unsigned sdst, const void* gsrc, int sz)
{
    asm volatile("cp.async.ca.shared.global [%0+%3], [%1], 4, %2;\n" ::"r"(sdst), "l"(gsrc), "r"(sz), "n"(DOFF)
                 : "memory");
}
__device__ __forceinline__ unsigned smem_addr(const void* p)
{
    return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
// f(std::integral_constant<int, I>) for I = B..E-1, where an offset must be a constant.
template <int B, int E, class F>
__device__ __forceinline__ void static_for(F&& f)
{
    if constexpr (B < E) {
        f(std::integral_constant<int, B>{});
        static_for<B + 1, E>(f);
    }
}
// Named barrier `id` over `nthreads` threads (bar.sync with an explicit count).  The
// two warp groups of the pipelined kernels reach their per-slot barrier from different
// code; a named barrier with a thread count is defined for that (every warp arrives as
// a whole), where __syncthreads() is only defined when all threads reach the same call.
// Barrier 0 stays with __syncthreads() in the block-wide code.
__device__ __forceinline__ void named_barrier_sync(int id, int nthreads)
{
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}
constexpr int BAR_SLOT = 1;   // the per-slot hand-off barrier of the two-group kernels

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

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
    // The condition is one shared-memory value read after the barrier, so it is the same
    // for every thread of the CTA: the barriers inside the branch are block-uniform.
    // No early return, so loops may call this.
    if (red[NT / 32] != 0.0) {
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

}  // namespace fssim

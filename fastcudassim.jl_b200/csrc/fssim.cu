// C ABI of libfastssim.so: argument checks, launch configuration and the single
// launch that replaces _ssim_fwd_bwd!'s device work (FastCUDASSIM.jl v0.2.1,
// src/core.jl:933-1107).  Declarations and the contract live in include/fastssim.h.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <map>
#include <mutex>

#include "fastssim.h"
#include "fssim_kernels.cuh"

namespace {

thread_local int g_status = FSSIM_OK;
thread_local char g_msg[512] = "";

int fail(int status, const char* fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof g_msg, fmt, ap);
    va_end(ap);
    g_status = status;
    return status;
}

int ok()
{
    g_status = FSSIM_OK;
    g_msg[0] = '\0';
    return FSSIM_OK;
}

}  // namespace

// Status and message of the calling thread, for the library's other translation unit
// (fssim_dist.cu); not part of the C ABI.
__attribute__((visibility("hidden"))) int fssim_host_fail(int status, const char* msg)
{
    return fail(status, "%s", msg);
}
__attribute__((visibility("hidden"))) int fssim_host_ok() { return ok(); }

namespace {

// Gaussian weights, sigma = 1.5, radius 5, evaluated like src/core.jl:40-46:
// Float32 exp(-0.5 (i/1.5)^2), normalised by their Float32 sum (left to right).
struct Weights {
    float k[fssim::TAPS];
    Weights()
    {
        const float sd = 1.5f;
        float raw[fssim::TAPS];
        float sum = 0.0f;
        for (int i = -fssim::RAD; i <= fssim::RAD; ++i) {
            const float r = static_cast<float>(i) / sd;
            raw[i + fssim::RAD] = static_cast<float>(std::exp(static_cast<double>(-0.5f * (r * r))));
        }
        for (int i = 0; i < fssim::TAPS; ++i) sum += raw[i];
        for (int i = 0; i < fssim::TAPS; ++i) k[i] = raw[i] / sum;
    }
};
const Weights& weights()
{
    static const Weights w;
    return w;
}

struct KInfo {
    const void* fn;
    int smem;
    int nt;        // band geometry parameter (rows of moments per band)
    int s;         // columns per streaming step
    int threads;   // CTA size
};

// Forward streaming kernel (Float32 inputs): band height NT (threads).
template <int NT>
KInfo kinfo()
{
    return KInfo{reinterpret_cast<const void*>(&fssim::band_kernel<NT>), fssim::Geo<NT>::total, NT,
                 fssim::Geo<NT>::S, NT};
}

// Forward two-group pipeline (images below 2^31 elements); IOM as pipe_kernel.
template <int NT, int IOM>
KInfo fpinfo()
{
    return KInfo{reinterpret_cast<const void*>(&fssim::fwd_pipe_kernel<NT, IOM>), fssim::FPGeo<NT>::total, NT,
                 fssim::FPGeo<NT>::S, 2 * NT};
}

template <int IOM>
KInfo fpinfo_nt(int nt)
{
    if (nt == 64) return fpinfo<64, IOM>();
    if (nt == 96) return fpinfo<96, IOM>();
    return fpinfo<128, IOM>();
}

template <int NT, bool WS, int IOM>
KInfo pinfo()
{
    return KInfo{reinterpret_cast<const void*>(&fssim::pipe_kernel<NT, WS, IOM>), fssim::PGeo<NT>::total, NT,
                 fssim::PGeo<NT>::S, 2 * NT};
}

template <int IOM>
KInfo pinfo_io(int nt, bool want_ssim)
{
    if (nt == 64) return want_ssim ? pinfo<64, true, IOM>() : pinfo<64, false, IOM>();
    return want_ssim ? pinfo<96, true, IOM>() : pinfo<96, false, IOM>();
}

template <int IM>
KInfo tinfo()
{
    return KInfo{reinterpret_cast<const void*>(&fssim::tile_fwd_kernel<IM>), fssim::TGeo::total, fssim::TGeo::TH,
                 fssim::TGeo::TW, fssim::TGeo::NT};
}

KInfo tile_tma_info()
{
    return KInfo{reinterpret_cast<const void*>(&fssim::tile_tma_kernel), fssim::TTGeo::total, fssim::TTGeo::TH,
                 fssim::TTGeo::TW, fssim::TTGeo::NT};
}

KInfo tile_info(bool f32io, int iom)
{
    if (f32io) return tinfo<0>();
    if (iom == fssim::IN_U8) return tinfo<fssim::IN_U8>();
    if (iom == fssim::IN_F16) return tinfo<fssim::IN_F16>();
    return tinfo<fssim::IN_ANY>();
}

// Forward-only calls up to 4 Mi elements run on the tile kernel: a streaming
// grid would need many short segments (halo warm-up, few warps per CTA).
// Float32 calls of several channels stream from 3 Mi elements on: measured with
// the L2 flushed, 16 x 3 x 256 x 256 and 3 x 720 x 1920 take 7-9 us less on the
// streaming kernel, while one-channel images (TMA tiles) and converted inputs
// keep the tiles up to 4 Mi.  Larger calls stream (fwd_pipe_kernel), except
// mixed input dtypes (decoded per element, the streaming loader would spill) and
// converted inputs in images of 2^31 elements or more, which only the tile
// kernel reads with 64-bit offsets.
constexpr int64_t kTileMaxElems = int64_t(1) << 22;
constexpr int64_t kTileMaxElemsF32Channels = int64_t(3) << 20;

bool use_tiles(int64_t c, int64_t h, int64_t w, int64_t n, bool f32io, int iom)
{
    if (f32io && c > 1 && c * h * w * n >= kTileMaxElemsF32Channels) return false;
    if (c * h * w * n <= kTileMaxElems) return true;
    return !f32io && (iom == fssim::IN_ANY || c * h * w >= (int64_t(1) << 31));
}

template <bool F, bool WS>
KInfo finfo()
{
    return KInfo{reinterpret_cast<const void*>(&fssim::f64_kernel<F, WS>), fssim::D64Geo::total, fssim::D64Geo::TO,
                 fssim::D64Geo::TO, fssim::D64Geo::NT};
}

// Gradients run the two-group pipelined kernel (32-bit in-image offsets: the
// caller guarantees C*H*W < 2^31); forward-only SSIM runs the two-group forward
// kernel, or tiles (see use_tiles), or for Float32 images of 2^31 elements or
// more the single-group streaming kernel.
KInfo kernel_info(int nt, bool fused, bool want_ssim, bool f32io, int iom, bool small_image)
{
    if (fused) {
        switch (f32io ? 0 : iom) {
            case 0: return pinfo_io<0>(nt, want_ssim);
            case fssim::IN_U8: return pinfo_io<fssim::IN_U8>(nt, want_ssim);
            case fssim::IN_F16: return pinfo_io<fssim::IN_F16>(nt, want_ssim);
            default: return pinfo_io<fssim::IN_ANY>(nt, want_ssim);
        }
    }
    if (small_image) {   // 32-bit in-image offsets; mixed dtypes run as tiles (see use_tiles)
        if (f32io) return fpinfo_nt<0>(nt);
        return iom == fssim::IN_U8 ? fpinfo_nt<fssim::IN_U8>(nt) : fpinfo_nt<fssim::IN_F16>(nt);
    }
    // images of 2^31 elements or more: Float32 only (converted inputs run as tiles)
    if (nt == 64) return kinfo<64>();
    if (nt == 96) return kinfo<96>();
    return kinfo<128>();
}

// Per-device facts, computed once per (device, kernel) under a lock.
struct DevInfo {
    int sms = 0;
    std::map<const void*, int> occ;   // resident CTAs per SM
};
std::mutex g_mu;
std::map<int, DevInfo> g_dev;

int device_facts(const KInfo& ki, int* sms, int* occ)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    std::lock_guard<std::mutex> lk(g_mu);
    DevInfo& d = g_dev[dev];
    if (d.sms == 0) {
        e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    }
    auto it = d.occ.find(ki.fn);
    if (it == d.occ.end()) {
        e = cudaFuncSetAttribute(ki.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, ki.smem);
        if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        int o = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, ki.fn, ki.threads, ki.smem);
        if (e != cudaSuccess)
            return fail(FSSIM_ERR_CUDA, "cudaOccupancyMaxActiveBlocksPerMultiprocessor: %s", cudaGetErrorString(e));
        if (o < 1) o = 1;
        it = d.occ.emplace(ki.fn, o).first;
    }
    *sms = d.sms;
    *occ = it->second;
    return FSSIM_OK;
}

// cuTensorMapEncodeTiled from the driver (through the runtime, so the library links no
// driver library); null where the driver does not provide it.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder()
{
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// The TMA view of one one-channel Float32 batch: dimensions (H, W, N), the tile kernel's
// 44 x 64 box.  The caller has checked that H is a multiple of 4 and the base is 16-byte
// aligned (the strides and the box start must be multiples of 16 bytes).
bool encode_tile_map(CUtensorMap* m, const void* base, int64_t h, int64_t w, int64_t n)
{
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(h), static_cast<cuuint64_t>(w), static_cast<cuuint64_t>(n)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(h) * 4u, static_cast<cuuint64_t>(h * w) * 4u};
    const cuuint32_t box[3] = {fssim::TTGeo::BR, fssim::TTGeo::IC, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct Cfg {
    bool fused = false, want_ssim = false;
    bool tma = false;   // tile kernel with TMA loads (tile_tma_kernel)
    int nt = 0, T = 0, nb = 0, nseg = 0, L = 0;
    int64_t cpi = 0, grid = 0;
    KInfo ki{};
    size_t ws_counters = 0, ws_bytes = 0;
};

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

constexpr int IOM_F64 = 4;   // configure(): compute in double precision

// Launch geometry: band height from {54, 86, 118} rows (gradient kernels) or
// {64, 96, 128} (forward only) to minimise padded rows, then the number of
// width segments that best fills the GPU (whole waves of resident CTAs
// versus the 10-20 warm-up columns each extra segment costs).
int configure(int64_t c, int64_t h, int64_t w, int64_t n, uint32_t flags, bool f32io, int iom, Cfg* cfg,
              bool tma_ok = false)
{
    Cfg g;
    g.fused = !(flags & FSSIM_SKIP_BACKWARD);
    g.want_ssim = !(flags & FSSIM_SKIP_SSIM);
    if (!g.fused && !g.want_ssim) {
        *cfg = g;
        return FSSIM_OK;
    }
    if (iom == IOM_F64) {   // double precision: one 16 x 16 tile per CTA
        g.ki = g.fused ? (g.want_ssim ? finfo<true, true>() : finfo<true, false>()) : finfo<false, true>();
        int sms = 0, occ = 0;
        int st = device_facts(g.ki, &sms, &occ);
        if (st != FSSIM_OK) return st;
        g.nt = fssim::D64Geo::TO;
        g.T = fssim::D64Geo::TO;
        g.nb = static_cast<int>(cdiv(h, fssim::D64Geo::TO));
        g.nseg = static_cast<int>(cdiv(w, fssim::D64Geo::TO));
        g.L = fssim::D64Geo::TO;
        g.cpi = c * g.nb * g.nseg;
        g.grid = n * g.cpi;
        g.ws_counters = ((static_cast<size_t>(n) * sizeof(unsigned) + 255) / 256) * 256;
        g.ws_bytes = g.want_ssim ? g.ws_counters + static_cast<size_t>(n) * g.cpi * sizeof(double) : 0;
        *cfg = g;
        return FSSIM_OK;
    }
    if (!g.fused && use_tiles(c, h, w, n, f32io, iom)) {   // small forward-only call: one TH x TW tile per CTA
        // one-channel Float32 images with a height divisible by 4 load their tiles with TMA
        // (tile rows shifted by TTGeo::SHIFT, so that every box starts 16-byte aligned)
        g.tma = tma_ok && f32io && c == 1 && h % 4 == 0;
        g.ki = g.tma ? tile_tma_info() : tile_info(f32io, iom);
        int sms = 0, occ = 0;
        int st = device_facts(g.ki, &sms, &occ);
        if (st != FSSIM_OK) return st;
        g.nt = fssim::TGeo::TH;
        g.T = fssim::TGeo::TH;
        g.nb = static_cast<int>(g.tma ? cdiv(h + fssim::TTGeo::SHIFT, fssim::TTGeo::TH) : cdiv(h, fssim::TGeo::TH));
        g.nseg = static_cast<int>(cdiv(w, fssim::TGeo::TW));
        g.L = fssim::TGeo::TW;
        g.cpi = c * g.nb * g.nseg;
        g.grid = n * g.cpi;   // one tile per CTA
        g.ws_counters = ((static_cast<size_t>(n) * sizeof(unsigned) + 255) / 256) * 256;
        g.ws_bytes = g.ws_counters + static_cast<size_t>(n) * g.cpi * sizeof(double);
        *cfg = g;
        return FSSIM_OK;
    }
    // Gradient kernels: bands of 54 or 86 rows; forward only: 64, 96 or 128 rows.
    const int cands_fused[2] = {64, 96};
    const int nfused = 2;
    const int cands_fwd[3] = {64, 96, 128};
    const int* cands = g.fused ? cands_fused : cands_fwd;
    const int ncand = g.fused ? nfused : 3;
    int64_t best = -1;
    for (int ci = 0; ci < ncand; ++ci) {
        const int nt = cands[ci];
        const int T = g.fused ? nt - 2 * fssim::RAD : nt;
        const int64_t nb = cdiv(h, T);
        const int64_t cost = g.fused ? nb * (4 * nt - 20) : nb * (2 * nt + 3);
        if (best < 0 || cost <= best) {
            best = cost;
            g.nt = nt;
            g.T = T;
            g.nb = static_cast<int>(nb);
        }
    }
    g.ki = kernel_info(g.nt, g.fused, g.want_ssim, f32io, iom, c * h * w < (int64_t(1) << 31));
    int sms = 0, occ = 0;
    int st = device_facts(g.ki, &sms, &occ);
    if (st != FSSIM_OK) return st;
    const int64_t slots = static_cast<int64_t>(sms) * occ;
    const int64_t base = n * c * g.nb;
    int64_t best_cost = -1;
    const int S = g.ki.s;
    const int lag2 = g.fused ? 4 * fssim::RAD : 2 * fssim::RAD;   // warm-up + drain columns
    const int64_t max_seg = std::max<int64_t>(1, cdiv(w, S));
    for (int64_t ns = 1; ns <= max_seg; ++ns) {
        const int64_t L = cdiv(cdiv(w, ns), S) * S;
        if (cdiv(w, L) != ns) continue;
        const int64_t steps = (L + lag2 - 1) / S + 1;
        const int64_t waves = cdiv(base * ns, slots);
        const int64_t cost = waves * steps;
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            g.nseg = static_cast<int>(ns);
            g.L = static_cast<int>(L);
        }
        if (base * ns > 8 * slots) break;   // further splits only add warm-up work
    }
    g.cpi = c * g.nb * g.nseg;
    g.grid = n * g.cpi;
    g.ws_counters = ((static_cast<size_t>(n) * sizeof(unsigned) + 255) / 256) * 256;
    g.ws_bytes = g.want_ssim ? g.ws_counters + static_cast<size_t>(n) * g.cpi * sizeof(double) : 0;
    *cfg = g;
    return FSSIM_OK;
}

bool is_input_dtype(int d)
{
    return d == FSSIM_FLOAT32 || d == FSSIM_FLOAT16 || d == FSSIM_N0F8 || d == FSSIM_FLOAT64;
}
bool is_float_dtype(int d) { return d == FSSIM_FLOAT32 || d == FSSIM_FLOAT16 || d == FSSIM_FLOAT64; }
size_t dsize(int d) { return d == FSSIM_FLOAT32 ? 4 : d == FSSIM_FLOAT16 ? 2 : d == FSSIM_N0F8 ? 1 : 8; }
bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
bool overlaps(const void* a, size_t an, const void* b, size_t bn)
{
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
    return a0 < b0 + bn && b0 < a0 + an;
}

int check_sizes(int64_t c, int64_t h, int64_t w, int64_t n)
{
    if (c < 1 || h < 1 || w < 1 || n < 1)
        return fail(FSSIM_ERR_INVALID_ARGUMENT, "sizes must be positive, got (c,h,w,n) = (%lld,%lld,%lld,%lld)",
                    (long long)c, (long long)h, (long long)w, (long long)n);
    const int64_t lim = (int64_t(1) << 31) - 1;
    if (c > lim || h > lim || w > lim || n > lim || c * h > lim || c * h * w > (int64_t(1) << 40) ||
        c * h * w > (int64_t(1) << 62) / n)   // the element count stays far inside int64
        return fail(FSSIM_ERR_INVALID_ARGUMENT, "sizes out of range (c,h,w,n) = (%lld,%lld,%lld,%lld)",
                    (long long)c, (long long)h, (long long)w, (long long)n);
    return FSSIM_OK;
}

}  // namespace

extern "C" {

#ifdef FSSIM_DEBUG_BOUNDS
const char* fssim_version(void) { return "fastssim 0.1.0 (abi 1, sm_100a, bounds-checked)"; }
#else
const char* fssim_version(void) { return "fastssim 0.1.0 (abi 1, sm_100a)"; }
#endif

int fssim_debug_bounds_status(unsigned* first_site, unsigned long long* count, int reset)
{
#ifdef FSSIM_DEBUG_BOUNDS
    if (!first_site || !count) return fail(FSSIM_ERR_INVALID_ARGUMENT, "first_site and count must not be NULL");
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(first_site, fssim::g_fssim_bounds_site, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(count, fssim::g_fssim_bounds_count, sizeof(unsigned long long));
    if (e == cudaSuccess && reset) {
        const unsigned z = 0u;
        const unsigned long long zz = 0ull;
        e = cudaMemcpyToSymbol(fssim::g_fssim_bounds_site, &z, sizeof(z));
        if (e == cudaSuccess) e = cudaMemcpyToSymbol(fssim::g_fssim_bounds_count, &zz, sizeof(zz));
    }
    if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, "bounds status: %s", cudaGetErrorString(e));
    return ok();
#else
    (void)first_site;
    (void)count;
    (void)reset;
    return fail(FSSIM_ERR_INVALID_ARGUMENT, "this library was built without FSSIM_DEBUG_BOUNDS");
#endif
}

int fssim_last_error(char* buf, size_t len)
{
    if (buf && len) {
        std::strncpy(buf, g_msg, len - 1);
        buf[len - 1] = '\0';
    }
    return g_status;
}

int fssim_workspace_size(int64_t c, int64_t h, int64_t w, int64_t n, uint32_t flags, size_t* bytes)
{
    if (!bytes) return fail(FSSIM_ERR_INVALID_ARGUMENT, "bytes is NULL");
    int st = check_sizes(c, h, w, n);
    if (st != FSSIM_OK) return st;
    // The launch geometry (and so the workspace) can differ between the
    // Float32 specialisation and the generic kernels: report the larger need.
    size_t most = 0;
    for (int v = 0; v <= IOM_F64; ++v) {
        Cfg g;
        st = configure(c, h, w, n, flags, v == 0, v == 0 ? fssim::IN_ANY : v, &g, v == 0);
        if (st != FSSIM_OK) return st;
        most = std::max(most, g.ws_bytes);
    }
    *bytes = most;
    return ok();
}

}  // extern "C"

namespace {

int fwd_bwd_impl(void* ssims, int ssims_dtype, int64_t ssims_len, void* dL_dimgs1, int grad_dtype,
                 const void* imgs1, int imgs1_dtype, const void* imgs2, int imgs2_dtype, void* qmp, int64_t c,
                 int64_t h, int64_t w, int64_t n, uint32_t flags, void* workspace, size_t workspace_bytes,
                 void* stream, const void* grad_scale, int grad_scale_dtype, bool clear_counters = false)
{
    (void)qmp;   // the partial gradients never leave the chip (see fastssim.h)
    const uint32_t known = FSSIM_SKIP_SSIM | FSSIM_SKIP_BACKWARD | FSSIM_USE_DSSIM | FSSIM_DIVIDE_BY_TWO |
                           FSSIM_SHOULD_ZERO;
    if (flags & ~known) return fail(FSSIM_ERR_INVALID_ARGUMENT, "unknown flag bits 0x%x", flags & ~known);
    int st = check_sizes(c, h, w, n);
    if (st != FSSIM_OK) return st;
    if (!imgs1 || !imgs2) return fail(FSSIM_ERR_INVALID_ARGUMENT, "imgs1 and imgs2 must not be NULL");
    if (!is_input_dtype(imgs1_dtype) || !is_input_dtype(imgs2_dtype))
        return fail(FSSIM_ERR_UNSUPPORTED_DTYPE, "image dtypes must be FLOAT32, FLOAT16, N0F8 or FLOAT64 (got %d, %d)",
                    imgs1_dtype, imgs2_dtype);
    if (!aligned(imgs1, dsize(imgs1_dtype)) || !aligned(imgs2, dsize(imgs2_dtype)))
        return fail(FSSIM_ERR_MISALIGNED, "image pointers must be aligned to their element size");
    const bool want_ssim = !(flags & FSSIM_SKIP_SSIM);
    const bool fused = !(flags & FSSIM_SKIP_BACKWARD);
    if (want_ssim) {
        if (!ssims) return fail(FSSIM_ERR_INVALID_ARGUMENT, "ssims must not be NULL unless FSSIM_SKIP_SSIM");
        if (!is_float_dtype(ssims_dtype))
            return fail(FSSIM_ERR_UNSUPPORTED_DTYPE, "ssims dtype must be FLOAT32, FLOAT64 or FLOAT16 (got %d)",
                        ssims_dtype);
        if (ssims_len != n)
            return fail(FSSIM_ERR_DIMENSION_MISMATCH,
                        "Expected the (d)ssims to be a vector of length the batch size %lld! Received length %lld.",
                        (long long)n, (long long)ssims_len);
        if (!aligned(ssims, dsize(ssims_dtype)))
            return fail(FSSIM_ERR_MISALIGNED, "ssims must be aligned to its element size");
    }
    if (fused) {
        if (!dL_dimgs1)
            return fail(FSSIM_ERR_INVALID_ARGUMENT, "dL_dimgs1 must not be NULL unless FSSIM_SKIP_BACKWARD");
        if (!is_float_dtype(grad_dtype))
            return fail(FSSIM_ERR_UNSUPPORTED_DTYPE, "gradient dtype must be FLOAT32, FLOAT16 or FLOAT64 (got %d)",
                        grad_dtype);
        if (!aligned(dL_dimgs1, dsize(grad_dtype)))
            return fail(FSSIM_ERR_MISALIGNED, "dL_dimgs1 must be aligned to its element size");
    }
    if (!want_ssim && !fused) return ok();   // nothing requested

    // The outputs must not share memory with the inputs: CTAs read input rows of
    // their neighbours' bands (the halo) after other CTAs have written outputs.
    // (The reference's separate backward launch tolerated dL_dimgs1 === imgs1;
    // the host layer copies an aliased input instead.)
    {
        const size_t elems = static_cast<size_t>(c * h * w * n);
        const size_t xb = elems * dsize(imgs1_dtype), yb = elems * dsize(imgs2_dtype);
        if (fused && (overlaps(dL_dimgs1, elems * dsize(grad_dtype), imgs1, xb) ||
                      overlaps(dL_dimgs1, elems * dsize(grad_dtype), imgs2, yb)))
            return fail(FSSIM_ERR_INVALID_ARGUMENT, "dL_dimgs1 overlaps imgs1 or imgs2; pass a copy of the input");
        if (want_ssim && (overlaps(ssims, static_cast<size_t>(n) * dsize(ssims_dtype), imgs1, xb) ||
                          overlaps(ssims, static_cast<size_t>(n) * dsize(ssims_dtype), imgs2, yb)))
            return fail(FSSIM_ERR_INVALID_ARGUMENT, "ssims overlaps imgs1 or imgs2");
        if (want_ssim && fused &&
            overlaps(ssims, static_cast<size_t>(n) * dsize(ssims_dtype), dL_dimgs1, elems * dsize(grad_dtype)))
            return fail(FSSIM_ERR_INVALID_ARGUMENT, "ssims overlaps dL_dimgs1");
    }

    if (fused && c * h * w >= (int64_t(1) << 31))
        return fail(FSSIM_ERR_INVALID_ARGUMENT, "gradient calls need C*H*W < 2^31 elements per image (got %lld)",
                    (long long)(c * h * w));
    const bool f32io = imgs1_dtype == FSSIM_FLOAT32 && imgs2_dtype == FSSIM_FLOAT32 &&
                       (!fused || grad_dtype == FSSIM_FLOAT32);
    const bool f32grad = !fused || grad_dtype == FSSIM_FLOAT32;
    const int iom = (imgs1_dtype == FSSIM_N0F8 && imgs2_dtype == FSSIM_N0F8 && f32grad)        ? fssim::IN_U8
                    : (imgs1_dtype == FSSIM_FLOAT16 && imgs2_dtype == FSSIM_FLOAT16 && f32grad) ? fssim::IN_F16
                                                                                             : fssim::IN_ANY;
    // Float64 on either input: compute in double (promote_type(T1, T2, Float32), src/core.jl:953-954)
    const bool f64 = imgs1_dtype == FSSIM_FLOAT64 || imgs2_dtype == FSSIM_FLOAT64;
    Cfg g;
    const bool tma_ok = aligned(imgs1, 16) && aligned(imgs2, 16);
    st = configure(c, h, w, n, flags, f32io && !f64, f64 ? IOM_F64 : iom, &g, tma_ok);
    if (st != FSSIM_OK) return st;
    CUtensorMap tmx, tmy;
    if (g.tma && !(encode_tile_map(&tmx, imgs1, h, w, n) && encode_tile_map(&tmy, imgs2, h, w, n))) {
        st = configure(c, h, w, n, flags, f32io && !f64, f64 ? IOM_F64 : iom, &g, false);   // plain tile loads
        if (st != FSSIM_OK) return st;
    }
    if (want_ssim) {
        if (!workspace || workspace_bytes < g.ws_bytes)
            return fail(FSSIM_ERR_WORKSPACE, "workspace of %zu bytes required, got %zu", g.ws_bytes,
                        workspace ? workspace_bytes : (size_t)0);
        if (!aligned(workspace, 256)) return fail(FSSIM_ERR_MISALIGNED, "workspace must be 256-byte aligned");
    }

    if (g.grid > (int64_t(1) << 31) - 1)
        return fail(FSSIM_ERR_INVALID_ARGUMENT, "%lld thread blocks needed, more than one launch allows; split the batch",
                    (long long)g.grid);

    fssim::Params p{};
    p.x = imgs1;
    p.y = imgs2;
    p.grad = fused ? dL_dimgs1 : nullptr;
    p.ssims = want_ssim ? ssims : nullptr;
    p.counters = want_ssim ? static_cast<unsigned*>(workspace) : nullptr;
    p.partials = want_ssim ? reinterpret_cast<double*>(static_cast<char*>(workspace) + g.ws_counters) : nullptr;
    p.img_elems = c * h * w;
    p.total_elems = c * h * w * n;
    p.C = static_cast<int>(c);
    p.H = static_cast<int>(h);
    p.W = static_cast<int>(w);
    p.N = static_cast<int>(n);
    p.nb = g.nb;
    p.nseg = g.nseg;
    p.L = g.L;
    p.cpi = static_cast<int>(g.cpi);
    p.xdt = imgs1_dtype;
    p.ydt = imgs2_dtype;
    p.gdt = grad_dtype;
    p.sdt = ssims_dtype;
    p.should_zero = (flags & FSSIM_SHOULD_ZERO) ? 1 : 0;
    p.use_dssim = (flags & FSSIM_USE_DSSIM) ? 1 : 0;
    p.div2 = (flags & FSSIM_DIVIDE_BY_TWO) ? 1 : 0;
    for (int i = 0; i <= fssim::RAD; ++i) p.kh[i] = weights().k[i];
    p.C1 = 0.01f * 0.01f;
    p.C2 = 0.03f * 0.03f;
    p.npx = static_cast<double>(c * h * w);
    // src/core.jl:584-589: N_inv = 1/N, or 0.5/N for DSSIM with divide_by_two; the
    // DSSIM sign (src/core.jl:648) is folded in here.
    const double scale = ((p.use_dssim && p.div2) ? 0.5 : 1.0) / p.npx;
    p.gscale = static_cast<float>(p.use_dssim ? -scale : scale);
    p.img_scale = grad_scale;
    p.isdt = grad_scale_dtype;

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (clear_counters && want_ssim) {
        // Allocation-free entry point: its shared scratch may hold counters that a call
        // which failed part-way left set.  Cleared only now, after every check has
        // passed, so a rejected call never touches the scratch.
        cudaError_t ce = cudaMemsetAsync(workspace, 0, g.ws_counters, s);
        if (ce != cudaSuccess) return fail(FSSIM_ERR_CUDA, "cudaMemsetAsync(scratch): %s", cudaGetErrorString(ce));
    }
    void* args[] = {&p, &tmx, &tmy};   // the tensor maps only for the TMA tile kernel
    cudaError_t e = cudaLaunchKernel(g.ki.fn, dim3(static_cast<unsigned>(g.grid)), dim3(g.ki.threads), args, g.ki.smem, s);
    if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(e));
    return ok();
}

}  // namespace

extern "C" {

int fssim_fwd_bwd(void* ssims, int ssims_dtype, int64_t ssims_len, void* dL_dimgs1, int grad_dtype,
                  const void* imgs1, int imgs1_dtype, const void* imgs2, int imgs2_dtype, void* qmp,
                  int64_t c, int64_t h, int64_t w, int64_t n, uint32_t flags, void* workspace,
                  size_t workspace_bytes, void* stream)
{
    return fwd_bwd_impl(ssims, ssims_dtype, ssims_len, dL_dimgs1, grad_dtype, imgs1, imgs1_dtype, imgs2,
                        imgs2_dtype, qmp, c, h, w, n, flags, workspace, workspace_bytes, stream, nullptr, 0);
}

int fssim_fwd_bwd_scaled(void* ssims, int ssims_dtype, int64_t ssims_len, void* dL_dimgs1, int grad_dtype,
                         const void* imgs1, int imgs1_dtype, const void* imgs2, int imgs2_dtype, int64_t c,
                         int64_t h, int64_t w, int64_t n, uint32_t flags, const void* grad_scale,
                         int grad_scale_dtype, void* workspace, size_t workspace_bytes, void* stream)
{
    if (!grad_scale) return fail(FSSIM_ERR_INVALID_ARGUMENT, "grad_scale must not be NULL");
    if (!is_float_dtype(grad_scale_dtype))
        return fail(FSSIM_ERR_UNSUPPORTED_DTYPE, "grad_scale dtype must be FLOAT32, FLOAT64 or FLOAT16 (got %d)",
                    grad_scale_dtype);
    if (!aligned(grad_scale, dsize(grad_scale_dtype)))
        return fail(FSSIM_ERR_MISALIGNED, "grad_scale must be aligned to its element size");
    return fwd_bwd_impl(ssims, ssims_dtype, ssims_len, dL_dimgs1, grad_dtype, imgs1, imgs1_dtype, imgs2,
                        imgs2_dtype, nullptr, c, h, w, n, flags, workspace, workspace_bytes, stream, grad_scale,
                        grad_scale_dtype);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free entry point.  The reduction scratch lives in this array,
// compiled into the library; host code must not pass the array's name to a
// kernel (on the host it only stands for the symbol), so each device's address
// is looked up once with cudaGetSymbolAddress while that device is current.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_fssim_scratch[FSSIM_NOALLOC_SCRATCH_BYTES];

namespace {

std::mutex g_scratch_mu;
std::map<int, void*> g_scratch_addr;

int scratch_address(void** out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    auto it = g_scratch_addr.find(dev);
    if (it == g_scratch_addr.end()) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_fssim_scratch);
        if (e != cudaSuccess || ptr == nullptr)
            return fail(FSSIM_ERR_CUDA, "cudaGetSymbolAddress(scratch) on device %d: %s", dev,
                        cudaGetErrorString(e));
        it = g_scratch_addr.emplace(dev, ptr).first;
    }
    *out = it->second;
    return FSSIM_OK;
}

}  // namespace

extern "C" int fssim_fwd_bwd_noalloc(void* ssims, int ssims_dtype, int64_t ssims_len, void* dL_dimgs1,
                                     int grad_dtype, const void* imgs1, int imgs1_dtype, const void* imgs2,
                                     int imgs2_dtype, int64_t c, int64_t h, int64_t w, int64_t n,
                                     uint32_t flags, void* stream)
{
    size_t need = 0;
    int st = fssim_workspace_size(c, h, w, n, flags, &need);
    if (st != FSSIM_OK) return st;
    if (need > FSSIM_NOALLOC_SCRATCH_BYTES)
        return fail(FSSIM_ERR_WORKSPACE,
                    "fssim_fwd_bwd_noalloc: these sizes need %zu bytes of reduction scratch, the built-in "
                    "scratch holds %u; call fssim_fwd_bwd with a caller-provided workspace instead",
                    need, (unsigned)FSSIM_NOALLOC_SCRATCH_BYTES);
    // The scratch used is the current device's: the stream must belong to that device too
    // (the legacy and per-thread default streams always do).
    const uintptr_t sv = reinterpret_cast<uintptr_t>(stream);
    if (sv > 2) {
        int cur = 0, sdev = 0;
        cudaError_t e = cudaGetDevice(&cur);
        if (e == cudaSuccess) e = cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev);
        if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, "stream device query: %s", cudaGetErrorString(e));
        if (sdev != cur)
            return fail(FSSIM_ERR_INVALID_ARGUMENT,
                        "fssim_fwd_bwd_noalloc: the stream belongs to device %d but device %d is current; "
                        "make the device of the buffers and the stream current", sdev, cur);
    }
    void* ws = nullptr;
    st = scratch_address(&ws);
    if (st != FSSIM_OK) return st;
    // fwd_bwd_impl clears the scratch counters on `stream` once all its argument checks
    // have passed, just before the launch.
    return fwd_bwd_impl(ssims, ssims_dtype, ssims_len, dL_dimgs1, grad_dtype, imgs1, imgs1_dtype, imgs2,
                        imgs2_dtype, nullptr, c, h, w, n, flags, ws, FSSIM_NOALLOC_SCRATCH_BYTES, stream, nullptr,
                        0, /*clear_counters=*/true);
}

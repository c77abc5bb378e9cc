// Multi-GPU entry points of libfastssim.so (host code only): a batch split into
// contiguous shards, one process per GPU, and the all-gather of the per-image
// (D)SSIM values over NCCL, with bounded waits and communicator abort.
//
// Images are independent (FastCUDASSIM.jl src/core.jl:186: one image per loop
// iteration), so the only exchange is the vector of per-image scores; each rank's
// gradient slice stays on its own GPU.  NCCL is loaded at run time (libnccl.so.2):
// the library links only the CUDA runtime, and a caller that already holds NCCL
// (NCCL.jl, torch) shares its copy, so a communicator created there can be passed in.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>   // types, enums and NCCL_CONFIG_INITIALIZER; the functions come from dlsym

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <thread>

#include "fastssim.h"

int fssim_host_fail(int status, const char* msg);
int fssim_host_ok();

namespace {

struct NcclApi {
    void* lib = nullptr;
    ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*commInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*commFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
    const char* (*getErrorString)(ncclResult_t) = nullptr;
    bool complete() const
    {
        return getUniqueId && commInitRankConfig && allGather && commGetAsyncError && commFinalize && commDestroy &&
               commAbort && getErrorString;
    }
};

const NcclApi& nccl()
{
    static const NcclApi api = [] {
        NcclApi a;
        a.lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!a.lib) a.lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!a.lib) return a;
        a.getUniqueId = reinterpret_cast<decltype(a.getUniqueId)>(dlsym(a.lib, "ncclGetUniqueId"));
        a.commInitRankConfig = reinterpret_cast<decltype(a.commInitRankConfig)>(dlsym(a.lib, "ncclCommInitRankConfig"));
        a.allGather = reinterpret_cast<decltype(a.allGather)>(dlsym(a.lib, "ncclAllGather"));
        a.commGetAsyncError = reinterpret_cast<decltype(a.commGetAsyncError)>(dlsym(a.lib, "ncclCommGetAsyncError"));
        a.commFinalize = reinterpret_cast<decltype(a.commFinalize)>(dlsym(a.lib, "ncclCommFinalize"));
        a.commDestroy = reinterpret_cast<decltype(a.commDestroy)>(dlsym(a.lib, "ncclCommDestroy"));
        a.commAbort = reinterpret_cast<decltype(a.commAbort)>(dlsym(a.lib, "ncclCommAbort"));
        a.getErrorString = reinterpret_cast<decltype(a.getErrorString)>(dlsym(a.lib, "ncclGetErrorString"));
        return a;
    }();
    return api;
}

int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int status, const char* fmt, ...)
{
    char buf[480];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return fssim_host_fail(status, buf);
}

int need_nccl()
{
    if (!nccl().complete())
        return fail(FSSIM_ERR_COMM, "NCCL is not available: libnccl.so.2 (2.14 or later) could not be loaded");
    return FSSIM_OK;
}

using Clock = std::chrono::steady_clock;

// Waits while the communicator reports ncclInProgress (a non-blocking communicator still
// initialising or enqueuing), up to `deadline`.  Any other error aborts the communicator.
int settle(ncclComm_t comm, Clock::time_point deadline, const char* what)
{
    for (;;) {
        ncclResult_t r = ncclSuccess;
        const ncclResult_t q = nccl().commGetAsyncError(comm, &r);
        if (q != ncclSuccess) r = q;
        if (r == ncclSuccess) return FSSIM_OK;
        if (r != ncclInProgress) {
            nccl().commAbort(comm);
            return fail(FSSIM_ERR_COMM, "%s: %s (communicator aborted)", what, nccl().getErrorString(r));
        }
        if (Clock::now() > deadline) {
            nccl().commAbort(comm);
            return fail(FSSIM_ERR_TIMEOUT, "%s: still in progress at the deadline (communicator aborted)", what);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

Clock::time_point after(double seconds)
{
    return Clock::now() + std::chrono::duration_cast<Clock::duration>(std::chrono::duration<double>(seconds));
}

size_t esize(int dt) { return dt == FSSIM_FLOAT64 ? 8 : dt == FSSIM_FLOAT16 ? 2 : 4; }
size_t up256(size_t b) { return (b + 255) / 256 * 256; }

// The contiguous shard of `rank`: the first n % world ranks hold one image more.
void shard(int64_t n, int world, int rank, int64_t* lo, int64_t* cnt)
{
    const int64_t base = n / world, rem = n % world;
    *lo = rank * base + (rank < rem ? rank : rem);
    *cnt = base + (rank < rem ? 1 : 0);
}

int check_shard_args(int64_t n_total, int world, int rank, int64_t n_local, int ssims_dtype)
{
    if (world < 1 || rank < 0 || rank >= world)
        return fail(FSSIM_ERR_INVALID_ARGUMENT, "rank %d of world %d is out of range", rank, world);
    if (n_total < 1) return fail(FSSIM_ERR_INVALID_ARGUMENT, "n_total must be positive (got %lld)", (long long)n_total);
    int64_t lo = 0, cnt = 0;
    shard(n_total, world, rank, &lo, &cnt);
    if (n_local != cnt)
        return fail(FSSIM_ERR_DIMENSION_MISMATCH,
                    "rank %d of %d holds images [%lld, %lld) of %lld: expected a shard of %lld images, got %lld", rank,
                    world, (long long)lo, (long long)(lo + cnt), (long long)n_total, (long long)cnt,
                    (long long)n_local);
    if (ssims_dtype != FSSIM_FLOAT32 && ssims_dtype != FSSIM_FLOAT16 && ssims_dtype != FSSIM_FLOAT64)
        return fail(FSSIM_ERR_UNSUPPORTED_DTYPE, "ssims dtype must be FLOAT32, FLOAT16 or FLOAT64 (got %d)", ssims_dtype);
    return FSSIM_OK;
}

ncclDataType_t nccl_type(int dt)
{
    return dt == FSSIM_FLOAT64 ? ncclFloat64 : dt == FSSIM_FLOAT16 ? ncclFloat16 : ncclFloat32;
}

}  // namespace

extern "C" {

int fssim_comm_unique_id(unsigned char id[128])
{
    if (!id) return fail(FSSIM_ERR_INVALID_ARGUMENT, "id must not be NULL");
    int st = need_nccl();
    if (st != FSSIM_OK) return st;
    ncclUniqueId u;
    const ncclResult_t r = nccl().getUniqueId(&u);
    if (r != ncclSuccess) return fail(FSSIM_ERR_COMM, "ncclGetUniqueId: %s", nccl().getErrorString(r));
    static_assert(sizeof(u.internal) == 128, "NCCL unique id of 128 bytes");
    std::memcpy(id, u.internal, 128);
    return fssim_host_ok();
}

int fssim_comm_init(void** comm, int world, int rank, const unsigned char id[128], double deadline_s)
{
    if (!comm || !id) return fail(FSSIM_ERR_INVALID_ARGUMENT, "comm and id must not be NULL");
    if (world < 1 || rank < 0 || rank >= world)
        return fail(FSSIM_ERR_INVALID_ARGUMENT, "rank %d of world %d is out of range", rank, world);
    int st = need_nccl();
    if (st != FSSIM_OK) return st;
    ncclUniqueId u;
    std::memcpy(u.internal, id, 128);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;   // the join is polled against the deadline below
    ncclComm_t c = nullptr;
    const ncclResult_t r = nccl().commInitRankConfig(&c, world, u, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress)
        return fail(FSSIM_ERR_COMM, "ncclCommInitRankConfig: %s", nccl().getErrorString(r));
    st = settle(c, after(deadline_s), "communicator initialisation (a rank did not join?)");
    if (st != FSSIM_OK) return st;
    *comm = c;
    return fssim_host_ok();
}

int fssim_comm_destroy(void* comm, int abort_it)
{
    if (!comm) return fail(FSSIM_ERR_INVALID_ARGUMENT, "comm must not be NULL");
    int st = need_nccl();
    if (st != FSSIM_OK) return st;
    ncclComm_t c = static_cast<ncclComm_t>(comm);
    if (!abort_it) {
        ncclResult_t r = nccl().commFinalize(c);
        if (r == ncclSuccess || r == ncclInProgress) {
            st = settle(c, after(10.0), "communicator finalisation");   // aborts on failure
            if (st != FSSIM_OK) return st;
            r = nccl().commDestroy(c);
            if (r != ncclSuccess) return fail(FSSIM_ERR_COMM, "ncclCommDestroy: %s", nccl().getErrorString(r));
            return fssim_host_ok();
        }
    }
    const ncclResult_t r = nccl().commAbort(c);
    if (r != ncclSuccess) return fail(FSSIM_ERR_COMM, "ncclCommAbort: %s", nccl().getErrorString(r));
    return fssim_host_ok();
}

int fssim_sharded_workspace_size(int64_t c, int64_t h, int64_t w, int64_t n_total, int world, int rank,
                                 uint32_t flags, int ssims_dtype, size_t* bytes)
{
    if (!bytes) return fail(FSSIM_ERR_INVALID_ARGUMENT, "bytes is NULL");
    int64_t lo = 0, cnt = 0;
    if (world < 1 || rank < 0 || rank >= world || n_total < 1)
        return fail(FSSIM_ERR_INVALID_ARGUMENT, "rank %d of world %d with %lld images is out of range", rank, world,
                    (long long)n_total);
    shard(n_total, world, rank, &lo, &cnt);
    int st = check_shard_args(n_total, world, rank, cnt, ssims_dtype);
    if (st != FSSIM_OK) return st;
    size_t local = 0;
    if (cnt > 0) {
        st = fssim_workspace_size(c, h, w, cnt, flags, &local);
        if (st != FSSIM_OK) return st;
    }
    const int64_t per = (n_total + world - 1) / world;
    size_t total = up256(local);
    if (per * world != n_total && !(flags & FSSIM_SKIP_SSIM))   // padded send and receive buffers
        total += up256(per * esize(ssims_dtype)) + up256(per * world * esize(ssims_dtype));
    *bytes = total;
    return fssim_host_ok();
}

int fssim_fwd_bwd_sharded(void* all_ssims, int ssims_dtype, int64_t n_total, void* dL_dimgs1, int grad_dtype,
                          const void* imgs1, int imgs1_dtype, const void* imgs2, int imgs2_dtype, int64_t c,
                          int64_t h, int64_t w, int64_t n_local, uint32_t flags, void* comm, int world, int rank,
                          void* workspace, size_t workspace_bytes, void* stream)
{
    int st = check_shard_args(n_total, world, rank, n_local, ssims_dtype);
    if (st != FSSIM_OK) return st;
    const bool want = !(flags & FSSIM_SKIP_SSIM);
    if (want && !all_ssims) return fail(FSSIM_ERR_INVALID_ARGUMENT, "all_ssims must not be NULL unless FSSIM_SKIP_SSIM");
    if (want && world > 1) {
        if (!comm) return fail(FSSIM_ERR_INVALID_ARGUMENT, "comm must not be NULL for a world of more than one rank");
        st = need_nccl();
        if (st != FSSIM_OK) return st;
    }
    size_t need = 0;
    st = fssim_sharded_workspace_size(c, h, w, n_total, world, rank, flags, ssims_dtype, &need);
    if (st != FSSIM_OK) return st;
    if (need > 0 && (!workspace || workspace_bytes < need))
        return fail(FSSIM_ERR_WORKSPACE, "workspace of %zu bytes required, got %zu", need,
                    workspace ? workspace_bytes : (size_t)0);
    size_t local = 0;
    if (n_local > 0) {
        st = fssim_workspace_size(c, h, w, n_local, flags, &local);
        if (st != FSSIM_OK) return st;
    }
    const size_t es = esize(ssims_dtype);
    const int64_t per = (n_total + world - 1) / world;
    const bool equal = per * world == n_total;
    int64_t lo = 0, cnt = 0;
    shard(n_total, world, rank, &lo, &cnt);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    unsigned char* send = ws ? ws + up256(local) : nullptr;
    unsigned char* recv = send ? send + up256(per * es) : nullptr;
    // The shard's values go straight to their place in the output when shards are equal
    // (the all-gather then runs in place), else to the padded send buffer.
    unsigned char* vals = want ? (equal ? static_cast<unsigned char*>(all_ssims) + lo * es : send) : nullptr;
    if (want && !equal && !(flags & FSSIM_SHOULD_ZERO) && n_local > 0) {   // accumulate onto the previous values
        const cudaError_t e = cudaMemcpyAsync(vals, static_cast<unsigned char*>(all_ssims) + lo * es, n_local * es,
                                              cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, "cudaMemcpyAsync: %s", cudaGetErrorString(e));
    }
    if (n_local > 0) {
        st = fssim_fwd_bwd(vals, ssims_dtype, want ? n_local : 0, dL_dimgs1, grad_dtype, imgs1, imgs1_dtype, imgs2,
                           imgs2_dtype, nullptr, c, h, w, n_local, flags, ws, local, stream);
        if (st != FSSIM_OK) return st;
    }
    if (!want || world == 1) return fssim_host_ok();
    ncclComm_t cm = static_cast<ncclComm_t>(comm);
    const ncclResult_t r = nccl().allGather(equal ? vals : send, equal ? all_ssims : recv, static_cast<size_t>(per),
                                            nccl_type(ssims_dtype), cm, s);
    if (r != ncclSuccess && r != ncclInProgress) {
        nccl().commAbort(cm);
        return fail(FSSIM_ERR_COMM, "ncclAllGather: %s (communicator aborted)", nccl().getErrorString(r));
    }
    st = settle(cm, after(30.0), "ncclAllGather enqueue");
    if (st != FSSIM_OK) return st;
    if (!equal) {   // drop the padding: rank q's values to [lo_q, lo_q + cnt_q)
        for (int q = 0; q < world; ++q) {
            int64_t lq = 0, cq = 0;
            shard(n_total, world, q, &lq, &cq);
            if (cq == 0) continue;
            const cudaError_t e = cudaMemcpyAsync(static_cast<unsigned char*>(all_ssims) + lq * es, recv + q * per * es,
                                                  cq * es, cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, "cudaMemcpyAsync: %s", cudaGetErrorString(e));
        }
    }
    return fssim_host_ok();
}

int fssim_comm_wait(void* comm, void* stream, double deadline_s)
{
    const Clock::time_point end = after(deadline_s);
    ncclComm_t cm = static_cast<ncclComm_t>(comm);
    if (cm) {
        int st = need_nccl();
        if (st != FSSIM_OK) return st;
    }
    for (;;) {
        const cudaError_t e = cudaStreamQuery(static_cast<cudaStream_t>(stream));
        if (e == cudaSuccess) return fssim_host_ok();
        if (e != cudaErrorNotReady) return fail(FSSIM_ERR_CUDA, "cudaStreamQuery: %s", cudaGetErrorString(e));
        if (cm) {
            ncclResult_t r = ncclSuccess;
            const ncclResult_t q = nccl().commGetAsyncError(cm, &r);
            if (q != ncclSuccess) r = q;
            if (r != ncclSuccess && r != ncclInProgress) {
                nccl().commAbort(cm);
                return fail(FSSIM_ERR_COMM, "communicator error: %s (communicator aborted)", nccl().getErrorString(r));
            }
        }
        if (Clock::now() > end) {
            if (cm) nccl().commAbort(cm);
            return fail(FSSIM_ERR_TIMEOUT, "the stream's work did not finish within %g s%s", deadline_s,
                        cm ? " (communicator aborted)" : "");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

}  // extern "C"

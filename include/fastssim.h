/*
 * fastssim.h - C ABI of the B200 (sm_100a) SSIM / DSSIM engine.
 *
 * One shared library, libfastssim.so, replaces the two CUDA.jl kernels of
 * FastCUDASSIM.jl v0.2.1 and their launch sites.  Every exported Julia function
 * of that package (src/interface.jl:31-338) funnels into
 *
 *     _ssim_fwd_bwd!(ssims, dL_dimgs1, imgs1, imgs2, N_dssims_dQMP, should_zero,
 *                    Val(skip_ssim), Val(skip_backward), use_dssim, divide_by_two)
 *                                                      (src/core.jl:933-1107)
 *
 * and fssim_fwd_bwd() below is the device-side half of that function: the Julia
 * side keeps canonicalisation, DimensionMismatch errors, allocation and the
 * scalar unpack (src/conversions.jl), and calls this entry point where the
 * reference issued its @cuda launches (src/core.jl:996, :1059) and its
 * broadcast divide (src/core.jl:1033).
 *
 * Conventions shared by all entry points
 *  - Image batches are canonical (C, H, W, N) column-major arrays: element
 *    (c, h, w, n) lives at c + C*(h + H*(w + W*n))  (src/core.jl:898-908).
 *  - All pointers are device pointers on the current CUDA device.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  The library
 *    launches only on that stream and never synchronises it.
 *  - The library allocates no device memory.  Scratch space for the per-image
 *    reductions is the caller's `workspace` (size from fssim_workspace_size);
 *    it must be zero-filled once before its first use, and every call leaves
 *    it zero-filled again.
 *  - Return value: FSSIM_OK (0) or a nonzero fssim_status; the message of the
 *    last error on the calling thread is available from fssim_last_error().
 */
#ifndef FASTSSIM_H
#define FASTSSIM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FSSIM_ABI_VERSION 1

/* Element types.  FSSIM_N0F8 is FixedPointNumbers' N0f8: a raw byte b read as
 * the Float32 value b/255 (correctly rounded). */
typedef enum fssim_dtype {
    FSSIM_FLOAT32 = 0,
    FSSIM_FLOAT16 = 1,
    FSSIM_N0F8 = 2,
    FSSIM_FLOAT64 = 3
} fssim_dtype;

/* Flags of fssim_fwd_bwd, one per argument of _ssim_fwd_bwd! (src/core.jl:933-940). */
enum fssim_flags {
    FSSIM_SKIP_SSIM = 1u << 0,      /* Val(skip_ssim): do not produce the (D)SSIM values      */
    FSSIM_SKIP_BACKWARD = 1u << 1,  /* Val(skip_backward): do not produce dL/dimgs1           */
    FSSIM_USE_DSSIM = 1u << 2,      /* use_dssim: L = 1 - SSIM (or (1 - SSIM)/2)               */
    FSSIM_DIVIDE_BY_TWO = 1u << 3,  /* divide_by_two_in_dssim                                  */
    FSSIM_SHOULD_ZERO = 1u << 4     /* should_zero: ignore the previous contents of `ssims`    */
};

typedef enum fssim_status {
    FSSIM_OK = 0,
    FSSIM_ERR_INVALID_ARGUMENT = 1,   /* null pointer, nonpositive size, unknown flag          */
    FSSIM_ERR_DIMENSION_MISMATCH = 2, /* e.g. ssims_len != N (the reference's DimensionMismatch) */
    FSSIM_ERR_UNSUPPORTED_DTYPE = 3,  /* dtype code not accepted for that argument             */
    FSSIM_ERR_WORKSPACE = 4,          /* workspace missing or smaller than fssim_workspace_size */
    FSSIM_ERR_MISALIGNED = 5,         /* a pointer not aligned to its element size             */
    FSSIM_ERR_CUDA = 6,               /* a CUDA runtime error (message has the details)        */
    FSSIM_ERR_COMM = 7,               /* NCCL missing, or an NCCL call / communicator failed   */
    FSSIM_ERR_TIMEOUT = 8             /* a collective did not finish within its deadline; the
                                         communicator has been aborted                          */
} fssim_status;

/* Library version string, e.g. "fastssim 0.1.0 (abi 1, sm_100a)". */
const char* fssim_version(void);

/* Bounds-checked builds only (compiled with -DFSSIM_DEBUG_BOUNDS: libfastssim_bounds.so).
 * There every global-memory access checks its element index first; an index
 * out of range is skipped and recorded.  Synchronises the current device, then
 * reports the site number of the first failing access (0 = none) and the count
 * of failing accesses since the last reset, and clears both if `reset`.  The
 * regular build returns FSSIM_ERR_INVALID_ARGUMENT.  No counterpart in the
 * reference (its kernels run under @inbounds, src/core.jl:186-187). */
int fssim_debug_bounds_status(unsigned* first_site, unsigned long long* count, int reset);

/* Copies the last error message of the calling thread into buf (NUL-terminated,
 * truncated to len).  Returns the status code of that error (FSSIM_OK if none). */
int fssim_last_error(char* buf, size_t len);

/* Bytes of workspace that fssim_fwd_bwd needs for these sizes and flags on the
 * current device.  Replaces no reference interface: the reference reduced with
 * float atomics into `ssims` (src/core.jl:412-440) and divided in a second
 * launch (src/core.jl:1123-1157); this engine reduces deterministically in one
 * launch and keeps its per-tile partial sums in the workspace. */
int fssim_workspace_size(int64_t c, int64_t h, int64_t w, int64_t n, uint32_t flags,
                         size_t* bytes);

/*
 * (D)SSIM of two image batches and/or its gradient with respect to the first.
 * Device half of _ssim_fwd_bwd! (src/core.jl:933-1107): one fused launch per call.
 *
 *  ssims        length-N vector of (D)SSIM values (dtype FLOAT32, FLOAT64 or FLOAT16).
 *               Required unless FSSIM_SKIP_SSIM.  Without FSSIM_SHOULD_ZERO the
 *               previous contents are added to the map sums before the division,
 *               as the reference's accumulation into N_ssims does (src/core.jl:919-922).
 *  ssims_len    must equal n (src/core.jl:967-969).
 *  dL_dimgs1    gradient, canonical (C,H,W,N) (dtype FLOAT32, FLOAT16 or FLOAT64).  Required
 *               unless FSSIM_SKIP_BACKWARD.
 *  imgs1, imgs2 canonical (C,H,W,N) inputs (dtype FLOAT32, FLOAT16, N0F8 or FLOAT64 each).
 *               With a FLOAT64 input the whole computation runs in double precision,
 *               as the reference's promote_type(T1, T2, Float32) does (src/core.jl:953-954).
 *  qmp          the reference's N_dssims_dQMP buffer (h,3,c,w,n).  Accepted for
 *               interface parity and never read or written: the fused kernel keeps
 *               the partial gradients on chip.  May be NULL.
 *  workspace    >= fssim_workspace_size() bytes, zero-filled before first use.
 *
 * The outputs (ssims, dL_dimgs1) must not overlap the inputs or each other
 * (FSSIM_ERR_INVALID_ARGUMENT): the fused kernel reads input rows around its
 * band after other blocks have written their outputs.  A caller that wants the
 * gradient in imgs1's own buffer copies imgs1 first.
 */
int fssim_fwd_bwd(void* ssims, int ssims_dtype, int64_t ssims_len,
                  void* dL_dimgs1, int grad_dtype,
                  const void* imgs1, int imgs1_dtype,
                  const void* imgs2, int imgs2_dtype,
                  void* qmp,
                  int64_t c, int64_t h, int64_t w, int64_t n,
                  uint32_t flags,
                  void* workspace, size_t workspace_bytes,
                  void* stream);

/*
 * fssim_fwd_bwd_scaled - fssim_fwd_bwd with a per-image factor on the gradient:
 * dL_dimgs1[:, :, :, i] = grad_scale[i] * d(D)SSIM_i / dimgs1.  Replaces the
 * pullback's separate broadcast `dL_dimgs1 .*= reshape(dL_dssims, 1, 1, 1, :)`
 * of the reference's rrules (ext/FastCUDASSIMChainRulesCoreExt.jl:28-36, :63-68)
 * when the gradient is computed at pullback time, with the cotangent known.
 * grad_scale: length-n device vector (FLOAT32, FLOAT64 or FLOAT16).  Other
 * arguments as fssim_fwd_bwd (without qmp); the (D)SSIM values are not scaled.
 */
int fssim_fwd_bwd_scaled(void* ssims, int ssims_dtype, int64_t ssims_len,
                         void* dL_dimgs1, int grad_dtype,
                         const void* imgs1, int imgs1_dtype,
                         const void* imgs2, int imgs2_dtype,
                         int64_t c, int64_t h, int64_t w, int64_t n,
                         uint32_t flags,
                         const void* grad_scale, int grad_scale_dtype,
                         void* workspace, size_t workspace_bytes,
                         void* stream);

/*
 * fssim_fwd_bwd_noalloc - fssim_fwd_bwd for callers that cannot allocate device memory.
 *
 * No counterpart in the reference: FastCUDASSIM.jl allocates its own buffers
 * through CUDA.jl.  Some callers of this library cannot: a plugin host that owns
 * all device memory through its own pool and hands the plugin no allocator, or
 * a real-time loop that forbids allocation once it has started.  They cannot
 * provide the reduction workspace that fssim_fwd_bwd asks for, so this entry
 * point uses a scratch array compiled into the library instead
 * (FSSIM_NOALLOC_SCRATCH_BYTES, resident on every GPU that loads the library
 * until the process exits).
 *
 * Arguments and results are those of fssim_fwd_bwd without `qmp` and the
 * workspace.  Limits and rules:
 *  - sizes whose workspace (fssim_workspace_size) exceeds
 *    FSSIM_NOALLOC_SCRATCH_BYTES are rejected with FSSIM_ERR_WORKSPACE;
 *  - no cudaMalloc, cudaFree or allocating library call is made; once every
 *    argument check has passed, the scratch counters are cleared with
 *    cudaMemsetAsync on `stream` just before the launch (a rejected call leaves
 *    the scratch untouched);
 *  - the scratch used is that of the CURRENT device at call time: as for
 *    fssim_fwd_bwd, the current device must be the device that holds the
 *    buffers, and `stream` must belong to it (FSSIM_ERR_INVALID_ARGUMENT if it
 *    does not);
 *  - the first call on a device looks up the scratch address on that device
 *    (cudaGetSymbolAddress) and keeps it for later calls; make that first call
 *    before any stream capture.  Calls must not continue across a
 *    cudaDeviceReset of that device (the address is not looked up again);
 *  - every call on a device shares the one scratch array: calls that overlap on
 *    the GPU (different streams, no ordering between them) race and give wrong
 *    (D)SSIM values.  Calls on one stream are ordered and safe.
 */
#define FSSIM_NOALLOC_SCRATCH_BYTES (4u << 20)

int fssim_fwd_bwd_noalloc(void* ssims, int ssims_dtype, int64_t ssims_len,
                          void* dL_dimgs1, int grad_dtype,
                          const void* imgs1, int imgs1_dtype,
                          const void* imgs2, int imgs2_dtype,
                          int64_t c, int64_t h, int64_t w, int64_t n,
                          uint32_t flags, void* stream);

/*
 * Multi-GPU: a batch split over the GPUs of one node, one process per GPU.
 *
 * No counterpart in the reference's code (FastCUDASSIM.jl runs one GPU per
 * call); it rests on the reference's per-image independence (src/core.jl:186,
 * test/batch_order.jl).  Rank `rank` of `world` owns the contiguous shard of
 * images [lo, lo + n_local) of the n_total images, where the first
 * n_total % world ranks hold one image more.  The library loads NCCL
 * (libnccl.so.2, 2.14 or later) at run time; FSSIM_ERR_COMM when it is absent.
 */

/* A fresh NCCL unique id (128 bytes) for fssim_comm_init; made on one rank and
 * sent to the others by the caller. */
int fssim_comm_unique_id(unsigned char id[128]);

/* An NCCL communicator for `rank` of `world` (ncclComm_t, returned as void*).
 * Created non-blocking and polled: if not every rank joins within deadline_s
 * seconds the attempt is aborted and FSSIM_ERR_TIMEOUT returned.  A communicator
 * made by the caller's own NCCL (NCCL.jl, torch) works as well. */
int fssim_comm_init(void** comm, int world, int rank, const unsigned char id[128], double deadline_s);

/* Destroys a communicator (abort_it = 0: finalise, then destroy) or aborts it
 * (abort_it != 0: ncclCommAbort, for a communicator a failed peer has left). */
int fssim_comm_destroy(void* comm, int abort_it);

/* Workspace bytes of fssim_fwd_bwd_sharded for this rank's shard. */
int fssim_sharded_workspace_size(int64_t c, int64_t h, int64_t w, int64_t n_total, int world, int rank,
                                 uint32_t flags, int ssims_dtype, size_t* bytes);

/*
 * fssim_fwd_bwd_sharded - fssim_fwd_bwd on this rank's shard, then the
 * all-gather of the per-image values, both enqueued on `stream`.
 *
 *  all_ssims  length-n_total output on every rank (device), dtype ssims_dtype;
 *             NULL with FSSIM_SKIP_SSIM (then nothing is exchanged)
 *  dL_dimgs1, imgs1, imgs2
 *             this rank's shard (C, H, W, n_local); the gradient stays local
 *  comm       ncclComm_t of the group (may be NULL when world == 1)
 * Equal shards are gathered in place in all_ssims; otherwise through padded
 * buffers in the workspace (size from fssim_sharded_workspace_size).  The
 * call returns once the work is enqueued: fssim_comm_wait bounds the wait for
 * it.  Without FSSIM_SHOULD_ZERO the values are added to all_ssims' previous
 * contents (src/core.jl:919-922).
 */
int fssim_fwd_bwd_sharded(void* all_ssims, int ssims_dtype, int64_t n_total,
                          void* dL_dimgs1, int grad_dtype,
                          const void* imgs1, int imgs1_dtype,
                          const void* imgs2, int imgs2_dtype,
                          int64_t c, int64_t h, int64_t w, int64_t n_local, uint32_t flags,
                          void* comm, int world, int rank,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Waits until `stream`'s work has finished, polling it and the communicator's
 * asynchronous error.  A communicator error, or a deadline that passes first (a
 * peer that died, hangs or never joined), aborts the communicator and returns
 * FSSIM_ERR_COMM or FSSIM_ERR_TIMEOUT; the caller then leaves the group. */
int fssim_comm_wait(void* comm, void* stream, double deadline_s);

#ifdef __cplusplus
}
#endif

#endif /* FASTSSIM_H */

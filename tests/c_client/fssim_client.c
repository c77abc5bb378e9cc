/*
 * A plain C client of libfastssim.so, calling it the way the Julia ccall shim
 * does: device buffers from the CUDA runtime, a caller-owned zeroed workspace,
 * one fssim_fwd_bwd call on the default stream.  No Python and no torch.
 *
 *   fssim_client C H W N flags x.bin y.bin ssims.bin grad.bin
 *
 * x.bin / y.bin hold C*H*W*N Float32 values in Julia (C,H,W,N) column-major
 * order; ssims.bin receives N Float32 values and grad.bin C*H*W*N.  It also
 * checks that a wrong ssims length is reported as FSSIM_ERR_DIMENSION_MISMATCH
 * with a message.  Exit status 0 on success.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime.h>

#include "fastssim.h"

static int read_file(const char* path, void* buf, size_t bytes)
{
    FILE* f = fopen(path, "rb");
    if (!f) return 1;
    size_t got = fread(buf, 1, bytes, f);
    fclose(f);
    return got == bytes ? 0 : 1;
}

static int write_file(const char* path, const void* buf, size_t bytes)
{
    FILE* f = fopen(path, "wb");
    if (!f) return 1;
    size_t put = fwrite(buf, 1, bytes, f);
    fclose(f);
    return put == bytes ? 0 : 1;
}

#define CUDA_OK(call)                                                             \
    do {                                                                          \
        cudaError_t e_ = (call);                                                  \
        if (e_ != cudaSuccess) {                                                  \
            fprintf(stderr, "%s: %s\n", #call, cudaGetErrorString(e_));           \
            return 3;                                                             \
        }                                                                         \
    } while (0)

int main(int argc, char** argv)
{
    if (argc != 10) {
        fprintf(stderr, "usage: %s C H W N flags x.bin y.bin ssims.bin grad.bin\n", argv[0]);
        return 2;
    }
    const int64_t c = atoll(argv[1]), h = atoll(argv[2]), w = atoll(argv[3]), n = atoll(argv[4]);
    /* SHOULD_ZERO: overwrite ssims (without it a call adds the previous contents, as the
       reference's accumulation into N_ssims does, and the second call below would) */
    const uint32_t flags = (uint32_t)strtoul(argv[5], NULL, 0) | FSSIM_SHOULD_ZERO;
    const size_t elems = (size_t)(c * h * w * n);
    float* hx = (float*)malloc(elems * sizeof(float));
    float* hy = (float*)malloc(elems * sizeof(float));
    float* hg = (float*)malloc(elems * sizeof(float));
    float* hs = (float*)malloc((size_t)n * sizeof(float));
    if (!hx || !hy || !hg || !hs) return 2;
    if (read_file(argv[6], hx, elems * sizeof(float)) || read_file(argv[7], hy, elems * sizeof(float))) {
        fprintf(stderr, "cannot read inputs\n");
        return 2;
    }
    printf("%s\n", fssim_version());

    float *dx, *dy, *dg, *ds;
    void* ws = NULL;
    size_t ws_bytes = 0;
    CUDA_OK(cudaMalloc((void**)&dx, elems * sizeof(float)));
    CUDA_OK(cudaMalloc((void**)&dy, elems * sizeof(float)));
    CUDA_OK(cudaMalloc((void**)&dg, elems * sizeof(float)));
    CUDA_OK(cudaMalloc((void**)&ds, (size_t)n * sizeof(float)));
    CUDA_OK(cudaMemcpy(dx, hx, elems * sizeof(float), cudaMemcpyHostToDevice));
    CUDA_OK(cudaMemcpy(dy, hy, elems * sizeof(float), cudaMemcpyHostToDevice));

    int st = fssim_workspace_size(c, h, w, n, flags, &ws_bytes);
    if (st != FSSIM_OK) {
        char msg[256];
        fssim_last_error(msg, sizeof msg);
        fprintf(stderr, "fssim_workspace_size: %d %s\n", st, msg);
        return 4;
    }
    if (ws_bytes) {
        CUDA_OK(cudaMalloc(&ws, ws_bytes));
        CUDA_OK(cudaMemset(ws, 0, ws_bytes));   /* zeroed once; every call leaves it zeroed */
    }

    /* a wrong ssims length is the reference's DimensionMismatch */
    st = fssim_fwd_bwd(ds, FSSIM_FLOAT32, n + 1, dg, FSSIM_FLOAT32, dx, FSSIM_FLOAT32, dy, FSSIM_FLOAT32, NULL,
                       c, h, w, n, flags, ws, ws_bytes, NULL);
    char msg[256];
    const int last = fssim_last_error(msg, sizeof msg);
    if (st != FSSIM_ERR_DIMENSION_MISMATCH || last != st || strlen(msg) == 0) {
        fprintf(stderr, "expected a dimension mismatch, got %d (%d: %s)\n", st, last, msg);
        return 5;
    }

    for (int rep = 0; rep < 2; ++rep) {   /* twice: the workspace must come back zeroed */
        st = fssim_fwd_bwd(ds, FSSIM_FLOAT32, n, dg, FSSIM_FLOAT32, dx, FSSIM_FLOAT32, dy, FSSIM_FLOAT32, NULL,
                           c, h, w, n, flags, ws, ws_bytes, NULL);
        if (st != FSSIM_OK) {
            fssim_last_error(msg, sizeof msg);
            fprintf(stderr, "fssim_fwd_bwd: %d %s\n", st, msg);
            return 6;
        }
    }
    CUDA_OK(cudaDeviceSynchronize());
    CUDA_OK(cudaMemcpy(hs, ds, (size_t)n * sizeof(float), cudaMemcpyDeviceToHost));
    CUDA_OK(cudaMemcpy(hg, dg, elems * sizeof(float), cudaMemcpyDeviceToHost));
    if (write_file(argv[8], hs, (size_t)n * sizeof(float)) || write_file(argv[9], hg, elems * sizeof(float)))
        return 2;
    cudaFree(dx);
    cudaFree(dy);
    cudaFree(dg);
    cudaFree(ds);
    if (ws) cudaFree(ws);
    free(hx);
    free(hy);
    free(hg);
    free(hs);
    printf("ok\n");
    return 0;
}

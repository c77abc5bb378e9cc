/*
 * Host cost of one libfastssim.so call from C (no Python): the forward SSIM of one
 * C x 1080 x 1920 image pair, as ssim!/ssim call it through the Julia ccall shim.
 *
 *   fssim_call_cost C [calls]
 *
 * Prints one JSON object:
 *   enqueue_us   host time of fssim_fwd_bwd, averaged over back-to-back calls
 *   device_us    device time per call, back to back (CUDA events)
 *   roundtrip_us host time of one call plus the 4-byte read of its value
 *                (cudaMemcpy on the default stream), median of the calls
 * Inputs are zero-filled device buffers: the cost does not depend on the values.
 */
#define _POSIX_C_SOURCE 199309L
#include <stdio.h>
#include <stdlib.h>
#include <time.h>

#include <cuda_runtime.h>

#include "fastssim.h"

static double now_us(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e6 + ts.tv_nsec * 1e-3;
}

static int cmp_d(const void* a, const void* b)
{
    const double x = *(const double*)a, y = *(const double*)b;
    return (x > y) - (x < y);
}

#define CUDA_OK(call)                                                        \
    do {                                                                     \
        cudaError_t e_ = (call);                                             \
        if (e_ != cudaSuccess) {                                             \
            fprintf(stderr, "%s: %s\n", #call, cudaGetErrorString(e_));      \
            return 3;                                                        \
        }                                                                    \
    } while (0)

int main(int argc, char** argv)
{
    if (argc < 2) {
        fprintf(stderr, "usage: %s C [calls]\n", argv[0]);
        return 2;
    }
    const int64_t c = atoll(argv[1]), h = 1080, w = 1920, n = 1;
    const int calls = argc > 2 ? atoi(argv[2]) : 200;
    const uint32_t flags = FSSIM_SKIP_BACKWARD | FSSIM_SHOULD_ZERO;
    const size_t bytes = (size_t)(c * h * w * n) * sizeof(float);
    float *dx = NULL, *dy = NULL, *ds = NULL;
    void* ws = NULL;
    size_t wsb = 0;
    CUDA_OK(cudaMalloc((void**)&dx, bytes));
    CUDA_OK(cudaMalloc((void**)&dy, bytes));
    CUDA_OK(cudaMalloc((void**)&ds, sizeof(float)));
    CUDA_OK(cudaMemset(dx, 0, bytes));
    CUDA_OK(cudaMemset(dy, 0, bytes));
    if (fssim_workspace_size(c, h, w, n, flags, &wsb) != FSSIM_OK) return 4;
    CUDA_OK(cudaMalloc(&ws, wsb > 0 ? wsb : 256));
    CUDA_OK(cudaMemset(ws, 0, wsb > 0 ? wsb : 256));
#define CALL() fssim_fwd_bwd(ds, FSSIM_FLOAT32, n, NULL, FSSIM_FLOAT32, dx, FSSIM_FLOAT32, dy, FSSIM_FLOAT32, \
                             NULL, c, h, w, n, flags, ws, wsb, NULL)
    for (int i = 0; i < 20; ++i)
        if (CALL() != FSSIM_OK) return 5;
    CUDA_OK(cudaDeviceSynchronize());

    /* host cost of the call itself: launches are asynchronous, so the loop measures the
       library's argument checks, configuration and launch */
    double t0 = now_us();
    for (int i = 0; i < calls; ++i) CALL();
    double t1 = now_us();
    CUDA_OK(cudaDeviceSynchronize());
    const double enqueue_us = (t1 - t0) / calls;

    /* device time per call, back to back */
    cudaEvent_t a, b;
    CUDA_OK(cudaEventCreate(&a));
    CUDA_OK(cudaEventCreate(&b));
    CUDA_OK(cudaEventRecord(a, 0));
    for (int i = 0; i < calls; ++i) CALL();
    CUDA_OK(cudaEventRecord(b, 0));
    CUDA_OK(cudaEventSynchronize(b));
    float ms = 0.f;
    CUDA_OK(cudaEventElapsedTime(&ms, a, b));

    /* one call plus the read of its value, as the scalar API does */
    double* rt = (double*)malloc(sizeof(double) * calls);
    float v = 0.f;
    for (int i = 0; i < calls; ++i) {
        const double s0 = now_us();
        CALL();
        CUDA_OK(cudaMemcpy(&v, ds, sizeof(float), cudaMemcpyDeviceToHost));
        rt[i] = now_us() - s0;
    }
    qsort(rt, calls, sizeof(double), cmp_d);
    printf("{\"channels\": %lld, \"calls\": %d, \"enqueue_us\": %.3f, \"device_us\": %.3f, \"roundtrip_us\": %.3f, "
           "\"ssim_of_zero_images\": %.6f}\n",
           (long long)c, calls, enqueue_us, ms * 1e3 / calls, rt[calls / 2], v);
    free(rt);
    cudaFree(dx);
    cudaFree(dy);
    cudaFree(ds);
    cudaFree(ws);
    return 0;
}

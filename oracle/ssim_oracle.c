/*
 * CPU oracle for the SSIM / DSSIM forward pass and the gradient with respect to
 * the first image batch.  TEST INFRASTRUCTURE ONLY: the parity tests, the smoke
 * check and the CPU-baseline leg of the benchmark load this file's library for
 * reference values.  No product code path may call it.
 *
 * It restates the arithmetic of FastCUDASSIM.jl v0.2.1, src/core.jl, in two modes:
 *
 *   - "f32": single precision, with the reference's operation order kept
 *     (no FMA contraction: build with -ffp-contract=off), so results agree with
 *     the reference's CUDA.jl kernels up to the order of the final per-image
 *     summation (the reference sums with float atomics in arbitrary order;
 *     here the sum is taken in double, in a fixed order);
 *   - "f64": the same algorithm evaluated in double precision, with the
 *     reference's Float32 constants (kernel weights, C1, C2) widened to double.
 *
 * Citations (file:line in the reference project):
 *   kernel weights, sigma, radius ......... src/core.jl:40-46
 *   C1, C2 ................................ src/core.jl:49-50
 *   forward u-pass (w direction, plain tap order) src/core.jl:260-305
 *   forward v-pass (h direction, symmetric pairing) src/core.jl:330-359
 *   SSIM map formula ...................... src/core.jl:363-378
 *   stored partial gradients Q, M, P ...... src/core.jl:383-389
 *   N_inv ................................. src/core.jl:584-589
 *   backward load (negate for DSSIM, zero outside the image) src/core.jl:640-661
 *   backward u-pass / v-pass (symmetric) .. src/core.jl:684-770
 *   backward combine ...................... src/core.jl:773-782
 *   divide by N and DSSIM transform ....... src/core.jl:1123-1157
 *
 * Memory layout of every image batch: canonical (C, H, W, N) column-major, i.e.
 * element (c, h, w, n) sits at c + C*(h + H*(w + W*n)).
 * The "u" direction of the reference is the width axis w, "v" is the height axis h.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <stdatomic.h>

#define ORC_RADIUS 5
#define ORC_TAPS 11

enum {
    ORC_SKIP_SSIM = 1,
    ORC_SKIP_BACKWARD = 2,
    ORC_USE_DSSIM = 4,
    ORC_DIVIDE_BY_TWO = 8
};

/* src/core.jl:40-46: k_i = exp(-0.5f0 * (i / 1.5f0)^2) for i = -5..5 in Float32,
 * divided by their Float32 sum.  The exponential is evaluated in double and
 * rounded once to float (a correctly rounded float exp for these 6 arguments);
 * the sum runs left to right in float. */
void oracle_kernel_weights(float k[ORC_TAPS])
{
    const float stdv = 1.5f;
    float raw[ORC_TAPS];
    float sum = 0.0f;
    for (int i = -ORC_RADIUS; i <= ORC_RADIUS; ++i) {
        float r = (float)i / stdv;
        float a = -0.5f * (r * r);
        raw[i + ORC_RADIUS] = (float)exp((double)a);
    }
    for (int i = 0; i < ORC_TAPS; ++i) sum += raw[i];
    for (int i = 0; i < ORC_TAPS; ++i) k[i] = raw[i] / sum;
}

/* src/core.jl:49-50 */
float oracle_c1(void) { return 0.01f * 0.01f; }
float oracle_c2(void) { return 0.03f * 0.03f; }

static inline size_t cidx(int64_t c, int64_t h, int64_t w, int64_t n,
                          int64_t C, int64_t H, int64_t W)
{
    return (size_t)(c + C * (h + H * (w + W * n)));
}

/* ------------------------------------------------------------------------- */
/* Single precision, reference operation order.                              */
/* ------------------------------------------------------------------------- */

/* One (image, channel) plane.  xp, yp: H*W floats, plane layout [w][h].
 * Returns the plane's sum of SSIM map values (double), and, when want_grad,
 * writes the per-pixel contributions N*dL/dx (before the N_inv scaling) into
 * gp (plane layout [w][h]) after negation for DSSIM.  Scratch is caller-owned. */
static double plane_f32(const float* xp, const float* yp, int64_t H, int64_t W,
                        const float* k, float C1, float C2, int want_grad, int use_dssim,
                        float* gp, float* scratch)
{
    const int64_t P = H * W;
    float* u = scratch;            /* 5 planes: u-convolved moments           */
    float* qmp = u + 5 * P;        /* 3 planes: partials Q, M, P              */
    float* bu = qmp + 3 * P;       /* 3 planes: u-convolved partials          */
    double sum = 0.0;

    /* forward u-pass (w direction), taps in plain order i = 0..10 */
    for (int64_t w = 0; w < W; ++w) {
        for (int64_t h = 0; h < H; ++h) {
            float s1 = 0.f, s11 = 0.f, s2 = 0.f, s22 = 0.f, s12 = 0.f;
            for (int i = 0; i < ORC_TAPS; ++i) {
                int64_t ww = w - ORC_RADIUS + i;
                float a = 0.f, b = 0.f;
                if (ww >= 0 && ww < W) { a = xp[ww * H + h]; b = yp[ww * H + h]; }
                float ak = a * k[i];
                float bk = b * k[i];
                s1 += ak;
                s11 += a * ak;
                s2 += bk;
                s22 += b * bk;
                s12 += a * bk;
            }
            size_t o = (size_t)(w * H + h);
            u[o] = s1; u[P + o] = s11; u[2 * P + o] = s2; u[3 * P + o] = s22; u[4 * P + o] = s12;
        }
    }

    /* forward v-pass (h direction), symmetric pairing, then the SSIM map */
    for (int64_t w = 0; w < W; ++w) {
        for (int64_t h = 0; h < H; ++h) {
            float mom[5];
            for (int j = 0; j < 5; ++j) {
                const float* uj = u + (size_t)j * P + (size_t)w * H;
                float acc = uj[h] * k[ORC_RADIUS];
                for (int iu = 0; iu < ORC_RADIUS; ++iu) {
                    int64_t hu = h - ORC_RADIUS + iu;
                    int64_t hd = h + ORC_RADIUS - iu;
                    float a = (hu >= 0) ? uj[hu] : 0.f;
                    float b = (hd < H) ? uj[hd] : 0.f;
                    acc += (a + b) * k[iu];
                }
                mom[j] = acc;
            }
            float m = mom[0], q = mom[1], mR = mom[2], qR = mom[3], p = mom[4];
            float m_sq = m * m;
            float v = q - m_sq;
            float mmR = m * mR;
            float c = p - mmR;
            float mR_sq = mR * mR;
            float vR = qR - mR_sq;
            float x = 2.f * mmR + C1;
            float y = 2.f * c + C2;
            float z = (m_sq + mR_sq) + C1;
            float t = (v + vR) + C2;
            float zt_inv = 1.f / (z * t);
            float s = (x * y) * zt_inv;
            sum += (double)s;
            if (want_grad) {
                size_t o = (size_t)(w * H + h);
                float Qv = (-s) / t;
                float Mv = (2.f * zt_inv) * (((y - x) * mR) + ((s * (z - t)) * m));
                float Pv = (2.f * x) * zt_inv;
                if (use_dssim) { Qv = -Qv; Mv = -Mv; Pv = -Pv; }
                qmp[o] = Qv; qmp[P + o] = Mv; qmp[2 * P + o] = Pv;
            }
        }
    }
    if (!want_grad) return sum;

    /* backward u-pass (w direction), symmetric pairing, zero outside the image */
    for (int j = 0; j < 3; ++j) {
        const float* src = qmp + (size_t)j * P;
        float* dst = bu + (size_t)j * P;
        for (int64_t w = 0; w < W; ++w) {
            for (int64_t h = 0; h < H; ++h) {
                float acc = src[w * H + h] * k[ORC_RADIUS];
                for (int iu = 0; iu < ORC_RADIUS; ++iu) {
                    int64_t wl = w - ORC_RADIUS + iu;
                    int64_t wr = w + ORC_RADIUS - iu;
                    float a = (wl >= 0) ? src[wl * H + h] : 0.f;
                    float b = (wr < W) ? src[wr * H + h] : 0.f;
                    acc += (a + b) * k[iu];
                }
                dst[w * H + h] = acc;
            }
        }
    }
    /* backward v-pass (h direction) and the combine (without N_inv) */
    for (int64_t w = 0; w < W; ++w) {
        for (int64_t h = 0; h < H; ++h) {
            float r[3];
            for (int j = 0; j < 3; ++j) {
                const float* src = bu + (size_t)j * P + (size_t)w * H;
                float acc = src[h] * k[ORC_RADIUS];
                for (int iu = 0; iu < ORC_RADIUS; ++iu) {
                    int64_t hu = h - ORC_RADIUS + iu;
                    int64_t hd = h + ORC_RADIUS - iu;
                    float a = (hu >= 0) ? src[hu] : 0.f;
                    float b = (hd < H) ? src[hd] : 0.f;
                    acc += (a + b) * k[iu];
                }
                r[j] = acc;
            }
            size_t o = (size_t)(w * H + h);
            float via_Q = (2.f * xp[o]) * r[0];
            float via_P = yp[o] * r[2];
            gp[o] = (via_Q + r[1]) + via_P;
        }
    }
    return sum;
}

/* ------------------------------------------------------------------------- */
/* Double precision, same algorithm, Float32 constants widened.              */
/* ------------------------------------------------------------------------- */
static double plane_f64(const double* xp, const double* yp, int64_t H, int64_t W,
                        const double* k, double C1, double C2, int want_grad, int use_dssim,
                        double* gp, double* scratch)
{
    const int64_t P = H * W;
    double* u = scratch;
    double* qmp = u + 5 * P;
    double* bu = qmp + 3 * P;
    double sum = 0.0;
    for (int64_t w = 0; w < W; ++w) {
        for (int64_t h = 0; h < H; ++h) {
            double s1 = 0, s11 = 0, s2 = 0, s22 = 0, s12 = 0;
            for (int i = 0; i < ORC_TAPS; ++i) {
                int64_t ww = w - ORC_RADIUS + i;
                double a = 0, b = 0;
                if (ww >= 0 && ww < W) { a = xp[ww * H + h]; b = yp[ww * H + h]; }
                double ak = a * k[i], bk = b * k[i];
                s1 += ak; s11 += a * ak; s2 += bk; s22 += b * bk; s12 += a * bk;
            }
            size_t o = (size_t)(w * H + h);
            u[o] = s1; u[P + o] = s11; u[2 * P + o] = s2; u[3 * P + o] = s22; u[4 * P + o] = s12;
        }
    }
    for (int64_t w = 0; w < W; ++w) {
        for (int64_t h = 0; h < H; ++h) {
            double mom[5];
            for (int j = 0; j < 5; ++j) {
                const double* uj = u + (size_t)j * P + (size_t)w * H;
                double acc = uj[h] * k[ORC_RADIUS];
                for (int iu = 0; iu < ORC_RADIUS; ++iu) {
                    int64_t hu = h - ORC_RADIUS + iu, hd = h + ORC_RADIUS - iu;
                    double a = (hu >= 0) ? uj[hu] : 0, b = (hd < H) ? uj[hd] : 0;
                    acc += (a + b) * k[iu];
                }
                mom[j] = acc;
            }
            double m = mom[0], q = mom[1], mR = mom[2], qR = mom[3], p = mom[4];
            double x = 2 * m * mR + C1;
            double y = 2 * (p - m * mR) + C2;
            double z = m * m + mR * mR + C1;
            double t = (q - m * m) + (qR - mR * mR) + C2;
            double zt_inv = 1 / (z * t);
            double s = x * y * zt_inv;
            sum += s;
            if (want_grad) {
                size_t o = (size_t)(w * H + h);
                double sg = use_dssim ? -1.0 : 1.0;
                qmp[o] = sg * (-s / t);
                qmp[P + o] = sg * (2 * zt_inv * ((y - x) * mR + s * (z - t) * m));
                qmp[2 * P + o] = sg * (2 * x * zt_inv);
            }
        }
    }
    if (!want_grad) return sum;
    for (int j = 0; j < 3; ++j) {
        const double* src = qmp + (size_t)j * P;
        double* dst = bu + (size_t)j * P;
        for (int64_t w = 0; w < W; ++w)
            for (int64_t h = 0; h < H; ++h) {
                double acc = src[w * H + h] * k[ORC_RADIUS];
                for (int iu = 0; iu < ORC_RADIUS; ++iu) {
                    int64_t wl = w - ORC_RADIUS + iu, wr = w + ORC_RADIUS - iu;
                    double a = (wl >= 0) ? src[wl * H + h] : 0, b = (wr < W) ? src[wr * H + h] : 0;
                    acc += (a + b) * k[iu];
                }
                dst[w * H + h] = acc;
            }
    }
    for (int64_t w = 0; w < W; ++w)
        for (int64_t h = 0; h < H; ++h) {
            double r[3];
            for (int j = 0; j < 3; ++j) {
                const double* src = bu + (size_t)j * P + (size_t)w * H;
                double acc = src[h] * k[ORC_RADIUS];
                for (int iu = 0; iu < ORC_RADIUS; ++iu) {
                    int64_t hu = h - ORC_RADIUS + iu, hd = h + ORC_RADIUS - iu;
                    double a = (hu >= 0) ? src[hu] : 0, b = (hd < H) ? src[hd] : 0;
                    acc += (a + b) * k[iu];
                }
                r[j] = acc;
            }
            size_t o = (size_t)(w * H + h);
            gp[o] = 2 * xp[o] * r[0] + r[1] + yp[o] * r[2];
        }
    return sum;
}

/* src/core.jl:1123-1157 (single precision): s = Sigma / N, then 1 - s or (1 - s) / 2. */
static float finish_f32(float sigma, int64_t N, int flags)
{
    float s = sigma / (float)N;
    if (flags & ORC_USE_DSSIM) return (flags & ORC_DIVIDE_BY_TWO) ? (1.f - s) / 2.f : 1.f - s;
    return s;
}
static double finish_f64(double sigma, int64_t N, int flags)
{
    double s = sigma / (double)N;
    if (flags & ORC_USE_DSSIM) return (flags & ORC_DIVIDE_BY_TWO) ? (1 - s) / 2 : 1 - s;
    return s;
}

/* Work distribution over (image, channel) planes with plain pthreads: each
 * worker owns its scratch and takes the next plane from an atomic counter. */
typedef struct {
    int dbl;                      /* 0: f32 mode, 1: f64 mode */
    const void* x; const void* y; void* grad;
    int64_t C, H, W, B;
    int flags, want_grad;
    double* sums;                 /* B*C plane sums */
    atomic_long next;
    atomic_int err;
} orc_job;

static void* orc_worker(void* arg)
{
    orc_job* J = (orc_job*)arg;
    const int64_t C = J->C, H = J->H, W = J->W, P = H * W;
    const int64_t NPX = C * H * W;
    const int use_dssim = (J->flags & ORC_USE_DSSIM) != 0;
    const int div2 = use_dssim && (J->flags & ORC_DIVIDE_BY_TWO);
    float kf[ORC_TAPS];
    oracle_kernel_weights(kf);
    if (!J->dbl) {
        const float* x = (const float*)J->x; const float* y = (const float*)J->y;
        float* grad = (float*)J->grad;
        /* src/core.jl:584-589: N_inv = Td1(1)/N or Td1(0.5)/N with Td1 = Float32 */
        const float N_inv = div2 ? 0.5f / (float)NPX : 1.0f / (float)NPX;
        float* buf = (float*)malloc(sizeof(float) * (size_t)P * 14);
        if (!buf) { atomic_store(&J->err, 2); return NULL; }
        float *xp = buf, *yp = xp + P, *gp = yp + P, *scratch = gp + P;
        for (;;) {
            int64_t nc = atomic_fetch_add(&J->next, 1);
            if (nc >= J->B * C) break;
            int64_t n = nc / C, c = nc % C;
            for (int64_t w = 0; w < W; ++w)
                for (int64_t h = 0; h < H; ++h) {
                    size_t g = cidx(c, h, w, n, C, H, W);
                    xp[w * H + h] = x[g]; yp[w * H + h] = y[g];
                }
            J->sums[nc] = plane_f32(xp, yp, H, W, kf, oracle_c1(), oracle_c2(),
                                    J->want_grad, use_dssim, gp, scratch);
            if (J->want_grad)
                for (int64_t w = 0; w < W; ++w)
                    for (int64_t h = 0; h < H; ++h)
                        grad[cidx(c, h, w, n, C, H, W)] = gp[w * H + h] * N_inv;
        }
        free(buf);
    } else {
        const double* x = (const double*)J->x; const double* y = (const double*)J->y;
        double* grad = (double*)J->grad;
        double k[ORC_TAPS];
        for (int i = 0; i < ORC_TAPS; ++i) k[i] = (double)kf[i];
        const double N_inv = div2 ? 0.5 / (double)NPX : 1.0 / (double)NPX;
        double* buf = (double*)malloc(sizeof(double) * (size_t)P * 14);
        if (!buf) { atomic_store(&J->err, 2); return NULL; }
        double *xp = buf, *yp = xp + P, *gp = yp + P, *scratch = gp + P;
        for (;;) {
            int64_t nc = atomic_fetch_add(&J->next, 1);
            if (nc >= J->B * C) break;
            int64_t n = nc / C, c = nc % C;
            for (int64_t w = 0; w < W; ++w)
                for (int64_t h = 0; h < H; ++h) {
                    size_t g = cidx(c, h, w, n, C, H, W);
                    xp[w * H + h] = x[g]; yp[w * H + h] = y[g];
                }
            J->sums[nc] = plane_f64(xp, yp, H, W, k, (double)oracle_c1(), (double)oracle_c2(),
                                    J->want_grad, use_dssim, gp, scratch);
            if (J->want_grad)
                for (int64_t w = 0; w < W; ++w)
                    for (int64_t h = 0; h < H; ++h)
                        grad[cidx(c, h, w, n, C, H, W)] = gp[w * H + h] * N_inv;
        }
        free(buf);
    }
    return NULL;
}

static int orc_run(orc_job* J, int nthreads, double* ssims)
{
    const int64_t planes = J->B * J->C;
    if (nthreads <= 0) nthreads = 1;
    if (nthreads > planes) nthreads = (int)planes;
    J->sums = (double*)calloc((size_t)planes, sizeof(double));
    if (!J->sums) return 2;
    atomic_init(&J->next, 0);
    atomic_init(&J->err, 0);
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
    int started = 0;
    if (th)
        for (; started < nthreads - 1; ++started)
            if (pthread_create(&th[started], NULL, orc_worker, J) != 0) break;
    orc_worker(J);   /* the calling thread works too */
    for (int i = 0; i < started; ++i) pthread_join(th[i], NULL);
    free(th);
    int err = atomic_load(&J->err);
    const int64_t NPX = J->C * J->H * J->W;
    if (!err && ssims) {
        for (int64_t n = 0; n < J->B; ++n) {
            double t = 0.0;
            for (int64_t c = 0; c < J->C; ++c) t += J->sums[n * J->C + c];
            ssims[n] = J->dbl ? finish_f64(t, NPX, J->flags)
                              : (double)finish_f32((float)t, NPX, J->flags);
        }
    }
    free(J->sums);
    return err;
}

/*
 * Entry points.  x, y: canonical (C,H,W,B) arrays, already converted to the
 * compute type (N0f8 -> raw/255 in float, Float16 -> float, exactly).
 * ssims (length B, nullable): final (D)SSIM values.  grad (C*H*W*B, nullable):
 * dL/dx in canonical layout.  Returns 0 on success, nonzero on bad arguments
 * or allocation failure.  nthreads: worker threads (the caller's included).
 */
int oracle_ssim_f32(const float* x, const float* y, int64_t C, int64_t H, int64_t W, int64_t B,
                    int flags, double* ssims, float* grad, int nthreads)
{
    if (!x || !y || C < 1 || H < 1 || W < 1 || B < 1) return 1;
    orc_job J;
    memset(&J, 0, sizeof J);
    J.dbl = 0; J.x = x; J.y = y; J.grad = grad;
    J.C = C; J.H = H; J.W = W; J.B = B; J.flags = flags;
    J.want_grad = !(flags & ORC_SKIP_BACKWARD) && grad != NULL;
    return orc_run(&J, nthreads, (flags & ORC_SKIP_SSIM) ? NULL : ssims);
}

int oracle_ssim_f64(const double* x, const double* y, int64_t C, int64_t H, int64_t W, int64_t B,
                    int flags, double* ssims, double* grad, int nthreads)
{
    if (!x || !y || C < 1 || H < 1 || W < 1 || B < 1) return 1;
    orc_job J;
    memset(&J, 0, sizeof J);
    J.dbl = 1; J.x = x; J.y = y; J.grad = grad;
    J.C = C; J.H = H; J.W = W; J.B = B; J.flags = flags;
    J.want_grad = !(flags & ORC_SKIP_BACKWARD) && grad != NULL;
    return orc_run(&J, nthreads, (flags & ORC_SKIP_SSIM) ? NULL : ssims);
}

/* N0f8 -> Float32: the correctly rounded value of raw / 255 (FixedPointNumbers'
 * Normed{UInt8,8} conversion). */
void oracle_n0f8_to_f32(const uint8_t* src, float* dst, int64_t n)
{
    for (int64_t i = 0; i < n; ++i) dst[i] = (float)src[i] / 255.0f;
}

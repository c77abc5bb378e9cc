// SSIM + gradient: the two-group pipelined kernel (pipe_kernel).
#pragma once

#include "fssim_common.cuh"

namespace fssim {

// ---------------------------------------------------------------------------
// Two-group pipelined kernel: SSIM + gradient (and gradient only), every input
// and gradient dtype but Float64.
//
// The streaming decomposition described in fssim_common.cuh, with the 5-row
// gradient halo (T = NT - 10); the CTA is split into two warp groups of NT
// threads that work on different steps at once:
//
//   group A (threads 0..NT-1):    cp.async loads (inputs, and the x/y values B2
//                                 needs), F1(t), B1(t-2)
//   group B (threads NT..2NT-1):  F2(t-1) + SSIM map + partials, B2(t-3)
//
// Every stage reads only what the other group wrote in the previous slot, so a
// single barrier per slot (named barrier BAR_SLOT over both groups) orders
// everything; the buffers passed between the groups are double-buffered by step
// parity.
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
    // 64-bit index arithmetic here on purpose: the 32-bit split of band_index() moves this
    // kernel to another register allocation that measured 3% slower
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
        named_barrier_sync(BAR_SLOT, 2 * NT);
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
            named_barrier_sync(BAR_SLOT, 2 * NT);
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
            named_barrier_sync(BAR_SLOT, 2 * NT);
        };

        named_barrier_sync(BAR_SLOT, 2 * NT);
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

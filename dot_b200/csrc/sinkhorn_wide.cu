// Fused single-pass Sinkhorn iterations for wide rows (8192 <= m <= 65536,
// m % 32 == 0): one launch per iteration reads the B x n x m matrix once.
//
//   u_i = la_i - LSE_j(K_ij + v_j),  then column partials of LSE_i(K_ij + u_i)
//   with the new u (Gauss-Seidel order, src/sinkhorn/torch_cuda.cpp:200-223).
//
// A row does not fit one CTA's registers, so a thread-block cluster of kWC
// CTAs shares every row: CTA r of a cluster owns columns [r*mc, (r+1)*mc),
// mc = m / kWC, and keeps v and its columns' running partials in registers
// (thread t: columns 4t + 4Tq, q < NQ, T threads).  The clusters split the
// B*nbat row batches into equal contiguous ranges.
// Per batch g (the rows of one stage, R <= 4), every warp of every CTA
//   pass A   waits for the batch's slice rows (1-D bulk copies on a 3-stage
//            mbarrier ring), forms t = K + v over its columns, a warp max,
//            E = exp(t - max) (written back in place) and the warp sum, and
//            stores that (max, sum) pair into every CTA of the cluster with
//            st.async, whose bytes complete a transaction on the receiver's
//            mbarrier (a 4-slot ring of exchange buffers);
//   u        of the previous batch g-1: waits for that batch's pairs from all
//            kWC x W warps of the cluster (they had this batch's pass A to
//            arrive) and merges them itself (every warp gets the same LSE);
//   pass B   of batch g-1: column partials S_j += E_ij * exp(max_i + u_i - A)
//            (one FFMA per element, A a warp-wide reference, as in
//            sinkhorn_fused.cu); the last warp done with a stage refills it.
// No barrier joins the warps inside the loop.  A sender reuses a slot only
// after every warp of the cluster has consumed the slot's previous batch:
// sending batch g follows the sender's own u of batch g-2, which needed
// batch g-2's pairs from every warp, each sent after that warp's u of g-4.
// When its range leaves a problem, a CTA publishes its columns' partials;
// the CTA that arrives last among the same-rank CTAs of every cluster that
// touched the problem merges that column slice in cluster order (atomic
// arrival counter, no waiting) and writes v.  Columns whose merged sum is
// too small to trust are recomputed exactly.  For a row shard of a larger
// problem the kernel only publishes the partials: skw_pairs_merge_kernel
// (every SM, one thread per column, the same arithmetic in the same order)
// merges them into the (max, sum) pairs of the cross-GPU combine, so no
// single CTA per slice runs the merge after the rest of the grid is done.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "sinkhorn.h"
#include "tma.cuh"

namespace dotb {

namespace {

constexpr int kWC = 8;                 // CTAs per cluster
constexpr int kWMaxR = 4;              // rows per batch (at most)
constexpr int kWX = 4;                 // row-pair exchange slots (batches in flight between CTAs)

// CTA shapes: threads, stage bytes, CTAs per SM, stages.  A batch is the
// rows one stage holds; its exponentials stay in the stage until the column
// update, so deep stages (few batches, little per-batch work) pay best.
template <int T_, int STAGE_, int MINB_, int S_>
struct WCfg {
    static constexpr int T = T_;
    static constexpr int W = T_ / 32;
    static constexpr int STAGE = STAGE_;
    static constexpr int MINB = MINB_;
    static constexpr int S = S_;
};
using WideA = WCfg<512, 65536, 1, 3>;   // 512 threads, one CTA per SM (slices up to 8192 columns)
using WideB = WCfg<256, 32768, 2, 3>;   // 256 threads, two CTAs per SM (slices up to 4096 columns)
enum WideShape { kShapeA = 0, kShapeB = 1 };
// Rows per batch for a shape and NQ (slices of at most 4*T*NQ columns): the
// rows of a full slice one stage holds, at most kWMaxR.
template <class CFG, int NQ>
__host__ __device__ constexpr int wide_rows_of() {
    return CFG::STAGE / (16 * CFG::T * NQ) < 1 ? 1
         : CFG::STAGE / (16 * CFG::T * NQ) > kWMaxR ? kWMaxR : CFG::STAGE / (16 * CFG::T * NQ);
}
constexpr int kWFix = 1024;            // exactly recomputed columns per slice merge (cap)
constexpr float kRaiseW = 60.0f;
constexpr float kTinyW = 8.077935669463161e-28f;   // 2^-90

__device__ __forceinline__ uint32_t w_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t w_cid() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void w_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void w_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
struct WideArgs {
    const float* X;
    float kinv;
    const float* la;
    float la_def;
    const float* lb;
    float lb_def;
    float* u2;
    float* v2;
    int64_t n, m, mc;   // rows per problem, row length, columns per CTA
    int R;              // rows per batch
    int nbat;           // batches per problem
    int TB;             // batches in the batch (B * nbat)
    int G;              // clusters
    int maxseg;         // most clusters touching one problem
    float2* part;       // [B][maxseg][m] column (max, sum) partials
    int32_t* cnt;       // [B][kWC] arrival counters, zero between launches
    float2* pairs;      // row-shard mode: merged column pairs [B][m]; nullptr: write v
    int32_t* err;       // bounded-wait expiry word
};

__host__ __device__ __forceinline__ int w_q(const WideArgs& a, int k) { return int(int64_t(k) * a.TB / a.G); }
__host__ __device__ __forceinline__ int w_owner(const WideArgs& a, int x) {
    return int((int64_t(x + 1) * a.G + a.TB - 1) / a.TB) - 1;
}

// Exact column (max, sum) pair over all n rows of problem b (max pass, then
// the sum of exp(t - max) -- at least 1); one warp, strided reads; only for
// columns whose shared-reference sum is too small to trust.
__device__ float2 w_exact_pair(const float* X, const float* u2, float kinv, int64_t b, int64_t n, int64_t m,
                               int64_t col) {
    const int lane = threadIdx.x & 31;
    const float* xb = X + b * n * m + col;
    const float* ub = u2 + b * n;
    float mx = kNegBig;
    for (int64_t i = lane; i < n; i += 32) mx = fmaxf(mx, kplus(__ldcg(xb + i * m), kinv, __ldcg(ub + i)));
    mx = warp_max<32>(mx);
    float sm = 0.0f;
    for (int64_t i = lane; i < n; i += 32) sm += exp_shift(kplus(__ldcg(xb + i * m), kinv, __ldcg(ub + i)) - mx);
    return make_float2(mx, warp_sum<32>(sm));
}

__device__ float w_exact_column(const float* X, const float* u2, float kinv, int64_t b, int64_t n, int64_t m,
                                int64_t col) {
    const float2 p = w_exact_pair(X, u2, kinv, b, n, m, col);
    return lse_finish(p.x, p.y);
}

template <class CFG, int NQ, bool FULL>
__global__ void __launch_bounds__(CFG::T, CFG::MINB) skw_iter_kernel(WideArgs a) {
    pdl_launch_dependents();   // the next iteration may set up while this one runs
    constexpr int NC = 4 * NQ, kWT = CFG::T, kWW = CFG::W, kWStage = CFG::STAGE, kWS = CFG::S;
    constexpr int RM = wide_rows_of<CFG, NQ>();   // rows per batch (the host passes a.R == RM)
    constexpr int kP = kWC * kWW;   // pairs per row of a batch: one per warp of the cluster
    constexpr int kPL = kP / 32;    // pairs per lane in the merge
    static_assert(kP % 32 == 0, "warps per cluster must be a multiple of 32");
    extern __shared__ __align__(128) unsigned char smem[];
    float2* xch = reinterpret_cast<float2*>(smem + size_t(kWS) * kWStage);   // [kWX][R][kP]
    __shared__ __align__(8) uint64_t full[kWS];   // a stage's rows have landed (bulk-copy bytes)
    __shared__ __align__(8) uint64_t xbar[kWX];   // a batch's row pairs from every warp of the cluster have landed
    __shared__ __align__(8) uint64_t ubar[kWX];   // a batch's u is in s_uv
    __shared__ float s_uv[kWX][kWMaxR];
    __shared__ unsigned s_rel[kWS];               // warps done with a stage (wrapping counter)
    __shared__ int s_flag, s_nfix, s_next, s_kfail;
    __shared__ volatile int s_abort;              // a bounded wait expired: stop copying and waiting
    __shared__ int s_fix[kWFix];

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const uint32_t rank = w_rank(), cid = w_cid();
    const int64_t n = a.n, m = a.m, mc = a.mc;
    const int64_t cbase = int64_t(rank) * mc;
    const int g0 = w_q(a, int(cid)), g1 = w_q(a, int(cid) + 1);
    auto live = [&](int q) -> bool { return FULL || (4 * tid + 4 * kWT * q) < mc; };
    auto sidx = [&](int g) -> int { return (g - g0) % kWS; };
    auto sphase = [&](int g) -> uint32_t { return uint32_t(((g - g0) / kWS) & 1); };
    auto stage = [&](int g) -> float* { return reinterpret_cast<float*>(smem + size_t(sidx(g)) * kWStage); };
    auto xidx = [&](int g) -> int { return (g - g0) % kWX; };
    auto xphase = [&](int g) -> uint32_t { return uint32_t(((g - g0) / kWX) & 1); };
    auto rows_of = [&](int g) -> int {
        const int jb = g % a.nbat;
        return int(min(int64_t(a.R), n - int64_t(jb) * a.R));
    };
    auto issue = [&](int g) {   // one thread
        const int b = g / a.nbat, jb = g - b * a.nbat;
        const int rows = rows_of(g);
        const uint32_t bytes = uint32_t(mc) * 4u;
        uint64_t* bb = &full[sidx(g)];
        mbar_arrive_expect_tx(bb, bytes * uint32_t(rows));
        const float* src = a.X + (int64_t(b) * n + int64_t(jb) * a.R) * m + cbase;
        for (int r = 0; r < rows; ++r) bulk_g2s(stage(g) + int64_t(r) * mc, src + int64_t(r) * m, bytes, bb);
        s_next = g + 1;
    };
    auto wait_full = [&](int g) -> bool {
        if (s_abort) return false;
        const bool r = mbar_wait_sleep(&full[sidx(g)], sphase(g), a.err);
        if (!r) s_abort = 1;
        return r;
    };
    auto wait_pairs = [&](int g) -> bool {
        if (s_abort) return false;
        const bool r = mbar_wait_cluster(&xbar[xidx(g)], xphase(g), a.err);
        if (!r) s_abort = 1;
        return r;
    };

    if (tid == 0) {
#pragma unroll
        for (int k = 0; k < kWS; ++k) {
            mbar_init(&full[k], 1);
            s_rel[k] = 0u;
        }
#pragma unroll
        for (int k = 0; k < kWX; ++k) {
            mbar_init(&xbar[k], 1);
            mbar_init(&ubar[k], 1);
        }
        s_abort = 0;
        s_nfix = 0;
        s_next = g0;
        s_kfail = g1;
        mbar_fence_init();
    }
    __syncthreads();
    w_arrive();   // every CTA of the cluster has initialised its barriers before a pair is sent to it
    w_wait();
    if (tid == 0)
        for (int g = g0; g < g1 && g < g0 + kWS; ++g) issue(g);
    // programmatic dependent launch: the set-up and first copies of the
    // (read-only) matrix above may overlap the previous kernel; v, u and the
    // merge buffers are touched only after it has completed
    pdl_wait();

    float vr[NC], cS[NC];
    float A = kNegBig;               // warp-wide column reference
    float tmc[RM], tmp[RM];  // warp row maxima: current batch, pending batch
    float crc[RM], crp[RM];  // their rounding remainders (mx*log2e - round(mx*log2e))
    float uw[RM];            // u of the pending batch's rows
    int cur = -1, pend = -1;

    auto load_v = [&](int b) {
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            const float4 v4 = live(q) ? __ldcg(reinterpret_cast<const float4*>(a.v2 + int64_t(b) * m + cbase +
                                                                              4 * tid + 4 * kWT * q))
                                      : make_float4(0, 0, 0, 0);
            vr[4 * q + 0] = v4.x;
            vr[4 * q + 1] = v4.y;
            vr[4 * q + 2] = v4.z;
            vr[4 * q + 3] = v4.w;
        }
#pragma unroll
        for (int e = 0; e < NC; ++e) cS[e] = 0.0f;
        A = kNegBig;
    };

    // u of batch gp's rows from the kP pairs of each row (every warp of the
    // cluster sent one), merged by one warp of the CTA (rotating with gp): max
    // over the lanes, then the rescaled sums added in a fixed order, so every
    // CTA gets the same value.  It is published in s_uv behind ubar; the
    // merging warp writes it out before its CTA's flush arrival.
    auto take_u = [&](int gp, int rp, int64_t grow0) {
        const int slot = xidx(gp);
        if (wid == (gp - g0) % kWW) {
            wait_pairs(gp);
            const float2* xs = xch + slot * a.R * kP;
#pragma unroll
            for (int ir = 0; ir < RM; ++ir) {
                if (ir < rp) {
                    float2 q[kPL];
                    float ml = kNegBig;
#pragma unroll
                    for (int k = 0; k < kPL; ++k) {
                        q[k] = xs[ir * kP + lane + 32 * k];
                        ml = fmaxf(ml, q[k].x);
                    }
                    const float mm = warp_max<32>(ml);
                    float sl = 0.0f;
#pragma unroll
                    for (int k = 0; k < kPL; ++k) sl = fmaf(q[k].y, exp_shift(q[k].x - mm), sl);
                    const float ss = warp_sum<32>(sl);
                    if (lane == 0) {
                        const int64_t grow = grow0 + ir;
                        const float u = (a.la ? __ldg(a.la + grow) : a.la_def) - lse_finish(mm, ss);
                        s_uv[slot][ir] = u;
                        a.u2[grow] = u;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&ubar[slot]);
        }
        if (!s_abort && !mbar_wait_sleep(&ubar[slot], xphase(gp), a.err)) s_abort = 1;
#pragma unroll
        for (int ir = 0; ir < RM; ++ir) uw[ir] = s_uv[slot][ir];
    };

    // column update of batch gp (E in its stage, u in uw); the last warp
    // done with the stage refills it
    auto pass_b = [&](int gp, int rows) {
        const float* es = stage(gp);
        if (!s_abort) {
#pragma unroll
            for (int ir = 0; ir < RM; ++ir) {
                if (ir < rows) {
                    const float ai = tmp[ir] + uw[ir];   // warp-uniform
                    if (ai > A + kRaiseW) {
                        const float sc = exp_shift(A - ai);
#pragma unroll
                        for (int e = 0; e < NC; ++e) cS[e] *= sc;
                        A = ai;
                    }
                    const float w = ex2(fmaf(ai - A, kLog2e, -crp[ir]));   // exp(ai - A) / 2^cr
#pragma unroll
                    for (int q = 0; q < NQ; ++q) {
                        if (live(q)) {
                            const float4 e4 =
                                *reinterpret_cast<const float4*>(es + ir * int(mc) + 4 * tid + 4 * kWT * q);
                            cS[4 * q + 0] = fmaf(e4.x, w, cS[4 * q + 0]);
                            cS[4 * q + 1] = fmaf(e4.y, w, cS[4 * q + 1]);
                            cS[4 * q + 2] = fmaf(e4.z, w, cS[4 * q + 2]);
                            cS[4 * q + 3] = fmaf(e4.w, w, cS[4 * q + 3]);
                        }
                    }
                }
            }
        }
        fence_proxy_async_smem();   // this thread's E stores before the stage's bulk-copy refill
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            if (atomicInc(&s_rel[sidx(gp)], unsigned(kWW - 1)) == unsigned(kWW - 1)) {
                __threadfence_block();
                if (gp + kWS < g1 && !s_abort) issue(gp + kWS);
            }
        }
    };

    // publish this CTA's column partials of problem b; the last same-rank
    // CTA over the problem's clusters merges the slice
    auto flush = [&](int b) {
        const int kfirst = w_owner(a, b * a.nbat);
        const int nseg = w_owner(a, (b + 1) * a.nbat - 1) - kfirst + 1;
        const int seg = int(cid) - kfirst;
        float2* mypart = a.part + (int64_t(b) * a.maxseg + seg) * m + cbase;
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            if (live(q)) {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    mypart[4 * tid + 4 * kWT * q + e] = make_float2(A - vr[4 * q + e], cS[4 * q + e]);
            }
        }
        if (a.pairs != nullptr) return;   // skw_pairs_merge_kernel merges them
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            s_flag = (atomicAdd(a.cnt + int64_t(b) * kWC + rank, 1) == nseg - 1) ? 1 : 0;
            s_nfix = 0;
        }
        __syncthreads();
        if (s_flag == 0) return;
        __threadfence();
        // the slice's columns over the segments in order: max pass, then the
        // rescaled sums (one exponential per partial); four columns per thread
        // at a time, so four independent chains are in flight
        const float2* pb = a.part + int64_t(b) * a.maxseg * m + cbase;
        constexpr int kCols = 4;
        for (int64_t lc0 = tid; lc0 < mc; lc0 += kCols * kWT) {
            float mm[kCols], ss[kCols];
#pragma unroll
            for (int c = 0; c < kCols; ++c) {
                mm[c] = kNegBig;
                ss[c] = 0.0f;
            }
            for (int sg = 0; sg < nseg; ++sg) {
#pragma unroll
                for (int c = 0; c < kCols; ++c) {
                    const int64_t lc = lc0 + int64_t(c) * kWT;
                    if (lc < mc) mm[c] = fmaxf(mm[c], __ldcg(pb + int64_t(sg) * m + lc).x);
                }
            }
            for (int sg = 0; sg < nseg; ++sg) {
#pragma unroll
                for (int c = 0; c < kCols; ++c) {
                    const int64_t lc = lc0 + int64_t(c) * kWT;
                    if (lc < mc) {
                        const float2 pp = __ldcg(pb + int64_t(sg) * m + lc);
                        ss[c] = fmaf(pp.y, exp_shift(pp.x - mm[c]), ss[c]);
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < kCols; ++c) {
                const int64_t lc = lc0 + int64_t(c) * kWT;
                if (lc >= mc) continue;
                const int64_t col = cbase + lc;
                if (ss[c] < kTinyW) {
                    const int k = atomicAdd(&s_nfix, 1);
                    if (k < kWFix) s_fix[k] = int(lc);
                    else a.v2[int64_t(b) * m + col] = (a.lb ? a.lb[int64_t(b) * m + col] : a.lb_def) -
                                                      lse_finish(mm[c], ss[c]);
                } else {
                    a.v2[int64_t(b) * m + col] = (a.lb ? a.lb[int64_t(b) * m + col] : a.lb_def) -
                                                 lse_finish(mm[c], ss[c]);
                }
            }
        }
        if (tid == 0) a.cnt[int64_t(b) * kWC + rank] = 0;
        __syncthreads();
        const int nfix = min(s_nfix, kWFix);
        for (int k = wid; k < nfix; k += kWW) {
            const int64_t col = cbase + s_fix[k];
            const float lse = w_exact_column(a.X, a.u2, a.kinv, b, n, m, col);
            if (lane == 0) a.v2[int64_t(b) * m + col] = (a.lb ? a.lb[int64_t(b) * m + col] : a.lb_def) - lse;
        }
        __syncthreads();
    };

    // Warps run decoupled: each waits for its stage, sends its own row pairs
    // and takes u itself; they meet only at problem boundaries (flush).
    // batch coordinates advance incrementally (no division per batch)
    int b = g0 / a.nbat, jb = g0 - b * a.nbat;
    int prows = 0;
    int64_t pgrow0 = 0;
    for (int g = g0; g < g1; ++g) {
        if (b != cur) {
            if (pend >= 0) {   // finish the previous problem's last batch
                take_u(pend, prows, pgrow0);
                pass_b(pend, prows);
                pend = -1;
            }
            if (cur >= 0) flush(cur);
            cur = b;
            load_v(b);
        }
        const int rows = min(a.R, int(n - int64_t(jb) * a.R));
        const int64_t grow0 = int64_t(b) * n + int64_t(jb) * a.R;
        if (tid == 0) mbar_arrive_expect_tx(&xbar[xidx(g)], uint32_t(rows * kP) * uint32_t(sizeof(float2)));
        const bool ok = __all_sync(0xffffffffu, wait_full(g));
        if (!ok && lane == 0) atomicMin(&s_kfail, g);

        // ---- pass A: row partials of this warp's columns; E written in place ----
        float* xs = stage(g);
#pragma unroll
        for (int ir = 0; ir < RM; ++ir) {
            if (ir < rows) {
                float mx = kNegBig, s = 0.0f;
                crc[ir] = 0.0f;
                if (ok) {
                    float t[NC];
#pragma unroll
                    for (int q = 0; q < NQ; ++q) {
                        if (live(q)) {
                            const float4 x =
                                *reinterpret_cast<const float4*>(xs + ir * int(mc) + 4 * tid + 4 * kWT * q);
                            t[4 * q + 0] = kplus(x.x, a.kinv, vr[4 * q + 0]);
                            t[4 * q + 1] = kplus(x.y, a.kinv, vr[4 * q + 1]);
                            t[4 * q + 2] = kplus(x.z, a.kinv, vr[4 * q + 2]);
                            t[4 * q + 3] = kplus(x.w, a.kinv, vr[4 * q + 3]);
                        } else {
                            t[4 * q + 0] = t[4 * q + 1] = t[4 * q + 2] = t[4 * q + 3] = -INFINITY;
                        }
                    }
                    mx = warp_max<32>(fmaxf(mx, tree_max(t)));
                    // exp(t - mx) as 2^(t*log2e - mL) in one FFMA, mL = mx*log2e
                    // rounded; every term carries 2^cr, cr = mx*log2e - mL exactly
                    // (FMA remainder), taken out of the sum here and out of the
                    // column weight in pass B
                    const float mxc = fmaxf(mx, -1.0e37f);   // a row of -inf terms keeps mL finite
                    const float mL = mxc * kLog2e;
                    crc[ir] = fmaf(mxc, kLog2e, -mL);
#pragma unroll
                    for (int e = 0; e < NC; ++e) t[e] = ex2(fmaf(t[e], kLog2e, -mL));
                    s = warp_sum<32>(tree_sum(t)) * ex2(-crc[ir]);
#pragma unroll
                    for (int q = 0; q < NQ; ++q) {
                        if (live(q))
                            *reinterpret_cast<float4*>(xs + ir * int(mc) + 4 * tid + 4 * kWT * q) =
                                make_float4(t[4 * q + 0], t[4 * q + 1], t[4 * q + 2], t[4 * q + 3]);
                    }
                }
                tmc[ir] = mx;
                if (lane < kWC) {   // this warp's pair of row ir to CTA `lane` of the cluster
                    const float2* dst = xch + (xidx(g) * a.R + ir) * kP + int(rank) * kWW + wid;
                    st_async_f2(cluster_map(dst, uint32_t(lane)), cluster_map(&xbar[xidx(g)], uint32_t(lane)),
                                make_float2(mx, s));
                }
            }
        }
        if (pend >= 0) {   // its pairs had this batch's pass A to arrive
            take_u(pend, prows, pgrow0);
            pass_b(pend, prows);
        }
#pragma unroll
        for (int ir = 0; ir < RM; ++ir) {
            tmp[ir] = tmc[ir];
            crp[ir] = crc[ir];
        }
        pend = g;
        prows = rows;
        pgrow0 = grow0;
        if (++jb == a.nbat) {
            jb = 0;
            ++b;
        }
    }
    if (pend >= 0) {
        take_u(pend, prows, pgrow0);
        pass_b(pend, prows);
    }
    if (cur >= 0) flush(cur);
    __syncthreads();
    if (tid == 0)   // copies still in flight after a failed wait
        for (int g = s_kfail; g < s_next && g < s_kfail + kWS; ++g)
            mbar_wait_sleep(&full[sidx(g)], sphase(g), nullptr);
    w_arrive();   // no CTA leaves while a peer may still store into its shared memory
    w_wait();
}

// Row-shard mode: merge the published column partials of every problem over
// the clusters that touched it, in cluster order (max pass, then the
// rescaled sums -- the arithmetic of the in-kernel slice merge), into the
// (max, sum) pairs [B][m].  One thread per column; segment loads are issued
// eight at a time so a thread waits on L2 about nseg/4 times in all.  A
// column whose merged sum is too small to trust (kTinyW, as in the in-kernel
// merge) gets its pair recomputed exactly over the shard's rows by one warp
// of the CTA, so the cross-shard merge never starts from an underflowed sum.
constexpr int kMT = 128;   // threads per merge CTA
constexpr int kMU = 8;     // segment loads in flight per thread
__global__ void __launch_bounds__(kMT) skw_pairs_merge_kernel(WideArgs a, int64_t B) {
    __shared__ int s_fix[kMT];
    __shared__ int s_nfix;
    pdl_launch_dependents();
    if (threadIdx.x == 0) s_nfix = 0;
    pdl_wait();   // the iteration kernel's partials are complete and visible
    __syncthreads();
    const int64_t idx = int64_t(blockIdx.x) * kMT + threadIdx.x;
    if (idx < B * a.m) {
        const int b = int(idx / a.m);
        const int64_t col = idx - int64_t(b) * a.m;
        const int kfirst = w_owner(a, b * a.nbat);
        const int nseg = w_owner(a, (b + 1) * a.nbat - 1) - kfirst + 1;
        const float2* pc = a.part + int64_t(b) * a.maxseg * a.m + col;
        float mm = kNegBig;
        for (int s0 = 0; s0 < nseg; s0 += kMU) {
            float x[kMU];
#pragma unroll
            for (int k = 0; k < kMU; ++k) x[k] = s0 + k < nseg ? __ldcg(&pc[int64_t(s0 + k) * a.m].x) : kNegBig;
#pragma unroll
            for (int k = 0; k < kMU; ++k) mm = fmaxf(mm, x[k]);
        }
        float ss = 0.0f;
        for (int s0 = 0; s0 < nseg; s0 += kMU) {
            float2 pp[kMU];
#pragma unroll
            for (int k = 0; k < kMU; ++k)
                pp[k] = s0 + k < nseg ? __ldcg(pc + int64_t(s0 + k) * a.m) : make_float2(kNegBig, 0.0f);
#pragma unroll
            for (int k = 0; k < kMU; ++k)
                if (s0 + k < nseg) ss = fmaf(pp[k].y, exp_shift(pp[k].x - mm), ss);
        }
        if (ss < kTinyW) s_fix[atomicAdd(&s_nfix, 1)] = int(threadIdx.x);
        else a.pairs[idx] = make_float2(mm, ss);
    }
    __syncthreads();
    const int nfix = s_nfix;
    for (int k = int(threadIdx.x >> 5); k < nfix; k += kMT / 32) {
        const int64_t j = int64_t(blockIdx.x) * kMT + s_fix[k];
        const int b = int(j / a.m);
        const float2 p = w_exact_pair(a.X, a.u2, a.kinv, b, a.n, a.m, j - int64_t(b) * a.m);
        if ((threadIdx.x & 31) == 0) a.pairs[j] = p;
    }
}

// Stages plus the pair-exchange slots for batches of R rows.
template <class CFG>
size_t wide_smem(int R) { return size_t(CFG::S) * CFG::STAGE + size_t(kWX) * R * kWC * CFG::W * sizeof(float2); }

template <class CFG>
cudaLaunchConfig_t wide_config(int grid, int R, cudaStream_t st, cudaLaunchAttribute* attr, bool pdl = false) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(grid));
    cfg.blockDim = dim3(CFG::T);
    cfg.dynamicSmemBytes = wide_smem<CFG>(R);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kWC;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (pdl) {   // attr holds two entries
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs = 2;
    }
    return cfg;
}

// CTA shape: b (two 256-thread CTAs per SM) where the slice fits it,
// mc <= 4096 columns, else a (one 512-thread CTA per SM).
int wide_shape(int64_t mc) { return mc <= 4096 ? kShapeB : kShapeA; }

template <class CFG>
int nq_of(int64_t mc) {
    const int64_t per = 4 * CFG::T;
    return mc <= per ? 1 : mc <= 2 * per ? 2 : 4;
}

// Consecutive forward iterations overlap through programmatic dependent
// launch.  A row shard's iteration follows the column merge instead, and
// there the programmatic launch measured twice the iteration time on one GPU
// (2307 vs 1254 us per 32768^2 iteration), so row shards launch plainly.
template <class CFG, int NQ>
void launch_nq(const WideArgs& a, cudaStream_t st) {
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = wide_config<CFG>(a.G * kWC, a.R, st, attr, a.pairs == nullptr);
    if (a.mc == 4 * CFG::T * NQ) cudaLaunchKernelEx(&cfg, skw_iter_kernel<CFG, NQ, true>, a);
    else cudaLaunchKernelEx(&cfg, skw_iter_kernel<CFG, NQ, false>, a);
}

template <class CFG>
void launch_cfg(const WideArgs& a, cudaStream_t st) {
    switch (nq_of<CFG>(a.mc)) {
        case 1: launch_nq<CFG, 1>(a, st); break;
        case 2: launch_nq<CFG, 2>(a, st); break;
        default: launch_nq<CFG, 4>(a, st); break;
    }
}

template <class CFG>
void set_attr_cfg() {
    const int bytes = int(wide_smem<CFG>(kWMaxR));
    cudaFuncSetAttribute(skw_iter_kernel<CFG, 1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(skw_iter_kernel<CFG, 1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(skw_iter_kernel<CFG, 2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(skw_iter_kernel<CFG, 2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(skw_iter_kernel<CFG, 4, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    cudaFuncSetAttribute(skw_iter_kernel<CFG, 4, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

template <class CFG>
int occupancy_clusters(int R) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = wide_config<CFG>(kWC, R, nullptr, attr);
    int ncl = 0;
    if (cudaOccupancyMaxActiveClusters(&ncl, skw_iter_kernel<CFG, 4, true>, &cfg) != cudaSuccess || ncl < 1) {
        cudaGetLastError();
        ncl = 1;
    }
    return ncl;
}

void launch_any(const WideArgs& a, cudaStream_t st) {
    if (wide_shape(a.mc) == kShapeA) launch_cfg<WideA>(a, st);
    else launch_cfg<WideB>(a, st);
}

// Resident clusters of the shape with R-row batches on this device (cached
// per device).
int max_clusters(int shape, int R) {
    static int cached[2][kWMaxR + 1][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && cached[shape][R][dev] > 0) return cached[shape][R][dev];
    set_attr_cfg<WideA>();
    set_attr_cfg<WideB>();
    const int ncl = shape == kShapeA ? occupancy_clusters<WideA>(R) : occupancy_clusters<WideB>(R);
    if (dev >= 0 && dev < 64) cached[shape][R][dev] = ncl;
    return ncl;
}

// Rows per batch of the shape for slices of mc columns (wide_rows_of).
int wide_rows(int64_t mc) {
    if (wide_shape(mc) == kShapeA) {
        const int q = nq_of<WideA>(mc);
        return q == 1 ? wide_rows_of<WideA, 1>() : q == 2 ? wide_rows_of<WideA, 2>() : wide_rows_of<WideA, 4>();
    }
    const int q = nq_of<WideB>(mc);
    return q == 1 ? wide_rows_of<WideB, 1>() : q == 2 ? wide_rows_of<WideB, 2>() : wide_rows_of<WideB, 4>();
}

struct WidePlan {
    int R, nbat, TB, G, maxseg;
    int64_t mc;
};

WidePlan wide_plan(int64_t B, int64_t n, int64_t m) {
    WidePlan p;
    p.mc = m / kWC;
    p.R = wide_rows(p.mc);
    p.nbat = int((n + p.R - 1) / p.R);
    p.TB = int(B * p.nbat);
    p.G = int(std::min<int64_t>(max_clusters(wide_shape(p.mc), p.R), p.TB));
    WideArgs tmp{};
    tmp.TB = p.TB;
    tmp.G = p.G;
    p.maxseg = 1;
    for (int b = 0; b < int(B); ++b) {
        const int k0 = w_owner(tmp, b * p.nbat), k1 = w_owner(tmp, (b + 1) * p.nbat - 1);
        p.maxseg = std::max(p.maxseg, k1 - k0 + 1);
    }
    return p;
}

// Segment slots: a problem of nbat batches meets at most (nbat-1)*G/TB + 2
// of the G ranges; bounded without the device by G <= 64 (a 148-SM part
// holds at most 2 * 148 / kWC = 37 clusters of these CTAs).
int64_t wide_seg_bound(int64_t B, int64_t n, int64_t m) {
    const int64_t mc = m / kWC, R = wide_rows(mc);
    const int64_t nbat = (n + R - 1) / R, TB = B * nbat;
    const int64_t G = std::min<int64_t>(TB, 64);
    return std::min<int64_t>(G, (nbat - 1) * G / TB + 2);
}

}  // namespace

bool sk_wide_supported(int64_t B, int64_t n, int64_t m, const void* X) {
    if (B < 1 || n < 1 || m < 8192 || m > 65536 || (m % 32) != 0) return false;
    if ((reinterpret_cast<uintptr_t>(X) & 15u) != 0) return false;
    const int64_t mc = m / kWC, R = wide_rows(mc);
    return B * ((n + R - 1) / R) < (int64_t(1) << 31);
}

size_t sk_wide_ws(int64_t B, int64_t n, int64_t m) {
    Carve c(nullptr);
    c.take<float2>(size_t(B * wide_seg_bound(B, n, m) * m));
    c.take<int32_t>(size_t(B * kWC));
    return c.size();
}

// All forward iterations (single GPU: v is merged in the kernels); records
// the potentials after every iteration when a.u_hist / a.v_hist are set.
int sk_wide_fwd(const SkFwdArgs& a, void* ws, cudaStream_t st) {
    const WidePlan p = wide_plan(a.B, a.n, a.m);
    if (p.maxseg > wide_seg_bound(a.B, a.n, a.m))
        return fail(DOT_ERR_WORKSPACE, "wide Sinkhorn: more row segments than the workspace holds");
    Carve c(ws);
    WideArgs w{};
    w.part = c.take<float2>(size_t(a.B * wide_seg_bound(a.B, a.n, a.m) * a.m));
    w.cnt = c.take<int32_t>(size_t(a.B * kWC));
    cudaMemsetAsync(w.cnt, 0, sizeof(int32_t) * size_t(a.B * kWC), st);
    w.X = a.X;
    w.kinv = a.kinv;
    w.la = a.la;
    w.la_def = a.la_def;
    w.lb = a.lb;
    w.lb_def = a.lb_def;
    w.u2 = a.u2;
    w.v2 = a.v2;
    w.n = a.n;
    w.m = a.m;
    w.mc = p.mc;
    w.R = p.R;
    w.nbat = p.nbat;
    w.TB = p.TB;
    w.G = p.G;
    w.maxseg = int(wide_seg_bound(a.B, a.n, a.m));
    w.pairs = nullptr;
    w.err = a.status + 3;
    const int64_t rows = a.B * a.n;
    const bool hist = a.u_hist != nullptr && a.v_hist != nullptr;
    ProfScope ps(DOT_K_SK_FWD_ITER, st, a.n_iters);
    for (int it = 0; it < a.n_iters; ++it) {
        launch_any(w, st);
        if (hist) {
            cudaMemcpyAsync(a.u_hist + int64_t(it) * rows, a.u2, sizeof(float) * size_t(rows),
                            cudaMemcpyDeviceToDevice, st);
            cudaMemcpyAsync(a.v_hist + int64_t(it) * a.B * a.m, a.v2, sizeof(float) * size_t(a.B * a.m),
                            cudaMemcpyDeviceToDevice, st);
        }
    }
    return check_launch("sinkhorn forward (wide rows)");
}

// One row half-step and the shard's column pairs for a row shard.
int sk_wide_rows_pairs(const float* X, float kinv, const float* la, float la_def, int64_t B, int64_t n, int64_t m,
                       const float* v2, float* u2, float2* pairs, int32_t* err, void* ws, cudaStream_t st) {
    const WidePlan p = wide_plan(B, n, m);
    if (p.maxseg > wide_seg_bound(B, n, m))
        return fail(DOT_ERR_WORKSPACE, "wide Sinkhorn: more row segments than the workspace holds");
    Carve c(ws);
    WideArgs w{};
    w.part = c.take<float2>(size_t(B * wide_seg_bound(B, n, m) * m));
    w.cnt = c.take<int32_t>(size_t(B * kWC));   // unused: no arrival counting in this mode
    w.X = X;
    w.kinv = kinv;
    w.la = la;
    w.la_def = la_def;
    w.lb = nullptr;
    w.lb_def = 0.0f;
    w.u2 = u2;
    w.v2 = const_cast<float*>(v2);
    w.n = n;
    w.m = m;
    w.mc = p.mc;
    w.R = p.R;
    w.nbat = p.nbat;
    w.TB = p.TB;
    w.G = p.G;
    w.maxseg = int(wide_seg_bound(B, n, m));
    w.pairs = pairs;
    w.err = err;
    {
        ProfScope ps(DOT_K_SK_FWD_ITER, st);
        launch_any(w, st);
    }
    // the pair merge starts (PDL) while the iteration kernel drains
    ProfScope ps(DOT_K_SK_EXCHANGE, st);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned((B * m + kMT - 1) / kMT));
    cfg.blockDim = dim3(kMT);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, skw_pairs_merge_kernel, w, B);
    return check_launch("sinkhorn rows + column pairs (wide rows)");
}

}  // namespace dotb

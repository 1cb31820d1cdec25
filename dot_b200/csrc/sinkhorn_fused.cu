// Fused single-pass Sinkhorn iterations for m <= 1024 (m % 4 == 0).
//
// One kernel launch per iteration reads the B x n x m matrix once (the
// streaming two-kernel path in sinkhorn_stream.cu reads it twice):
//
//   forward   for each row i:   u_i = la_i - LSE_j(K_ij + v_j)
//             then, with the fresh u, per-column partials of LSE_i(K_ij + u_i)
//   backward  lambda_i = (sum_k P G - sum_k P_ik mu_k) / max(sum_k P, 1e-12)
//             then per-column partials of sum_i P_ik lambda_i
//
// This is exactly the reference's Gauss-Seidel order (u from the previous v,
// v from the new u: src/sinkhorn/torch_cuda.cpp:200-223; lambda from the
// previous mu, mu from the new lambda: kernels.cu:1715-1718).
//
// Work decomposition (persistent, balanced): every problem is cut into row
// blocks of R rows (R*m <= 8192 floats, 32 KB); the B*nblk blocks, in memory
// order, are split into G contiguous ranges of equal length, one per CTA,
// with G = the number of CTAs the GPU holds at once (one wave).  A CTA
// streams its range through shared memory with an S-stage ring of 1-D bulk
// copies (cp.async.bulk, the TMA engine) completing on mbarriers.  Warp per
// row; each lane owns fixed columns, so after its row's reduction it folds
// the same registers into its columns' running partials.  When the CTA's
// range leaves a problem (or ends), it merges its warps' partials through the
// just-consumed stage buffer and publishes them as that problem's segment
// partial; the CTA that arrives last for a problem (atomic arrival counter,
// no waiting) merges the problem's segments in segment order and writes v
// (or mu), so results are deterministic.  The next launch consumes them.
//
// Launches of consecutive iterations overlap through programmatic dependent
// launch: a CTA initialises its barriers and starts its first bulk copies of
// the (read-only) matrix, then waits for the previous iteration's grid before
// reading the potentials.  Every iteration but the last copies with an L2
// evict_first policy (the matrix streams through L2; keeping a fixed part of
// it resident across iterations with evict_last measured no gain at 48, 64 or
// 96 MiB); the last uses plain copies, which leave the lines at normal
// priority.
#include <cmath>

#include "common.cuh"
#include "internal.h"
#include "pack.cuh"
#include "sinkhorn.h"
#include "tma.cuh"

namespace dotb {

namespace {

constexpr int kFT = 256;              // threads per CTA
constexpr int kFW = kFT / 32;         // warps per CTA
constexpr int kTileFloats = 8192;     // one stage buffer (32 KB)
constexpr int kMergeCols = 512;       // columns merged per round (kFW * 512 * 8 B = 32 KB)

template <int VPL>
struct FCfg {
    static constexpr int R = 64 / VPL;    // rows per block (R * 128 * VPL floats = 32 KB)
    static constexpr int RPW = R / kFW;   // rows per warp per block
    static constexpr int NC = 4 * VPL;    // columns per lane
};

// Balanced schedule: CTA k owns blocks [q(k), q(k+1)), q(k) = floor(k*T/G).
struct Sched {
    int T;           // total blocks B * nblk (< 2^31: sk_fused_supported)
    int nblk;        // blocks per problem
    int G;           // CTAs
    int maxseg;      // max segments (CTAs) touching one problem
    int hint;        // 0: plain copies; 1: evict_first copies
};

__host__ __device__ __forceinline__ int sched_q(const Sched& s, int k) { return int(int64_t(k) * s.T / s.G); }
// The CTA whose range contains block x: the largest k with q(k) <= x.
__host__ __device__ __forceinline__ int sched_owner(const Sched& s, int x) {
    return int((int64_t(x + 1) * s.G + s.T - 1) / s.T) - 1;
}

struct FusedCommon {
    const float* data;   // X (forward) or P (backward), [B, n, m]
    int64_t n, m;
    int R;               // rows per block
    Sched s;
    int32_t* cnt;        // [B] arrival counters, zero between launches
    int32_t* err;        // device error word (bounded-wait timeouts)
};

struct FwdIter {
    FusedCommon c;
    float kinv;
    const float* la;
    float la_def;
    const float* lb;
    float lb_def;
    float* u2;
    float* v2;
    float2* part;        // [B, maxseg, m] column (max, sum) partials
    float* delta;        // tol > 0: per-iteration max |du|; else nullptr
    int32_t* status;
    float tol;
    int iter;
};

struct BwdIter {
    FusedCommon c;
    const float2* rinv;  // [B, n] (sum_k P G, sum_k P)
    const float2* cinv;  // [B, m] (sum_i P G, sum_i P)
    float* lam;
    float* mu;
    float* part;         // [B, maxseg, m] column sums
};

// S-stage ring over the CTA's block range [g0, g1).  Only the range bounds
// live in registers; shapes and schedule come from the kernel parameters.
template <int S>
struct Ring {
    const FusedCommon* c;
    unsigned char* smem; // stage k at smem + k * 32 KB
    uint64_t* bar;       // S mbarriers
    int g0, g1;

    __device__ float* buf(int g) const {
        return reinterpret_cast<float*>(smem) + int((g - g0) % S) * kTileFloats;
    }
    __device__ uint64_t* barrier(int g) const { return bar + (g - g0) % S; }
    __device__ uint32_t parity(int g) const { return uint32_t(((g - g0) / S) & 1); }
    __device__ int rows_in(int g) const {
        const int jb = g % c->s.nblk;
        return int(min(int64_t(c->R), c->n - int64_t(jb) * c->R));
    }
    __device__ void issue(int g) const {   // one thread
        const int b = g / c->s.nblk, jb = g - b * c->s.nblk;
        const uint32_t bytes = uint32_t(rows_in(g)) * uint32_t(c->m) * 4u;
        const float* src = c->data + (int64_t(b) * c->n + int64_t(jb) * c->R) * c->m;
        uint64_t* bb = barrier(g);
        mbar_arrive_expect_tx(bb, bytes);
        if (c->s.hint) {
            bulk_g2s_hint(buf(g), src, bytes, bb, l2_policy_evict_first());
        } else {
            bulk_g2s(buf(g), src, bytes, bb);
        }
    }
    __device__ bool wait(int g, int32_t* err) const { return mbar_wait_sleep(barrier(g), parity(g), err); }
};

template <int S>
__device__ __forceinline__ Ring<S> ring_init(const FusedCommon& c, uint64_t* bars, unsigned char* smem) {
    Ring<S> r;
    r.c = &c;
    r.smem = smem;
    r.bar = bars;
    r.g0 = sched_q(c.s, blockIdx.x);
    r.g1 = sched_q(c.s, int(blockIdx.x) + 1);
    if (threadIdx.x == 0) {
#pragma unroll
        for (int k = 0; k < S; ++k) mbar_init(&bars[k], 1);
        mbar_fence_init();
    }
    __syncthreads();
    return r;
}

template <int S>
__device__ __forceinline__ void ring_prime(const Ring<S>& r) {
    if (threadIdx.x == 0)
        for (int g = r.g0; g < r.g1 && g < r.g0 + S; ++g) r.issue(g);
}

// After a failed wait at block g: wait (bounded) for the copies still in
// flight into this CTA's shared memory before the CTA exits.
template <int S>
__device__ __forceinline__ void ring_drain(const Ring<S>& r, int g, int32_t* err) {
    if (threadIdx.x == 0)
        for (int k = g; k < r.g1 && k < g + S; ++k) r.wait(k, err);
    __syncthreads();
}

// Arrival at the end of a problem segment; returns true (to every thread) in
// the CTA that arrived last for problem b.
__device__ __forceinline__ bool arrive_last(int32_t* cnt, int64_t b, int nseg, int* s_flag) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *s_flag = (atomicAdd(cnt + b, 1) == nseg - 1) ? 1 : 0;
    __syncthreads();
    const bool last = *s_flag != 0;
    if (last) __threadfence();
    return last;
}

// ---------------------------------------------------------------------------
// forward iteration
// ---------------------------------------------------------------------------
// Column partials reuse the row pass's exponentials.  For row i,
//     E_ij = exp(t_ij - mx_i)      (t_ij = K_ij + v_j, computed for the row LSE)
//     exp(K_ij + u_i) = E_ij * exp(a_i) * exp(-v_j),   a_i = mx_i + u_i,
// so a warp keeps, per column, S_j = sum_i E_ij * exp(a_i - A) against one
// warp-wide reference A (raised, with a rescale, only when a row's a_i
// exceeds it by kRaise; a_i = log a_i(marginal) - log(row sum) spans only the
// marginals' range plus log m).  The warp's partial for column j is then the
// (max, sum) pair (A - v_j, S_j): one FFMA per element and no second
// exponential.  Terms whose E_ij flushed to zero (t_ij more than ~87 below
// the row maximum) are dropped; that is exact to fp32 unless column j is that
// far below the maximum of every row, in which case its merged sum comes out
// below 2^-90 of its reference and the merging CTA recomputes the column with
// a max-based LSE over all rows (exact_column).
constexpr float kRaise = 60.0f;
constexpr float kTinySum = 8.077935669463161e-28f;   // 2^-90

// Exact column LSE over all n rows of problem b: LSE_i(K_ij + u_i), max pass
// then sum pass (one warp per column; strided reads, used only for columns
// flagged as too small for the shared-reference partials).
__device__ __forceinline__ float exact_column(const float* X, const float* u2, float kinv, int64_t b,
                                              int64_t n, int64_t m, int64_t col) {
    const int lane = threadIdx.x & 31;
    const float* xb = X + b * n * m + col;
    const float* ub = u2 + b * n;
    float mx = kNegBig;
    for (int64_t i = lane; i < n; i += 32) mx = fmaxf(mx, kplus(__ldcg(xb + i * m), kinv, __ldcg(ub + i)));
    mx = warp_max<32>(mx);
    float sm = 0.0f;
    for (int64_t i = lane; i < n; i += 32) sm += exp_shift(kplus(__ldcg(xb + i * m), kinv, __ldcg(ub + i)) - mx);
    sm = warp_sum<32>(sm);
    return lse_finish(mx, sm);
}

template <int VPL, bool FULL, int S>
__global__ void __launch_bounds__(kFT, (FULL || VPL >= 8 || S >= 3) ? 2 : 3) skf_fwd_iter_kernel(FwdIter a) {
    using Cfg = FCfg<VPL>;
    constexpr int R = Cfg::R, RPW = Cfg::RPW, NC = Cfg::NC;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[S];
    __shared__ float s_dmax[kFW];
    __shared__ int s_flag;
    __shared__ int s_nfix;
    __shared__ int s_fix[1024];
    __shared__ unsigned s_rel[S];        // warps done with a stage (wrapping counter)
    __shared__ int s_issued, s_kfail;    // blocks issued so far; first block whose wait expired
    __shared__ volatile int s_abort;     // a bounded wait expired: stop waiting and copying

    pdl_launch_dependents();
    const FusedCommon& c = a.c;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int64_t m = c.m, n = c.n;
    Ring<S> rg = ring_init<S>(c, bars, smem);
    const bool tolmode = a.delta != nullptr;
    if (!tolmode) ring_prime(rg);   // the matrix is read-only across launches
    pdl_wait();
    if (tolmode) {   // device-side early stop
        if (*reinterpret_cast<volatile int32_t*>(a.status + 2) != 0) return;
        if (a.iter > 0 && __ldcg(a.delta + a.iter - 1) < a.tol) {
            if (blockIdx.x == 0 && tid == 0) {
                a.status[0] = a.iter;
                a.status[1] = 1;
                a.status[2] = 1;
            }
            return;
        }
        ring_prime(rg);
    }
    if (tid == 0) {
        s_nfix = 0;
        s_abort = 0;
        s_kfail = rg.g1;
        s_issued = min(rg.g1, rg.g0 + S);   // ring_prime issued these
#pragma unroll
        for (int k = 0; k < S; ++k) s_rel[k] = 0u;
    }
    __syncthreads();

    auto live = [&](int p) -> bool { return FULL || (4 * lane + 128 * p) < m; };
    // packed two-lane arithmetic (pack.cuh) on element pairs (2k, 2k+1)
    float2 vr[NC / 2], cS[NC / 2];
    float A = kNegBig;   // warp-wide column reference (uniform across the warp)
    float dmax = 0.0f;
    int cur = -1;

    int b = rg.g0 / c.s.nblk, jb = rg.g0 - b * c.s.nblk;   // advanced per block, no division
    for (int g = rg.g0; g < rg.g1; ++g) {
        if (b != cur) {   // first block of a problem in this range
            cur = b;
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                const int64_t col = 4 * lane + 128 * p;
                const float4 v4 = live(p) ? __ldcg(reinterpret_cast<const float4*>(a.v2 + b * m + col))
                                          : make_float4(0, 0, 0, 0);
                vr[2 * p] = make_float2(v4.x, v4.y);
                vr[2 * p + 1] = make_float2(v4.z, v4.w);
            }
#pragma unroll
            for (int k = 0; k < NC / 2; ++k) cS[k] = make_float2(0.0f, 0.0f);
            A = kNegBig;
        }
        const int rj = int(min(int64_t(R), n - int64_t(jb) * R));
        const int64_t grow0 = int64_t(b) * n + int64_t(jb) * R;   // global row of the block's row 0
        float lar[RPW];
#pragma unroll
        for (int q = 0; q < RPW; ++q) {
            const int i = wid + kFW * q;
            lar[q] = (a.la != nullptr && i < rj) ? __ldg(a.la + grow0 + i) : a.la_def;
        }
        // warps run decoupled inside a problem segment: each waits for the
        // stage itself, and the last warp done with it refills it (below)
        const bool ok = __all_sync(0xffffffffu, !s_abort && rg.wait(g, c.err));
        if (!ok && lane == 0) {
            atomicMin(&s_kfail, g);
            s_abort = 1;
        }
        const float* xs = rg.buf(g);
        auto do_row = [&](int q) {
            const int i = wid + kFW * q;
            float2 t[NC / 2];
            const float2 k2 = splat2(a.kinv);
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                if (live(p)) {
                    const float4 x = *reinterpret_cast<const float4*>(xs + i * int(m) + 4 * lane + 128 * p);
                    // K + v: ptxas contracts this packed multiply and add into
                    // one fused multiply-add (measured), so t = fma(X, kinv, v)
                    // rounds once where the reference rounds log_K = X * kinv
                    // first; the two differ by at most one rounding of t
                    t[2 * p] = add2(mul2(make_float2(x.x, x.y), k2), vr[2 * p]);
                    t[2 * p + 1] = add2(mul2(make_float2(x.z, x.w), k2), vr[2 * p + 1]);
                } else {
                    t[2 * p] = t[2 * p + 1] = make_float2(-INFINITY, -INFINITY);
                }
            }
            // row LSE, max pass then sum pass (the reference's two-pass order)
            const float mx = warp_max<32>(max_of(t));
            // exp(t - mx) as 2^(t*log2e - mL) in one FFMA, mL = mx*log2e
            // rounded; cr = mx*log2e - mL exactly (FMA remainder), so every
            // term carries the common factor 2^cr, taken out of the row LSE
            // and out of the column weight below
            const float mxc = fmaxf(mx, -1.0e37f);   // a row of -inf terms keeps mL finite
            const float mL = mxc * kLog2e;
            const float cr = fmaf(mxc, kLog2e, -mL);
            const float2 l2 = splat2(kLog2e), nm = splat2(-mL);
#pragma unroll
            for (int k = 0; k < NC / 2; ++k) {   // t now holds E_ij * 2^cr
                const float2 e = fma2(t[k], l2, nm);
                t[k] = make_float2(ex2(e.x), ex2(e.y));
            }
            const float2 s2 = tree_sum2(t);
            const float s = warp_sum<32>(s2.x + s2.y);
            const int64_t grow = grow0 + i;
            const float unew = lar[q] - (mx + (fast_log(fmaxf(s, kSumFloor)) - cr * kLn2));
            if (lane == 0) {
                if (tolmode) dmax = fmaxf(dmax, fabsf(unew - __ldcg(a.u2 + grow)));
                a.u2[grow] = unew;
            }
            const float ai = mx + unew;
            if (ai > A + kRaise) {            // warp-uniform
                const float2 sc = splat2(exp_shift(A - ai));
#pragma unroll
                for (int k = 0; k < NC / 2; ++k) cS[k] = mul2(cS[k], sc);
                A = ai;
            }
            const float2 w = splat2(ex2(fmaf(ai - A, kLog2e, -cr)));   // exp(ai - A) / 2^cr
#pragma unroll
            for (int k = 0; k < NC / 2; ++k) cS[k] = fma2(t[k], w, cS[k]);
        };
        // all of the warp's rows of a full block at once: the RPW rows' chains
        // (loads, maxima, exponentials, sums and their warp reductions)
        // interleave; the column updates then follow in row order, as in do_row
        auto do_rows = [&]() {
            float2 t[RPW][NC / 2];
            const float2 k2 = splat2(a.kinv), l2 = splat2(kLog2e);
#pragma unroll
            for (int q = 0; q < RPW; ++q) {
                const int i = wid + kFW * q;
#pragma unroll
                for (int p = 0; p < VPL; ++p) {
                    const float4 x = *reinterpret_cast<const float4*>(xs + i * int(m) + 4 * lane + 128 * p);
                    t[q][2 * p] = add2(mul2(make_float2(x.x, x.y), k2), vr[2 * p]);
                    t[q][2 * p + 1] = add2(mul2(make_float2(x.z, x.w), k2), vr[2 * p + 1]);
                }
            }
            float mx[RPW], cr[RPW], sl[RPW];
#pragma unroll
            for (int q = 0; q < RPW; ++q) mx[q] = max_of(t[q]);
#pragma unroll
            for (int q = 0; q < RPW; ++q) mx[q] = warp_max<32>(mx[q]);
#pragma unroll
            for (int q = 0; q < RPW; ++q) {
                const float mxc = fmaxf(mx[q], -1.0e37f);
                const float mL = mxc * kLog2e;
                cr[q] = fmaf(mxc, kLog2e, -mL);
                const float2 nm = splat2(-mL);
#pragma unroll
                for (int k = 0; k < NC / 2; ++k) {
                    const float2 e = fma2(t[q][k], l2, nm);
                    t[q][k] = make_float2(ex2(e.x), ex2(e.y));
                }
                const float2 s2 = tree_sum2(t[q]);
                sl[q] = s2.x + s2.y;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
                for (int q = 0; q < RPW; ++q) sl[q] += __shfl_xor_sync(0xffffffffu, sl[q], off);
            }
#pragma unroll
            for (int q = 0; q < RPW; ++q) {
                const int64_t grow = grow0 + wid + kFW * q;
                const float unew = lar[q] - (mx[q] + (fast_log(fmaxf(sl[q], kSumFloor)) - cr[q] * kLn2));
                if (lane == 0) {
                    if (tolmode) dmax = fmaxf(dmax, fabsf(unew - __ldcg(a.u2 + grow)));
                    a.u2[grow] = unew;
                }
                const float ai = mx[q] + unew;
                if (ai > A + kRaise) {            // warp-uniform
                    const float2 sc = splat2(exp_shift(A - ai));
#pragma unroll
                    for (int k = 0; k < NC / 2; ++k) cS[k] = mul2(cS[k], sc);
                    A = ai;
                }
                const float2 w = splat2(ex2(fmaf(ai - A, kLog2e, -cr[q])));   // exp(ai - A) / 2^cr
#pragma unroll
                for (int k = 0; k < NC / 2; ++k) cS[k] = fma2(t[q][k], w, cS[k]);
            }
        };
        if (!ok) {
        } else if (FULL && rj == R) {
            do_rows();
        } else if (rj == R) {
#pragma unroll
            for (int q = 0; q < RPW; ++q) do_row(q);
        } else {
            for (int q = 0; q < RPW; ++q)
                if (wid + kFW * q < rj) do_row(q);
        }

        if (g + 1 != rg.g1 && jb + 1 != c.s.nblk) {
            // inside a segment: release the stage; the last warp to do so
            // issues the copy of block g + S into it
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();
                const int st = (g - rg.g0) % S;
                if (atomicInc(&s_rel[st], unsigned(kFW - 1)) == unsigned(kFW - 1)) {
                    __threadfence_block();
                    if (g + S < rg.g1 && !s_abort) {
                        rg.issue(g + S);
                        s_issued = g + S + 1;
                    }
                }
            }
        } else {
            __syncthreads();   // every warp is done with the segment's rows (and with stage g)
            if (__syncthreads_or(s_abort)) {   // results are void; keep the barrier sequence
                if (++jb == c.s.nblk) {
                    jb = 0;
                    ++b;
                }
                continue;
            }
            // ---- end of this CTA's part of problem b: publish its column partials ----
            const int kfirst = sched_owner(c.s, b * c.s.nblk);
            const int nseg = sched_owner(c.s, (b + 1) * c.s.nblk - 1) - kfirst + 1;
            const int seg = int(blockIdx.x) - kfirst;
            float2* mb = reinterpret_cast<float2*>(rg.buf(g));   // [kFW][kMergeCols]
            float2* mypart = a.part + (b * c.s.maxseg + seg) * m;
            auto finish = [&](int64_t col, float mm, float ss) {
                if (ss < kTinySum) s_fix[atomicAdd(&s_nfix, 1)] = int(col);
                else a.v2[b * m + col] = (a.lb ? a.lb[b * m + col] : a.lb_def) - lse_finish(mm, ss);
            };
#pragma unroll
            for (int ch = 0; ch < (VPL + 3) / 4; ++ch) {
#pragma unroll
                for (int p = 4 * ch; p < VPL && p < 4 * ch + 4; ++p) {
                    if (live(p)) {
                        float2* dst = mb + wid * kMergeCols + 4 * lane + 128 * (p - 4 * ch);
                        dst[0] = make_float2(A - vr[2 * p].x, cS[2 * p].x);
                        dst[1] = make_float2(A - vr[2 * p].y, cS[2 * p].y);
                        dst[2] = make_float2(A - vr[2 * p + 1].x, cS[2 * p + 1].x);
                        dst[3] = make_float2(A - vr[2 * p + 1].y, cS[2 * p + 1].y);
                    }
                }
                __syncthreads();
                const int ncols = int(min(int64_t(kMergeCols), m - int64_t(kMergeCols) * ch));
                for (int cl = tid; cl < ncols; cl += kFT) {
                    float mm = kNegBig, ss = 0.0f;
#pragma unroll
                    for (int w = 0; w < kFW; ++w) {
                        const float2 pw = mb[w * kMergeCols + cl];
                        lse_merge(mm, ss, pw.x, pw.y);
                    }
                    const int64_t col = int64_t(kMergeCols) * ch + cl;
                    if (nseg == 1) finish(col, mm, ss);
                    else mypart[col] = make_float2(mm, ss);
                }
                __syncthreads();
            }
            bool merged = nseg == 1;
            if (nseg > 1 && arrive_last(c.cnt, b, nseg, &s_flag)) {
                merged = true;
                for (int64_t col = tid; col < m; col += kFT) {
                    float mm = kNegBig, ss = 0.0f;
                    for (int sg = 0; sg < nseg; ++sg) {
                        const float2 pp = __ldcg(a.part + (b * c.s.maxseg + sg) * m + col);
                        lse_merge(mm, ss, pp.x, pp.y);
                    }
                    finish(col, mm, ss);
                }
                if (tid == 0) c.cnt[b] = 0;
            }
            if (merged) {
                if (nseg == 1) __threadfence();   // this CTA's u rows are read back by exact_column
                __syncthreads();
                const int nfix = s_nfix;
                for (int k = wid; k < nfix; k += kFW) {
                    const int64_t col = s_fix[k];
                    const float lse = exact_column(c.data, a.u2, a.kinv, b, n, m, col);
                    if (lane == 0) a.v2[b * m + col] = (a.lb ? a.lb[b * m + col] : a.lb_def) - lse;
                }
                __syncthreads();
                if (tid == 0) s_nfix = 0;
            }
            fence_proxy_async_smem();   // merge-buffer writes before the stage is refilled by a bulk copy
            __syncthreads();
            if (tid == 0 && g + S < rg.g1) {
                rg.issue(g + S);
                s_issued = g + S + 1;
            }
        }
        if (++jb == c.s.nblk) {
            jb = 0;
            ++b;
        }
    }
    __syncthreads();
    if (s_abort) {   // copies still in flight after an expired wait
        if (tid == 0)
            for (int k = s_kfail; k < s_issued && k < s_kfail + S; ++k) rg.wait(k, nullptr);
        __syncthreads();
    }

    if (tolmode) {
        if (lane == 0) s_dmax[wid] = dmax;
        __syncthreads();
        if (tid == 0) {
            float mx = 0.0f;
#pragma unroll
            for (int w = 0; w < kFW; ++w) mx = fmaxf(mx, s_dmax[w]);
            atomic_max_nonneg(a.delta + a.iter, mx);
        }
    }
}

// ---------------------------------------------------------------------------
// forward iteration for mid-width rows (1024 < m <= 8192)
// ---------------------------------------------------------------------------
// A row is too wide for one warp's registers, so the whole CTA shares every
// row: thread t owns columns 4t + 1024p (p < VPL) of every row (its v and
// column partials stay in registers), a block holds R = 8 / VPL rows, and
// each row's max and sum are reduced over the CTA with one barrier each,
// for all R rows of the block at once.  The stage is free after the first
// barrier, so its refill is issued there and overlaps the rest of the block.
// The arithmetic per element and the column partials against a CTA-wide
// reference A are those of skf_fwd_iter_kernel (row values are the same in
// every thread here, so A needs no warp agreement); a thread owns its
// columns for the whole CTA, so a segment's partials are published without
// an intra-CTA merge.
constexpr int kMidFix = 1024;   // exactly recomputed columns per merge (cap)
// A block holds 8 / VPL rows (at most 8192 floats, one stage): its rows are
// held in registers at once (32 floats per thread), beside v and the
// partials.

// VS: v in shared memory (after the S stages) instead of registers, for the
// widest rows (VPL 8), where t, v and the partials would not all fit.
template <int VPL, int S, bool VS>
__global__ void __launch_bounds__(kFT, 2) skm_fwd_iter_kernel(FwdIter a) {
    constexpr int NC = 4 * VPL;
    constexpr int RMAX = 8 / VPL;   // rows per block (rows_mid): RMAX * NC = 32 floats of t per thread
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[S];
    __shared__ float s_pm[RMAX][kFW];   // per-warp row maxima
    __shared__ float s_ps[RMAX][kFW];   // per-warp row sums
    __shared__ float s_dmax;
    __shared__ int s_flag, s_nfix;
    __shared__ int s_fix[kMidFix];

    pdl_launch_dependents();
    const FusedCommon& c = a.c;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int64_t m = c.m, n = c.n;
    const int R = c.R;
    Ring<S> rg = ring_init<S>(c, bars, smem);
    const bool tolmode = a.delta != nullptr;
    if (!tolmode) ring_prime(rg);   // the matrix is read-only across launches
    pdl_wait();
    if (tolmode) {   // device-side early stop (as skf_fwd_iter_kernel)
        if (*reinterpret_cast<volatile int32_t*>(a.status + 2) != 0) return;
        if (a.iter > 0 && __ldcg(a.delta + a.iter - 1) < a.tol) {
            if (blockIdx.x == 0 && tid == 0) {
                a.status[0] = a.iter;
                a.status[1] = 1;
                a.status[2] = 1;
            }
            return;
        }
        ring_prime(rg);
    }
    if (tid == 0) {
        s_nfix = 0;
        s_dmax = 0.0f;
    }

    auto live = [&](int p) -> bool { return (4 * tid + 1024 * p) < m; };
    constexpr int NV = VS ? 1 : NC / 2;
    float2 vr[NV] = {}, cS[NC / 2];   // vr is loaded at each problem's first block, before any use
    float* s_v = reinterpret_cast<float*>(smem + size_t(S) * kTileFloats * sizeof(float));   // VS: [m]
    // v of column pair h of this thread's float4 p
    auto vpair = [&](int p, int h) -> float2 {
        if constexpr (VS) {
            return *reinterpret_cast<const float2*>(s_v + 4 * tid + 1024 * p + 2 * h);
        } else {
            return vr[2 * p + h];
        }
    };
    float A = kNegBig;   // CTA-wide column reference
    int cur = -1;

    int b = rg.g0 / c.s.nblk, jb = rg.g0 - b * c.s.nblk;
    for (int g = rg.g0; g < rg.g1; ++g) {
        if (b != cur) {   // first block of a problem in this range (the barrier below orders s_v)
            cur = b;
            if constexpr (VS) {
                for (int64_t q = tid; q < (m >> 2); q += kFT)
                    reinterpret_cast<float4*>(s_v)[q] = __ldcg(reinterpret_cast<const float4*>(a.v2 + b * m) + q);
            } else {
#pragma unroll
                for (int p = 0; p < VPL; ++p) {
                    const int64_t col = 4 * tid + 1024 * p;
                    const float4 v4 = live(p) ? __ldcg(reinterpret_cast<const float4*>(a.v2 + b * m + col))
                                              : make_float4(0, 0, 0, 0);
                    vr[2 * p] = make_float2(v4.x, v4.y);
                    vr[2 * p + 1] = make_float2(v4.z, v4.w);
                }
            }
#pragma unroll
            for (int k = 0; k < NC / 2; ++k) cS[k] = make_float2(0.0f, 0.0f);
            A = kNegBig;
        }
        const int rj = int(min(int64_t(R), n - int64_t(jb) * R));
        const int64_t grow0 = int64_t(b) * n + int64_t(jb) * R;
        const bool ok = rg.wait(g, c.err);
        if (!__syncthreads_and(ok)) {
            ring_drain(rg, g, c.err);
            return;
        }
        const float* xs = rg.buf(g);
        float2 t[RMAX][NC / 2];
        const float2 k2 = splat2(a.kinv), l2 = splat2(kLog2e);
        // t = K + v and the thread's maxima (ptxas contracts the packed
        // multiply and add into one FMA, as in skf_fwd_iter_kernel)
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
            if (r < rj) {
#pragma unroll
                for (int p = 0; p < VPL; ++p) {
                    if (live(p)) {
                        const float4 x = *reinterpret_cast<const float4*>(xs + r * int(m) + 4 * tid + 1024 * p);
                        t[r][2 * p] = add2(mul2(make_float2(x.x, x.y), k2), vpair(p, 0));
                        t[r][2 * p + 1] = add2(mul2(make_float2(x.z, x.w), k2), vpair(p, 1));
                    } else {
                        t[r][2 * p] = t[r][2 * p + 1] = make_float2(-INFINITY, -INFINITY);
                    }
                }
                const float pm = warp_max<32>(max_of(t[r]));
                if (lane == 0) s_pm[r][wid] = pm;
            }
        }
        __syncthreads();   // row maxima complete; every thread is done with the stage
        if (tid == 0 && g + S < rg.g1) rg.issue(g + S);
        float mx[RMAX], cr[RMAX];
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
            if (r < rj) {
                float mm = s_pm[r][0];
#pragma unroll
                for (int w = 1; w < kFW; ++w) mm = fmaxf(mm, s_pm[r][w]);
                mx[r] = mm;
                const float mxc = fmaxf(mm, -1.0e37f);
                const float mL = mxc * kLog2e;
                cr[r] = fmaf(mxc, kLog2e, -mL);
                const float2 nm = splat2(-mL);
#pragma unroll
                for (int k = 0; k < NC / 2; ++k) {
                    const float2 e = fma2(t[r][k], l2, nm);
                    t[r][k] = make_float2(ex2(e.x), ex2(e.y));
                }
                const float2 s2 = tree_sum2(t[r]);
                const float ps = warp_sum<32>(s2.x + s2.y);
                if (lane == 0) s_ps[r][wid] = ps;
            }
        }
        __syncthreads();   // row sums complete
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
            if (r < rj) {
                float ss = 0.0f;
#pragma unroll
                for (int w = 0; w < kFW; ++w) ss += s_ps[r][w];
                const int64_t grow = grow0 + r;
                const float la = a.la != nullptr ? __ldg(a.la + grow) : a.la_def;
                const float unew = la - (mx[r] + (fast_log(fmaxf(ss, kSumFloor)) - cr[r] * kLn2));
                if (tid == 0) {
                    if (tolmode) s_dmax = fmaxf(s_dmax, fabsf(unew - __ldcg(a.u2 + grow)));
                    a.u2[grow] = unew;
                }
                const float ai = mx[r] + unew;   // the same in every thread
                if (ai > A + kRaise) {
                    const float2 sc = splat2(exp_shift(A - ai));
#pragma unroll
                    for (int k = 0; k < NC / 2; ++k) cS[k] = mul2(cS[k], sc);
                    A = ai;
                }
                const float2 w = splat2(ex2(fmaf(ai - A, kLog2e, -cr[r])));   // exp(ai - A) / 2^cr
#pragma unroll
                for (int k = 0; k < NC / 2; ++k) cS[k] = fma2(t[r][k], w, cS[k]);
            }
        }

        if (g + 1 == rg.g1 || jb + 1 == c.s.nblk) {
            // ---- end of this CTA's part of problem b: publish its column partials ----
            const int kfirst = sched_owner(c.s, b * c.s.nblk);
            const int nseg = sched_owner(c.s, (b + 1) * c.s.nblk - 1) - kfirst + 1;
            const int seg = int(blockIdx.x) - kfirst;
            auto finish = [&](int64_t col, float mm, float ss) {
                const float l = a.lb ? a.lb[b * m + col] : a.lb_def;
                if (ss < kTinySum) {
                    const int k = atomicAdd(&s_nfix, 1);
                    if (k < kMidFix) s_fix[k] = int(col);
                    else a.v2[b * m + col] = l - lse_finish(mm, ss);
                } else {
                    a.v2[b * m + col] = l - lse_finish(mm, ss);
                }
            };
            float2* mypart = a.part + (b * c.s.maxseg + seg) * m;
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                if (live(p)) {
                    const int64_t col = 4 * tid + 1024 * p;
                    const float2 v0 = vpair(p, 0), v1 = vpair(p, 1);
                    const float2 q[4] = {make_float2(A - v0.x, cS[2 * p].x), make_float2(A - v0.y, cS[2 * p].y),
                                         make_float2(A - v1.x, cS[2 * p + 1].x),
                                         make_float2(A - v1.y, cS[2 * p + 1].y)};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        if (nseg == 1) finish(col + e, q[e].x, q[e].y);
                        else mypart[col + e] = q[e];
                    }
                }
            }
            bool merged = nseg == 1;
            if (nseg > 1 && arrive_last(c.cnt, b, nseg, &s_flag)) {
                merged = true;
                for (int64_t col = tid; col < m; col += kFT) {
                    float mm = kNegBig, ss = 0.0f;
                    for (int sg = 0; sg < nseg; ++sg) {
                        const float2 pp = __ldcg(a.part + (b * c.s.maxseg + sg) * m + col);
                        lse_merge(mm, ss, pp.x, pp.y);
                    }
                    finish(col, mm, ss);
                }
                if (tid == 0) c.cnt[b] = 0;
            }
            if (merged) {
                if (nseg == 1) __threadfence();   // this CTA's u rows are read back by exact_column
                __syncthreads();
                const int nfix = min(s_nfix, kMidFix);
                for (int k = wid; k < nfix; k += kFW) {
                    const int64_t col = s_fix[k];
                    const float lse = exact_column(c.data, a.u2, a.kinv, b, n, m, col);
                    if (lane == 0) a.v2[b * m + col] = (a.lb ? a.lb[b * m + col] : a.lb_def) - lse;
                }
                __syncthreads();
                if (tid == 0) s_nfix = 0;
            }
            __syncthreads();
        }
        if (++jb == c.s.nblk) {
            jb = 0;
            ++b;
        }
    }

    if (tolmode) {
        __syncthreads();
        if (tid == 0) atomic_max_nonneg(a.delta + a.iter, s_dmax);
    }
}

// Adjoint sweep for mid-width rows (1024 < m <= 8192), laid out as
// skm_fwd_iter_kernel: thread t owns columns 4t + 1024p, a block holds
// 8 / VPL rows, each row's dot product with mu is reduced over the CTA with
// one barrier for the block's rows together (the stage is refilled there),
// then lambda_i and the column sums sum_i P_ik lambda_i in registers; the
// arithmetic is skf_bwd_iter_kernel's.  VS: mu in shared memory.
template <int VPL, int S, bool VS>
__global__ void __launch_bounds__(kFT, 2) skm_bwd_iter_kernel(BwdIter a) {
    constexpr int NC = 4 * VPL;
    constexpr int RMAX = 8 / VPL;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[S];
    __shared__ float s_pd[RMAX][kFW];   // per-warp row dot products
    __shared__ int s_flag;

    pdl_launch_dependents();
    const FusedCommon& c = a.c;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int64_t m = c.m, n = c.n;
    Ring<S> rg = ring_init<S>(c, bars, smem);
    ring_prime(rg);   // the plan is read-only across launches
    pdl_wait();

    auto live = [&](int p) -> bool { return (4 * tid + 1024 * p) < m; };
    constexpr int NM = VS ? 1 : NC;
    float mr[NM] = {}, acc[NC];   // mr is loaded at each problem's first block, before any use
    float* s_mu = reinterpret_cast<float*>(smem + size_t(S) * kTileFloats * sizeof(float));   // VS: [m]
    auto mu4 = [&](int p) -> float4 {
        if constexpr (VS) {
            return *reinterpret_cast<const float4*>(s_mu + 4 * tid + 1024 * p);
        } else {
            return make_float4(mr[4 * p], mr[4 * p + 1], mr[4 * p + 2], mr[4 * p + 3]);
        }
    };
    int cur = -1;

    int b = rg.g0 / c.s.nblk, jb = rg.g0 - b * c.s.nblk;
    for (int g = rg.g0; g < rg.g1; ++g) {
        if (b != cur) {   // the barrier below orders the s_mu writes before their reads
            cur = b;
            if constexpr (VS) {
                for (int64_t q = tid; q < (m >> 2); q += kFT)
                    reinterpret_cast<float4*>(s_mu)[q] = __ldcg(reinterpret_cast<const float4*>(a.mu + b * m) + q);
            } else {
#pragma unroll
                for (int p = 0; p < VPL; ++p) {
                    const int64_t col = 4 * tid + 1024 * p;
                    const float4 u4 = live(p) ? __ldcg(reinterpret_cast<const float4*>(a.mu + b * m + col))
                                              : make_float4(0, 0, 0, 0);
                    mr[4 * p + 0] = u4.x;
                    mr[4 * p + 1] = u4.y;
                    mr[4 * p + 2] = u4.z;
                    mr[4 * p + 3] = u4.w;
                }
            }
#pragma unroll
            for (int e = 0; e < NC; ++e) acc[e] = 0.0f;
        }
        const int rj = int(min(int64_t(RMAX), n - int64_t(jb) * RMAX));
        const int64_t grow0 = int64_t(b) * n + int64_t(jb) * RMAX;
        float2 ri[RMAX];   // row invariants, loaded before waiting on the block
#pragma unroll
        for (int r = 0; r < RMAX; ++r) ri[r] = r < rj ? __ldg(a.rinv + grow0 + r) : make_float2(0.0f, 1.0f);
        const bool ok = rg.wait(g, c.err);
        if (!__syncthreads_and(ok)) {
            ring_drain(rg, g, c.err);
            return;
        }
        const float* ps = rg.buf(g);
        float pv[RMAX][NC];
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
            if (r < rj) {
                float sd = 0.0f;
#pragma unroll
                for (int p = 0; p < VPL; ++p) {
                    if (live(p)) {
                        const float4 x = *reinterpret_cast<const float4*>(ps + r * int(m) + 4 * tid + 1024 * p);
                        const float4 u = mu4(p);
                        pv[r][4 * p + 0] = x.x;
                        pv[r][4 * p + 1] = x.y;
                        pv[r][4 * p + 2] = x.z;
                        pv[r][4 * p + 3] = x.w;
                        sd += x.x * u.x + x.y * u.y + x.z * u.z + x.w * u.w;
                    } else {
                        pv[r][4 * p + 0] = pv[r][4 * p + 1] = pv[r][4 * p + 2] = pv[r][4 * p + 3] = 0.0f;
                    }
                }
                sd = warp_sum<32>(sd);
                if (lane == 0) s_pd[r][wid] = sd;
            }
        }
        __syncthreads();   // row dots complete; every thread is done with the stage
        if (tid == 0 && g + S < rg.g1) rg.issue(g + S);
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
            if (r < rj) {
                float sd = 0.0f;
#pragma unroll
                for (int w = 0; w < kFW; ++w) sd += s_pd[r][w];
                const float l = (ri[r].x - sd) / fmaxf(ri[r].y, kSumFloor);
                if (tid == 0) a.lam[grow0 + r] = l;
#pragma unroll
                for (int e = 0; e < NC; ++e) acc[e] += pv[r][e] * l;
            }
        }
        __syncthreads();   // s_pd is read before the next block writes it

        if (g + 1 == rg.g1 || jb + 1 == c.s.nblk) {
            const int kfirst = sched_owner(c.s, b * c.s.nblk);
            const int nseg = sched_owner(c.s, (b + 1) * c.s.nblk - 1) - kfirst + 1;
            const int seg = int(blockIdx.x) - kfirst;
            float* mypart = a.part + (b * c.s.maxseg + seg) * m;
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                if (live(p)) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int64_t col = 4 * tid + 1024 * p + e;
                        if (nseg == 1) {
                            const float2 ci = a.cinv[b * m + col];
                            a.mu[b * m + col] = (ci.x - acc[4 * p + e]) / fmaxf(ci.y, kSumFloor);
                        } else {
                            mypart[col] = acc[4 * p + e];
                        }
                    }
                }
            }
            if (nseg > 1 && arrive_last(c.cnt, b, nseg, &s_flag)) {
                for (int64_t col = tid; col < m; col += kFT) {
                    float sum = 0.0f;
                    for (int sg = 0; sg < nseg; ++sg) sum += __ldcg(a.part + (b * c.s.maxseg + sg) * m + col);
                    const float2 ci = a.cinv[b * m + col];
                    a.mu[b * m + col] = (ci.x - sum) / fmaxf(ci.y, kSumFloor);
                }
                if (tid == 0) c.cnt[b] = 0;
            }
            __syncthreads();
        }
        if (++jb == c.s.nblk) {
            jb = 0;
            ++b;
        }
    }
}

// ---------------------------------------------------------------------------
// backward (adjoint) iteration
// ---------------------------------------------------------------------------
template <int VPL, bool FULL, int S>
__global__ void __launch_bounds__(kFT, (VPL >= 8 ? 2 : (S >= 3 ? 2 : 3))) skf_bwd_iter_kernel(BwdIter a) {
    using Cfg = FCfg<VPL>;
    constexpr int R = Cfg::R, RPW = Cfg::RPW, NC = Cfg::NC;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[S];
    __shared__ int s_flag;

    pdl_launch_dependents();
    const FusedCommon& c = a.c;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int64_t m = c.m, n = c.n;
    Ring<S> rg = ring_init<S>(c, bars, smem);
    ring_prime(rg);   // the plan is read-only across launches
    pdl_wait();

    auto live = [&](int p) -> bool { return FULL || (4 * lane + 128 * p) < m; };
    float mr[NC], acc[NC];
    int cur = -1;

    int b = rg.g0 / c.s.nblk, jb = rg.g0 - b * c.s.nblk;   // advanced per block, no division
    for (int g = rg.g0; g < rg.g1; ++g) {
        if (b != cur) {
            cur = b;
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                const int64_t col = 4 * lane + 128 * p;
                const float4 u4 = live(p) ? __ldcg(reinterpret_cast<const float4*>(a.mu + b * m + col))
                                          : make_float4(0, 0, 0, 0);
                mr[4 * p + 0] = u4.x;
                mr[4 * p + 1] = u4.y;
                mr[4 * p + 2] = u4.z;
                mr[4 * p + 3] = u4.w;
            }
#pragma unroll
            for (int e = 0; e < NC; ++e) acc[e] = 0.0f;
        }
        const int rj = int(min(int64_t(R), n - int64_t(jb) * R));
        const int64_t grow0 = int64_t(b) * n + int64_t(jb) * R;
        float2 ri[RPW];   // row invariants, loaded before waiting on the block
#pragma unroll
        for (int q = 0; q < RPW; ++q) {
            const int i = wid + kFW * q;
            ri[q] = i < rj ? __ldg(a.rinv + grow0 + i) : make_float2(0.0f, 1.0f);
        }
        const bool ok = rg.wait(g, c.err);
        if (!__syncthreads_and(ok)) {
            ring_drain(rg, g, c.err);
            return;
        }
        const float* ps = rg.buf(g);
#pragma unroll
        for (int q = 0; q < RPW; ++q) {
            const int i = wid + kFW * q;
            if (i >= rj) break;
            float pv[NC];
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                if (live(p)) {
                    const float4 x = *reinterpret_cast<const float4*>(ps + i * int(m) + 4 * lane + 128 * p);
                    pv[4 * p + 0] = x.x;
                    pv[4 * p + 1] = x.y;
                    pv[4 * p + 2] = x.z;
                    pv[4 * p + 3] = x.w;
                } else {
                    pv[4 * p + 0] = pv[4 * p + 1] = pv[4 * p + 2] = pv[4 * p + 3] = 0.0f;
                }
            }
            float s = 0.0f;
#pragma unroll
            for (int e = 0; e < NC; ++e) s += pv[e] * mr[e];
            s = warp_sum<32>(s);
            const float l = (ri[q].x - s) / fmaxf(ri[q].y, kSumFloor);
            if (lane == 0) a.lam[grow0 + i] = l;
#pragma unroll
            for (int e = 0; e < NC; ++e) acc[e] += pv[e] * l;
        }
        __syncthreads();

        if (g + 1 == rg.g1 || jb + 1 == c.s.nblk) {
            const int kfirst = sched_owner(c.s, b * c.s.nblk);
            const int nseg = sched_owner(c.s, (b + 1) * c.s.nblk - 1) - kfirst + 1;
            const int seg = int(blockIdx.x) - kfirst;
            float* mb = rg.buf(g);   // [kFW][m], m <= 1024: 32 KB
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                if (live(p)) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) mb[wid * int(m) + 4 * lane + 128 * p + e] = acc[4 * p + e];
                }
            }
            __syncthreads();
            float* mypart = a.part + (b * c.s.maxseg + seg) * m;
            for (int64_t col = tid; col < m; col += kFT) {
                float sum = 0.0f;
#pragma unroll
                for (int w = 0; w < kFW; ++w) sum += mb[w * int(m) + col];
                if (nseg == 1) {
                    const float2 ci = a.cinv[b * m + col];
                    a.mu[b * m + col] = (ci.x - sum) / fmaxf(ci.y, kSumFloor);
                } else {
                    mypart[col] = sum;
                }
            }
            __syncthreads();
            if (nseg > 1 && arrive_last(c.cnt, b, nseg, &s_flag)) {
                for (int64_t col = tid; col < m; col += kFT) {
                    float sum = 0.0f;
                    for (int sg = 0; sg < nseg; ++sg) sum += __ldcg(a.part + (b * c.s.maxseg + sg) * m + col);
                    const float2 ci = a.cinv[b * m + col];
                    a.mu[b * m + col] = (ci.x - sum) / fmaxf(ci.y, kSumFloor);
                }
                if (tid == 0) c.cnt[b] = 0;
            }
            fence_proxy_async_smem();   // merge-buffer writes before the stage is refilled by a bulk copy
            __syncthreads();
        }
        if (tid == 0 && g + S < rg.g1) rg.issue(g + S);
        if (++jb == c.s.nblk) {
            jb = 0;
            ++b;
        }
    }
}

// ---------------------------------------------------------------------------
// backward set-up: the invariants of the adjoint system in one sweep
// ---------------------------------------------------------------------------
// rinv_i = (sum_k P_ik G_ik, sum_k P_ik) and cinv_k = (sum_i P_ik G_ik,
// sum_i P_ik) with G = grad_cost_b * X + grad_P (autograd's rounding), read
// from one pass over P and X on the adjoint iterations' persistent schedule:
// warp per row (row sums by warp reduction), each lane's columns accumulated
// over the CTA's rows, merged per CTA through shared memory and across CTAs
// by the one that arrives last for the problem (segment order).  The
// reference computes the same sums inside its adjoint kernels
// (src/sinkhorn/kernels.cu:965-1047).
struct BwdPrep {
    const float* P;
    const float* X;
    const float* gP;       // may be nullptr
    const float* gcost;    // may be nullptr
    int64_t n, m;
    int R;
    Sched s;
    float2* rinv;          // [B, n]
    float2* cinv;          // [B, m]
    float2* part;          // [B, maxseg, m]
    int32_t* cnt;          // [B] arrival counters, zero between launches
};

template <int VPL, bool FULL>
__global__ void __launch_bounds__(kFT, (VPL >= 8 ? 2 : 3)) skf_bwd_prep_kernel(BwdPrep a) {
    constexpr int NC = 4 * VPL, RPW = FCfg<VPL>::RPW;
    extern __shared__ __align__(128) unsigned char smem[];   // [kFW][kMergeCols] float2
    __shared__ int s_flag;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int64_t m = a.m, n = a.n;
    const int g0 = sched_q(a.s, blockIdx.x), g1 = sched_q(a.s, int(blockIdx.x) + 1);
    auto live = [&](int p) -> bool { return FULL || (4 * lane + 128 * p) < m; };
    float cpg[NC], cp[NC];
    float gc = 0.0f;
    int cur = -1;
    int b = g0 / a.s.nblk, jb = g0 - b * a.s.nblk;
    for (int g = g0; g < g1; ++g) {
        if (b != cur) {
            cur = b;
            gc = a.gcost ? __ldg(a.gcost + b) : 0.0f;
#pragma unroll
            for (int e = 0; e < NC; ++e) cpg[e] = cp[e] = 0.0f;
        }
        const int rj = int(min(int64_t(a.R), n - int64_t(jb) * a.R));
        const int64_t grow0 = int64_t(b) * n + int64_t(jb) * a.R;
#pragma unroll 1
        for (int q = 0; q < RPW; ++q) {   // one row in flight per warp: the accumulators fill the registers
            const int i = wid + kFW * q;
            if (i >= rj) break;   // warp-uniform
            const int64_t rbase = (grow0 + i) * m;
            float spg = 0.0f, sp = 0.0f;
#pragma unroll
            for (int c0 = 0; c0 < VPL; c0 += 4) {   // at most four float4 of each input live at a time
                constexpr int CH = VPL < 4 ? VPL : 4;
                float4 p4[CH], x4[CH];
#pragma unroll
                for (int k = 0; k < CH; ++k) {   // the chunk's loads first: bytes in flight
                    const int p = c0 + k;
                    const int64_t col = 4 * lane + 128 * p;
                    p4[k] = live(p) ? __ldg(reinterpret_cast<const float4*>(a.P + rbase + col)) : make_float4(0, 0, 0, 0);
                    x4[k] = live(p) ? __ldg(reinterpret_cast<const float4*>(a.X + rbase + col)) : make_float4(0, 0, 0, 0);
                }
#pragma unroll
                for (int k = 0; k < CH; ++k) {
                    const int p = c0 + k;
                    const float pv[4] = {p4[k].x, p4[k].y, p4[k].z, p4[k].w};
                    const float xv[4] = {x4[k].x, x4[k].y, x4[k].z, x4[k].w};
                    float gpv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    if (a.gP != nullptr && live(p)) {
                        const float4 g4 = __ldg(reinterpret_cast<const float4*>(a.gP + rbase + 4 * lane + 128 * p));
                        gpv[0] = g4.x;
                        gpv[1] = g4.y;
                        gpv[2] = g4.z;
                        gpv[3] = g4.w;
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        float gv = __fmul_rn(gc, xv[e]);
                        if (a.gP != nullptr) gv = __fadd_rn(gv, gpv[e]);
                        const float pg = pv[e] * gv;
                        spg += pg;
                        sp += pv[e];
                        cpg[4 * p + e] += pg;
                        cp[4 * p + e] += pv[e];
                    }
                }
            }
            spg = warp_sum<32>(spg);
            sp = warp_sum<32>(sp);
            if (lane == 0) a.rinv[grow0 + i] = make_float2(spg, sp);
        }
        if (g + 1 == g1 || jb + 1 == a.s.nblk) {
            // ---- end of this CTA's part of problem b: merge the warps, publish ----
            const int kfirst = sched_owner(a.s, b * a.s.nblk);
            const int nseg = sched_owner(a.s, (b + 1) * a.s.nblk - 1) - kfirst + 1;
            const int seg = int(blockIdx.x) - kfirst;
            float2* mb = reinterpret_cast<float2*>(smem);
            float2* dst = nseg == 1 ? a.cinv + int64_t(b) * m : a.part + (int64_t(b) * a.s.maxseg + seg) * m;
#pragma unroll
            for (int ch = 0; ch < (VPL + 3) / 4; ++ch) {
                __syncthreads();   // the merge buffer is free
#pragma unroll
                for (int p = 4 * ch; p < VPL && p < 4 * ch + 4; ++p) {
                    if (live(p)) {
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            mb[wid * kMergeCols + 4 * lane + 128 * (p - 4 * ch) + e] =
                                make_float2(cpg[4 * p + e], cp[4 * p + e]);
                    }
                }
                __syncthreads();
                const int ncols = int(min(int64_t(kMergeCols), m - int64_t(kMergeCols) * ch));
                for (int cl = tid; cl < ncols; cl += kFT) {
                    float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
                    for (int w = 0; w < kFW; ++w) {
                        const float2 v = mb[w * kMergeCols + cl];
                        acc.x += v.x;
                        acc.y += v.y;
                    }
                    dst[int64_t(kMergeCols) * ch + cl] = acc;
                }
            }
            if (nseg > 1 && arrive_last(a.cnt, b, nseg, &s_flag)) {
                const float2* pb = a.part + int64_t(b) * a.s.maxseg * m;
                for (int64_t col = tid; col < m; col += kFT) {
                    float2 acc = make_float2(0.0f, 0.0f);
                    for (int sg = 0; sg < nseg; ++sg) {
                        const float2 v = __ldcg(pb + int64_t(sg) * m + col);
                        acc.x += v.x;
                        acc.y += v.y;
                    }
                    a.cinv[int64_t(b) * m + col] = acc;
                }
                if (tid == 0) a.cnt[b] = 0;
            }
        }
        if (++jb == a.s.nblk) {
            jb = 0;
            ++b;
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
int vpl_for(int64_t m) { return m <= 128 ? 1 : m <= 256 ? 2 : m <= 512 ? 4 : 8; }
int rows_per_block(int64_t m) { return 64 / vpl_for(m); }

int sm_count() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

// Pipeline depth: 2 stages (3 CTAs per SM); 3 stages (2 CTAs per SM)
// measured 64 vs 60 us per cfg2 forward iteration.
constexpr int kStages = 2;
// The forward's full-width kernel runs 2 CTAs per SM (registers), which
// leaves room for a third stage of the ring.
constexpr int kStagesFullFwd = 3;

template <int VPL, bool FULL, int S>
void set_attr_one() {
    const int sm = S * kTileFloats * int(sizeof(float));
    cudaFuncSetAttribute(skf_fwd_iter_kernel<VPL, FULL, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
    cudaFuncSetAttribute(skf_bwd_iter_kernel<VPL, FULL, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
}

template <int S>
void set_attrs_s() {
    set_attr_one<1, false, S>();
    set_attr_one<1, true, S>();
    set_attr_one<2, false, S>();
    set_attr_one<2, true, S>();
    set_attr_one<4, false, S>();
    set_attr_one<4, true, S>();
    set_attr_one<8, false, S>();
    set_attr_one<8, true, S>();
}

// Mid-width rows, 2 CTAs per SM (registers: all of a block's rows are held
// at once): 3 stages, or 2 stages and v in shared memory for VPL 8.
int vpl_mid(int64_t m) { return m <= 2048 ? 2 : m <= 4096 ? 4 : 8; }
int rows_mid(int64_t m) { return 8 / vpl_mid(m); }
constexpr size_t kMidSmem3 = size_t(3) * kTileFloats * sizeof(float);
constexpr size_t kMidSmem8 = size_t(2) * kTileFloats * sizeof(float) + 8192 * sizeof(float);
#define SKM2 skm_fwd_iter_kernel<2, 3, false>
#define SKM4 skm_fwd_iter_kernel<4, 3, false>
#define SKM8 skm_fwd_iter_kernel<8, 2, true>
#define SKMB2 skm_bwd_iter_kernel<2, 3, false>
#define SKMB4 skm_bwd_iter_kernel<4, 3, false>
#define SKMB8 skm_bwd_iter_kernel<8, 2, true>

void set_attrs_mid() {
    cudaFuncSetAttribute(SKM2, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMidSmem3));
    cudaFuncSetAttribute(SKM4, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMidSmem3));
    cudaFuncSetAttribute(SKM8, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMidSmem8));
    cudaFuncSetAttribute(SKMB2, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMidSmem3));
    cudaFuncSetAttribute(SKMB4, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMidSmem3));
    cudaFuncSetAttribute(SKMB8, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMidSmem8));
}

void ensure_attrs() {
    constexpr int kMaxDev = 64;
    static bool done[kMaxDev] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < kMaxDev && done[dev]) return;
    set_attrs_s<2>();
    set_attrs_s<3>();
    set_attrs_mid();
    if (dev >= 0 && dev < kMaxDev) done[dev] = true;
}

template <int S, bool FULL>
int per_sm_for(int vpl) {
    const int sm = S * kTileFloats * int(sizeof(float));
    int nb = 0;
    switch (vpl) {
        case 1: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, skf_fwd_iter_kernel<1, FULL, S>, kFT, sm); break;
        case 2: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, skf_fwd_iter_kernel<2, FULL, S>, kFT, sm); break;
        case 4: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, skf_fwd_iter_kernel<4, FULL, S>, kFT, sm); break;
        default: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, skf_fwd_iter_kernel<8, FULL, S>, kFT, sm); break;
    }
    return nb > 0 ? nb : 1;
}

template <typename Args, typename K>
void launch(K kernel, const Args& a, int G, int S, bool pdl, cudaStream_t st, size_t smem_bytes = 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(G));
    cfg.blockDim = dim3(kFT);
    cfg.dynamicSmemBytes = smem_bytes ? smem_bytes : size_t(S) * kTileFloats * sizeof(float);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kernel, a);
}

template <int VPL, int S>
void launch_fwd_v(const FwdIter& a, int G, bool pdl, cudaStream_t st) {
    if (a.c.m == 128 * VPL) launch(skf_fwd_iter_kernel<VPL, true, S>, a, G, S, pdl, st);
    else launch(skf_fwd_iter_kernel<VPL, false, S>, a, G, S, pdl, st);
}
template <int VPL, int S>
void launch_bwd_v(const BwdIter& a, int G, bool pdl, cudaStream_t st) {
    if (a.c.m == 128 * VPL) launch(skf_bwd_iter_kernel<VPL, true, S>, a, G, S, pdl, st);
    else launch(skf_bwd_iter_kernel<VPL, false, S>, a, G, S, pdl, st);
}

template <int S>
void launch_fwd_s(const FwdIter& a, int G, bool pdl, cudaStream_t st) {
    switch (vpl_for(a.c.m)) {
        case 1: launch_fwd_v<1, S>(a, G, pdl, st); break;
        case 2: launch_fwd_v<2, S>(a, G, pdl, st); break;
        case 4: launch_fwd_v<4, S>(a, G, pdl, st); break;
        default: launch_fwd_v<8, S>(a, G, pdl, st); break;
    }
}
template <int S>
void launch_bwd_s(const BwdIter& a, int G, bool pdl, cudaStream_t st) {
    switch (vpl_for(a.c.m)) {
        case 1: launch_bwd_v<1, S>(a, G, pdl, st); break;
        case 2: launch_bwd_v<2, S>(a, G, pdl, st); break;
        case 4: launch_bwd_v<4, S>(a, G, pdl, st); break;
        default: launch_bwd_v<8, S>(a, G, pdl, st); break;
    }
}

Sched sched_of(const FusedPlan& p) {
    Sched s;
    s.T = int(p.total_blocks);
    s.nblk = int(p.nblk);
    s.G = p.G;
    s.maxseg = p.maxseg;
    s.hint = 1;
    return s;
}

}  // namespace

bool sk_fused_shape_ok(int64_t B, int64_t n, int64_t m) {
    if (B < 1 || n < 1 || m < 4 || m > 1024 || (m % 4) != 0) return false;
    const int64_t R = rows_per_block(m);
    return B * ((n + R - 1) / R) < (int64_t(1) << 31);   // block indices are 32-bit
}

bool sk_fused_supported(int64_t B, int64_t n, int64_t m, const void* data) {
    return sk_fused_shape_ok(B, n, m) && (reinterpret_cast<uintptr_t>(data) & 15u) == 0;
}

FusedPlan sk_fused_plan(int64_t B, int64_t n, int64_t m, bool fwd) {
    FusedPlan p;
    ensure_attrs();
    const int R = rows_per_block(m);
    const bool full = fwd && m == 128 * vpl_for(m);   // the forward's full-width kernel holds fewer CTAs
    p.stages = full ? kStagesFullFwd : kStages;
    const int per_sm = full ? (p.stages == 3 ? per_sm_for<3, true>(vpl_for(m)) : per_sm_for<2, true>(vpl_for(m)))
                            : (p.stages == 3 ? per_sm_for<3, false>(vpl_for(m)) : per_sm_for<2, false>(vpl_for(m)));
    p.nblk = (n + R - 1) / R;
    p.total_blocks = B * p.nblk;
    const int64_t slots = int64_t(sm_count()) * per_sm;
    p.G = int(std::min<int64_t>(p.total_blocks, slots));
    Sched s = sched_of(p);
    int maxseg = 1;
    for (int b = 0; b < int(B); ++b) {
        const int k0 = sched_owner(s, b * s.nblk), k1 = sched_owner(s, (b + 1) * s.nblk - 1);
        maxseg = std::max(maxseg, k1 - k0 + 1);
    }
    p.maxseg = maxseg;
    p.nseg = maxseg;
    return p;
}

bool sk_mid_shape_ok(int64_t B, int64_t n, int64_t m) {
    if (B < 1 || n < 1 || m <= 1024 || m > 8192 || (m % 4) != 0) return false;
    const int64_t R = rows_mid(m);
    return B * ((n + R - 1) / R) < (int64_t(1) << 31);   // block indices are 32-bit
}

bool sk_mid_supported(int64_t B, int64_t n, int64_t m, const void* data) {
    return sk_mid_shape_ok(B, n, m) && (reinterpret_cast<uintptr_t>(data) & 15u) == 0;
}

FusedPlan sk_mid_plan(int64_t B, int64_t n, int64_t m, bool fwd) {
    FusedPlan p;
    ensure_attrs();
    const int R = rows_mid(m);
    p.stages = vpl_mid(m) == 8 ? 2 : 3;
    int nb = 0;
    const int v = vpl_mid(m);
    const size_t sm = v == 8 ? kMidSmem8 : kMidSmem3;
    cudaError_t e;
    if (fwd) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, v == 2 ? SKM2 : v == 4 ? SKM4 : SKM8, kFT, sm);
    else e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, v == 2 ? SKMB2 : v == 4 ? SKMB4 : SKMB8, kFT, sm);
    if (e != cudaSuccess) nb = 0;
    if (nb < 1) {
        cudaGetLastError();
        nb = 1;
    }
    p.nblk = (n + R - 1) / R;
    p.total_blocks = B * p.nblk;
    p.G = int(std::min<int64_t>(p.total_blocks, int64_t(sm_count()) * nb));
    Sched s = sched_of(p);
    int maxseg = 1;
    for (int b = 0; b < int(B); ++b) {
        const int k0 = sched_owner(s, b * s.nblk), k1 = sched_owner(s, (b + 1) * s.nblk - 1);
        maxseg = std::max(maxseg, k1 - k0 + 1);
    }
    p.maxseg = maxseg;
    p.nseg = maxseg;
    return p;
}

int sk_mid_fwd_iter(const SkFwdArgs& a, const FusedPlan& p, float2* part, int32_t* cnt, float* delta, int iter,
                    bool first, bool last, cudaStream_t st) {
    FwdIter f{};
    f.c.data = a.X;
    f.c.n = a.n;
    f.c.m = a.m;
    f.c.R = rows_mid(a.m);
    f.c.s = sched_of(p);
    f.c.s.hint = last ? 0 : 1;
    f.c.cnt = cnt;
    f.c.err = a.status + 3;
    f.kinv = a.kinv;
    f.la = a.la;
    f.la_def = a.la_def;
    f.lb = a.lb;
    f.lb_def = a.lb_def;
    f.u2 = a.u2;
    f.v2 = a.v2;
    f.part = part;
    f.delta = delta;
    f.status = a.status;
    f.tol = a.tol;
    f.iter = iter;
    switch (vpl_mid(a.m)) {
        case 2: launch(SKM2, f, p.G, 3, !first, st); break;
        case 4: launch(SKM4, f, p.G, 3, !first, st); break;
        default: launch(SKM8, f, p.G, 2, !first, st, kMidSmem8); break;
    }
    return DOT_OK;
}

int sk_mid_bwd_iter(const SkBwdArgs& a, const FusedPlan& p, const float2* rinv, const float2* cinv, float* lam,
                    float* mu, float* part, int32_t* cnt, int32_t* err, bool first, bool last, cudaStream_t st) {
    BwdIter f{};
    f.c.data = a.P;
    f.c.n = a.n;
    f.c.m = a.m;
    f.c.R = rows_mid(a.m);
    f.c.s = sched_of(p);
    f.c.s.hint = last ? 0 : 1;
    f.c.cnt = cnt;
    f.c.err = err;
    f.rinv = rinv;
    f.cinv = cinv;
    f.lam = lam;
    f.mu = mu;
    f.part = part;
    switch (vpl_mid(a.m)) {
        case 2: launch(SKMB2, f, p.G, 3, !first, st); break;
        case 4: launch(SKMB4, f, p.G, 3, !first, st); break;
        default: launch(SKMB8, f, p.G, 2, !first, st, kMidSmem8); break;
    }
    return DOT_OK;
}

int sk_fused_fwd_iter(const SkFwdArgs& a, const FusedPlan& p, float2* part, int32_t* cnt, float* delta,
                      int iter, bool first, bool last, cudaStream_t st) {
    FwdIter f{};
    f.c.data = a.X;
    f.c.n = a.n;
    f.c.m = a.m;
    f.c.R = rows_per_block(a.m);
    f.c.s = sched_of(p);
    f.c.s.hint = last ? 0 : 1;
    f.c.cnt = cnt;
    f.c.err = a.status + 3;
    f.kinv = a.kinv;
    f.la = a.la;
    f.la_def = a.la_def;
    f.lb = a.lb;
    f.lb_def = a.lb_def;
    f.u2 = a.u2;
    f.v2 = a.v2;
    f.part = part;
    f.delta = delta;
    f.status = a.status;
    f.tol = a.tol;
    f.iter = iter;
    if (p.stages == 3) launch_fwd_s<3>(f, p.G, !first, st);
    else launch_fwd_s<2>(f, p.G, !first, st);
    return DOT_OK;
}

int sk_fused_bwd_prep(const SkBwdArgs& a, const FusedPlan& p, float2* rinv, float2* cinv, float2* part,
                      int32_t* cnt, cudaStream_t st) {
    BwdPrep f{};
    f.P = a.P;
    f.X = a.X;
    f.gP = a.gP;
    f.gcost = a.gcost;
    f.n = a.n;
    f.m = a.m;
    f.R = rows_per_block(a.m);
    f.s = sched_of(p);
    f.rinv = rinv;
    f.cinv = cinv;
    f.part = part;
    f.cnt = cnt;
    const size_t sm = size_t(kFW) * kMergeCols * sizeof(float2);
    const bool full = a.m == 128 * vpl_for(a.m);
    switch (vpl_for(a.m)) {
        case 1: full ? skf_bwd_prep_kernel<1, true><<<p.G, kFT, sm, st>>>(f) : skf_bwd_prep_kernel<1, false><<<p.G, kFT, sm, st>>>(f); break;
        case 2: full ? skf_bwd_prep_kernel<2, true><<<p.G, kFT, sm, st>>>(f) : skf_bwd_prep_kernel<2, false><<<p.G, kFT, sm, st>>>(f); break;
        case 4: full ? skf_bwd_prep_kernel<4, true><<<p.G, kFT, sm, st>>>(f) : skf_bwd_prep_kernel<4, false><<<p.G, kFT, sm, st>>>(f); break;
        default: full ? skf_bwd_prep_kernel<8, true><<<p.G, kFT, sm, st>>>(f) : skf_bwd_prep_kernel<8, false><<<p.G, kFT, sm, st>>>(f); break;
    }
    return DOT_OK;
}

int sk_fused_bwd_iter(const SkBwdArgs& a, const FusedPlan& p, const float2* rinv, const float2* cinv,
                      float* lam, float* mu, float* part, int32_t* cnt, int32_t* err, bool first, bool last,
                      cudaStream_t st) {
    BwdIter f{};
    f.c.data = a.P;
    f.c.n = a.n;
    f.c.m = a.m;
    f.c.R = rows_per_block(a.m);
    f.c.s = sched_of(p);
    f.c.s.hint = last ? 0 : 1;
    f.c.cnt = cnt;
    f.c.err = err;
    f.rinv = rinv;
    f.cinv = cinv;
    f.lam = lam;
    f.mu = mu;
    f.part = part;
    if (p.stages == 3) launch_bwd_s<3>(f, p.G, !first, st);
    else launch_bwd_s<2>(f, p.G, !first, st);
    return DOT_OK;
}

}  // namespace dotb

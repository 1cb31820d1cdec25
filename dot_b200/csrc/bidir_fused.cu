// Bidirectional softmax for rows that fit a warp's registers (L2 <= 1024;
// fp32 input with L2 % 4 == 0 or bf16 input with L2 % 8 == 0; 16-byte
// aligned tensors): one persistent launch per direction, one thread-block
// cluster per problem at a time.
//
//   out_ij  = sqrt(1e-9 + row_ij * col_ij),  row = softmax_j(sim/T),
//             col = softmax_i(sim/T), 0 outside the length window
//   grad_ij = (d_row - rdot_i)*row/T + (d_col - cdot_j)*col/T
//           = (2 q_ij - rdot_i*row_ij - cdot_j*col_ij) / T,
//             q = dp*row*col, dp = g * 0.5 / out, rdot_i = sum_j q_ij,
//             cdot_j = sum_i q_ij
// (reference: src/bidirectional_softmax/kernels_cpu.cpp:41-232).
//
// Layout of the work.  A cluster of kC CTAs takes one problem at a time
// (problems cid, cid + nclusters, ...); CTA r of the cluster owns rows
// [r*rows_per, (r+1)*rows_per) of the problem and columns
// [r*cols_per, (r+1)*cols_per) for the column reduction.  Per problem:
//   pass 1   stream the CTA's rows through shared memory (1-D bulk copies on
//            an S-stage mbarrier ring, L2 evict_last): forward -- row
//            (max, 1/sum) exactly (max then sum over the row in registers)
//            and column partial sums reusing the row exponentials,
//            exp(v_ij - A) = E_ij * exp(max_i - A) for a warp-wide reference
//            A >= every row max; backward -- rdot_i and column partial sums
//            of q.  The CTA's warps are merged into one partial per column.
//   reduce   cluster barrier; each CTA merges its column slice over the kC
//            partials read through distributed shared memory (in rank
//            order: deterministic), then after a second barrier gathers
//            every column's result from its owner.  A forward column whose
//            merged sum is too small to trust is recomputed exactly from sim.
//   pass 2   stream the same rows again (served from L2, evict_first) and
//            write out (forward) or grad_sim (backward) with evict_first stores.
// Pass 2 of one problem and pass 1 of the next run on the same ring, so the
// copies of the next rows are in flight across the barriers.  No CTA waits
// on anything but its own copies and the cluster's hardware barriers.
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "common.cuh"
#include "internal.h"
#include "tma.cuh"

namespace dotb {

namespace {

constexpr int kC = 8;               // CTAs per cluster
constexpr int kStage = 32768;       // bytes per ring stage
constexpr int kMaxL2 = 1024;
constexpr int kFwdWarps = 8;
constexpr int kBwdWarps = 8;
constexpr int kFwdStages = 2;
constexpr int kBwdStages = 3;
constexpr float kRaiseB = 60.0f;
constexpr float kTinyB = 8.077935669463161e-28f;   // 2^-90

// ---------------------------------------------------------------------------
// cluster primitives (sm_90+)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// Every thread of every CTA of the cluster; release/acquire orders the
// shared-memory writes before it with the remote reads after it.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// `p` (in this CTA's shared memory) as seen in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t dsmem(const void* p, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
    return a;
}
__device__ __forceinline__ float2 ld_dsmem2(uint32_t a) {
    float2 v;
    asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ float ld_dsmem(uint32_t a) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
    return v;
}

// ---------------------------------------------------------------------------
// element access
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ld4s(const float* p, float (&v)[4]) {   // shared memory
    const float4 x = *reinterpret_cast<const float4*>(p);
    v[0] = x.x;
    v[1] = x.y;
    v[2] = x.z;
    v[3] = x.w;
}
__device__ __forceinline__ void ld4s(const __nv_bfloat16* p, float (&v)[4]) {
    const uint2 x = *reinterpret_cast<const uint2*>(p);
    v[0] = __uint_as_float(x.x << 16);
    v[1] = __uint_as_float(x.x & 0xffff0000u);
    v[2] = __uint_as_float(x.y << 16);
    v[3] = __uint_as_float(x.y & 0xffff0000u);
}
__device__ __forceinline__ void st4g(float* p, const float (&v)[4], uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "f"(v[0]), "f"(v[1]),
                 "f"(v[2]), "f"(v[3]), "l"(pol)
                 : "memory");
}
__device__ __forceinline__ void st4g(__nv_bfloat16* p, const float (&v)[4], uint64_t pol) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
    const __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
    const uint32_t x = *reinterpret_cast<const uint32_t*>(&a);
    const uint32_t y = *reinterpret_cast<const uint32_t*>(&b);
    asm volatile("st.global.L2::cache_hint.v2.u32 [%0], {%1, %2}, %3;" ::"l"(p), "r"(x), "r"(y), "l"(pol)
                 : "memory");
}

__device__ __forceinline__ float rsqrt_approx(float x) {
    float y;
    asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void window(const int32_t* lengths, int64_t b, int64_t L1, int64_t L2, int64_t& l1,
                                       int64_t& l2) {
    l1 = min(max(int64_t(__ldg(lengths + 2 * b)), int64_t(0)), L1);
    l2 = min(max(int64_t(__ldg(lengths + 2 * b + 1)), int64_t(0)), L2);
}

// Per-element values from the statistics, the same expressions in every pass
// (so the backward sees the forward's values bit for bit):
//   row = exp(v - rmax) * rinv, col = exp(v - cmax) * cinv, rc = row * col,
//   out = min(sqrt(1e-9 + rc), 1), iout = 1 / out.
// sqrt and 1/sqrt come from one rsqrt (SFU, ~2^-22 relative).  The column
// value's numerator exp(v - A) and its share of the column sum (accumulated
// as E*w) can differ by an ulp, so rc may exceed 1 by rounding where one
// element dominates its row and column; out is capped at 1, its
// exact-arithmetic bound.  out >= sqrt(1e-9) > 1e-9, so the reference's guard
// dp = 0 for out <= 1e-9 never applies.
struct BsVals {
    float row, col, rc, out, iout;
};
__device__ __forceinline__ BsVals bs_vals(float v, float2 rs, float2 cs) {
    BsVals q;
    q.row = exp_shift(v - rs.x) * rs.y;
    q.col = exp_shift(v - cs.x) * cs.y;
    q.rc = q.row * q.col;
    const float x = 1e-9f + q.rc;
    const float r = rsqrt_approx(x);
    q.out = fminf(x * r, 1.0f);
    q.iout = fmaxf(r, 1.0f);
    return q;
}

// Exact column softmax statistics (max, 1/sum) over rows [0, l1) -- one warp.
template <typename T>
__device__ float2 exact_col_stats(const T* sb, int64_t L2, int64_t l1, int64_t col, float invT) {
    const int lane = threadIdx.x & 31;
    float mx = kNegBig;
    for (int64_t i = lane; i < l1; i += 32) mx = fmaxf(mx, __fmul_rn(float(sb[i * L2 + col]), invT));
    mx = warp_max<32>(mx);
    float s = 0.0f;
    for (int64_t i = lane; i < l1; i += 32) s += exp_shift(__fmul_rn(float(sb[i * L2 + col]), invT) - mx);
    s = warp_sum<32>(s);
    return make_float2(mx, s > 0.0f ? 1.0f / s : 0.0f);
}

// ---------------------------------------------------------------------------
// the CTA's block sequence: for each of its cluster's problems, the nb blocks
// of its row slice for pass 1, then the same nb blocks for pass 2
// ---------------------------------------------------------------------------
struct ClArgs {
    const unsigned char* src[2];   // sim, grad_out (backward)
    uint32_t row_bytes[2];
    uint32_t tile_off1;            // byte offset of grad_out's tile in a stage
    int nsrc;
    const int32_t* lengths;
    int64_t B, L1, L2;
    int64_t rows_per, cols_per;    // per CTA of a cluster
    int R;                         // rows per block
    float invT;
    float2* rstat;                 // [B, L1] forward output / backward input
    float2* cstat;                 // [B, L2]
    float* out;                    // forward: [B, L1, L2]
    void* gsim;                    // backward: [B, L1, L2], float or bf16
    float* rdot;                   // backward scratch [B, L1]
    float* tau_row;                // backward: [B, L1] or nullptr
    int32_t* err;                  // bounded-wait expiry word
};

template <int S>
struct ClRing {
    const ClArgs* a;
    unsigned char* smem;
    uint64_t* bar;
    int64_t r0, r1;   // row slice
    int nb;           // blocks per pass
    int K;            // blocks in the whole sequence
    uint32_t cid, ncl;

    __device__ unsigned char* stage(int k) const { return smem + size_t(k % S) * kStage; }
    __device__ int rows_in(int j) const { return int(min(int64_t(a->R), r1 - (r0 + int64_t(j) * a->R))); }
    __device__ void issue(int k) const {   // one thread
        const int per = 2 * nb;
        const int64_t b = cid + int64_t(k / per) * ncl;
        const int pass = (k % per) / nb, j = k % nb;
        const int rows = rows_in(j);
        const int64_t row = b * a->L1 + r0 + int64_t(j) * a->R;
        uint64_t* bb = bar + k % S;
        uint32_t total = 0;
        for (int s = 0; s < a->nsrc; ++s) total += uint32_t(rows) * a->row_bytes[s];
        mbar_arrive_expect_tx(bb, total);
        const uint64_t pol = pass == 0 ? l2_policy_evict_last() : l2_policy_evict_first();
        for (int s = 0; s < a->nsrc; ++s)
            bulk_g2s_hint(stage(k) + (s == 0 ? 0u : a->tile_off1), a->src[s] + row * a->row_bytes[s],
                          uint32_t(rows) * a->row_bytes[s], bb, pol);
    }
    __device__ bool wait(int k, int32_t* err) const {
        return mbar_wait_sleep(bar + k % S, uint32_t((k / S) & 1), err);
    }
};

template <int S>
__device__ __forceinline__ ClRing<S> cl_ring_init(const ClArgs& a, uint64_t* bars, unsigned char* smem) {
    ClRing<S> r;
    r.a = &a;
    r.smem = smem;
    r.bar = bars;
    r.cid = cluster_id();
    r.ncl = cluster_count();
    const int64_t rank = cluster_rank();
    r.r0 = min(a.L1, rank * a.rows_per);
    r.r1 = min(a.L1, r.r0 + a.rows_per);
    r.nb = int((r.r1 - r.r0 + a.R - 1) / a.R);
    const int64_t nprob = int64_t(r.cid) < a.B ? (a.B - 1 - r.cid) / r.ncl + 1 : 0;
    r.K = int(nprob * 2 * r.nb);
    if (threadIdx.x == 0) {
#pragma unroll
        for (int k = 0; k < S; ++k) mbar_init(&bars[k], 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x == 0)
        for (int k = 0; k < r.K && k < S; ++k) r.issue(k);
    return r;
}

// Wait for block k of the sequence; after a failed wait the CTA stops waiting
// and issuing (results are invalid, *err is set) but keeps taking part in the
// cluster barriers.  Returns whether the block may be used.
template <int S>
__device__ __forceinline__ bool cl_wait(const ClRing<S>& r, int k, int& kfail) {
    if (kfail >= 0) return false;
    const bool ok = __syncthreads_and(r.wait(k, r.a->err));
    if (!ok) kfail = k;
    return ok;
}

// Issue block k + S once block k's stage is free.
template <int S>
__device__ __forceinline__ void cl_next(const ClRing<S>& r, int k, int kfail) {
    if (threadIdx.x == 0 && kfail < 0 && k + S < r.K) r.issue(k + S);
}

// Before exit after a failed wait: wait (bounded) for copies still in flight.
template <int S>
__device__ __forceinline__ void cl_drain(const ClRing<S>& r, int kfail) {
    if (kfail >= 0 && threadIdx.x == 0)
        for (int k = kfail; k < r.K && k < kfail + S; ++k) r.wait(k, nullptr);
    __syncthreads();
}

// Warp layout.  The NW warps of a CTA form NW/WPR row slots of WPR warps;
// slot q takes rows q, q + NW/WPR, ... of each block, and warp c of a slot
// takes columns c*128*VPLW + 4*lane + 128*p (p < VPLW) of its rows, so a lane
// keeps NC = 4*VPLW columns in registers.  Rows of 1024 columns are split
// over WPR = 2 warps (16 columns per lane); the per-row reductions of the WPR
// warps meet in shared memory after the block's barrier.
template <int VPL>
struct WL {
    static constexpr int WPR = VPL >= 8 ? 2 : 1;   // warps per row
    static constexpr int VPLW = VPL / WPR;          // float4 groups per lane
    static constexpr int NC = 4 * VPLW;             // columns per lane
};

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
template <typename T, int VPL>
__global__ void __launch_bounds__(kFwdWarps * 32, 3) bs_fwd_cluster_kernel(ClArgs a) {
    constexpr int NW = kFwdWarps, S = kFwdStages, NT = NW * 32;
    constexpr int WPR = WL<VPL>::WPR, VPLW = WL<VPL>::VPLW, NC = WL<VPL>::NC, SLOTS = NW / WPR;
    extern __shared__ __align__(128) unsigned char smem[];
    float2* cs = reinterpret_cast<float2*>(smem + size_t(S) * kStage);   // [kMaxL2] column statistics
    __shared__ __align__(8) uint64_t bars[S];
    __shared__ float2 s_rp[64][WPR];   // per-row (max, sum) of each warp of the row
    __shared__ int s_nfix;
    __shared__ int s_fix[kMaxL2 / kC];

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int slot = wid / WPR, cpart = wid % WPR;
    const int64_t cbase = int64_t(cpart) * 128 * VPLW;
    const int64_t L1 = a.L1, L2 = a.L2;
    const uint32_t rank = cluster_rank();
    ClRing<S> rg = cl_ring_init<S>(a, bars, smem);
    const int64_t c0 = min(L2, int64_t(rank) * a.cols_per), c1 = min(L2, c0 + a.cols_per);
    const uint64_t pol_out = l2_policy_evict_first();
    int kfail = -1;
    int k = 0;
    for (int64_t b = rg.cid; b < a.B; b += rg.ncl) {
        int64_t l1, l2;
        window(a.lengths, b, L1, L2, l1, l2);
        const T* sb = reinterpret_cast<const T*>(a.src[0]) + b * L1 * L2;
        const bool full = l2 == L2;

        // ---- pass 1: row statistics, column partials ----
        float Sc[NC];
#pragma unroll
        for (int e = 0; e < NC; ++e) Sc[e] = 0.0f;
        float A = kNegBig;
        float2* cp = nullptr;   // merged column partials, in the last pass-1 stage
        int kcp = -1;
        for (int j = 0; j < rg.nb; ++j, ++k) {
            const bool ok = cl_wait(rg, k, kfail);
            const T* xs = reinterpret_cast<const T*>(rg.stage(k));
            const int rows = rg.rows_in(j);
            for (int il = slot; ok && il < rows; il += SLOTS) {
                const int64_t i = rg.r0 + int64_t(j) * a.R + il;
                if (i >= l1 || l2 == 0) {
                    if (lane == 0) s_rp[il][cpart] = make_float2(kNegBig, 0.0f);
                    continue;
                }
                float t[NC];
#pragma unroll
                for (int p = 0; p < VPLW; ++p) {
                    const int64_t col = cbase + 4 * lane + 128 * p;
                    float v[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                    if (col < L2) {
                        ld4s(xs + il * L2 + col, v);
                        if (full) {
#pragma unroll
                            for (int e = 0; e < 4; ++e) v[e] = __fmul_rn(v[e], a.invT);
                        } else {
#pragma unroll
                            for (int e = 0; e < 4; ++e) v[e] = (col + e < l2) ? __fmul_rn(v[e], a.invT) : -INFINITY;
                        }
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) t[4 * p + e] = v[e];
                }
                float mx = t[0];
#pragma unroll
                for (int e = 1; e < NC; ++e) mx = fmaxf(mx, t[e]);
                mx = warp_max<32>(mx);
                float s = 0.0f;
                if (mx != -INFINITY) {   // warp-uniform; else every column of this warp's part is masked
#pragma unroll
                    for (int e = 0; e < NC; ++e) t[e] = exp_shift(t[e] - mx);
                    s = warp_sum<32>(tree_sum(t));
                    if (mx > A + kRaiseB) {
                        const float sc = exp_shift(A - mx);
#pragma unroll
                        for (int e = 0; e < NC; ++e) Sc[e] *= sc;
                        A = mx;
                    }
                    const float w = exp_shift(mx - A);
#pragma unroll
                    for (int e = 0; e < NC; ++e) Sc[e] = fmaf(t[e], w, Sc[e]);
                }
                if (lane == 0) s_rp[il][cpart] = make_float2(mx == -INFINITY ? kNegBig : mx, s);
            }
            __syncthreads();
            // row statistics from the WPR warps of each row
            if (ok && tid < rows) {
                const int64_t i = rg.r0 + int64_t(j) * a.R + tid;
                float2 st = make_float2(0.0f, 0.0f);
                if (i < l1 && l2 > 0) {
                    float mm = kNegBig, ss = 0.0f;
#pragma unroll
                    for (int c = 0; c < WPR; ++c) lse_merge(mm, ss, s_rp[tid][c].x, s_rp[tid][c].y);
                    st = make_float2(mm, ss > 0.0f ? 1.0f / ss : 0.0f);
                }
                a.rstat[b * L1 + i] = st;
            }
            if (j == rg.nb - 1) {
                // merge the slots' partials into cp (aliasing the stage buffer:
                // [SLOTS][L2] float2 <= 32 KB); the stage is refilled only after
                // the cluster has read cp
                float2* mb = reinterpret_cast<float2*>(rg.stage(k));
#pragma unroll
                for (int p = 0; p < VPLW; ++p) {
                    const int64_t col = cbase + 4 * lane + 128 * p;
                    if (col < L2) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) mb[slot * L2 + col + e] = make_float2(A, Sc[4 * p + e]);
                    }
                }
                __syncthreads();
                for (int64_t col = tid; col < L2; col += NT) {
                    float mm = kNegBig, ss = 0.0f;
#pragma unroll
                    for (int q = 0; q < SLOTS; ++q) {
                        const float2 v = mb[q * L2 + col];
                        lse_merge(mm, ss, v.x, v.y);
                    }
                    mb[col] = make_float2(mm, ss);   // only this thread reads column col
                }
                cp = mb;
                kcp = k;
            } else {
                cl_next(rg, k, kfail);
            }
        }
        float2* cpx = cp != nullptr ? cp : reinterpret_cast<float2*>(rg.stage(0));
        if (rg.nb == 0)   // no rows: neutral partials (no copies are ever in flight)
            for (int64_t col = tid; col < L2; col += NT) cpx[col] = make_float2(kNegBig, 0.0f);
        if (tid == 0) s_nfix = 0;
        cluster_sync();

        // ---- column reduction: this CTA's slice over the cluster's partials ----
        for (int64_t col = c0 + tid; col < c1; col += NT) {
            float mm = kNegBig, ss = 0.0f;
            for (uint32_t rr = 0; rr < kC; ++rr) {
                const float2 q = ld_dsmem2(dsmem(cpx + col, rr));
                lse_merge(mm, ss, q.x, q.y);
            }
            float2 st = make_float2(0.0f, 0.0f);
            if (col < l2) {
                if (ss < kTinyB) s_fix[atomicAdd(&s_nfix, 1)] = int(col);
                else st = make_float2(mm, 1.0f / ss);
            }
            cs[col] = st;
            a.cstat[b * L2 + col] = st;
        }
        __syncthreads();
        for (int f = wid; f < s_nfix; f += NW) {
            const int64_t col = s_fix[f];
            const float2 st = exact_col_stats(sb, L2, l1, col, a.invT);
            if (lane == 0) {
                cs[col] = st;
                a.cstat[b * L2 + col] = st;
            }
        }
        cluster_sync();
        if (kcp >= 0) {   // cp has been read by the whole cluster: refill its stage
            fence_proxy_async_smem();
            __syncthreads();
            cl_next(rg, kcp, kfail);
        }
        for (int64_t col = tid; col < L2; col += NT) {
            const uint32_t owner = uint32_t(col / a.cols_per);
            if (owner != rank) cs[col] = ld_dsmem2(dsmem(cs + col, owner));
        }
        __syncthreads();

        // ---- pass 2: out ----
        for (int j = 0; j < rg.nb; ++j, ++k) {
            const bool ok = cl_wait(rg, k, kfail);
            const T* xs = reinterpret_cast<const T*>(rg.stage(k));
            const int rows = rg.rows_in(j);
            for (int il = slot; ok && il < rows; il += SLOTS) {
                const int64_t i = rg.r0 + int64_t(j) * a.R + il;
                const float2 rs = __ldcg(a.rstat + b * L1 + i);
                float* orow = a.out + (b * L1 + i) * L2;
                const bool live = i < l1;
#pragma unroll
                for (int p = 0; p < VPLW; ++p) {
                    const int64_t col = cbase + 4 * lane + 128 * p;
                    if (col >= L2) continue;
                    float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    if (live && col < l2) {
                        float v[4];
                        ld4s(xs + il * L2 + col, v);
                        const float4 c01 = *reinterpret_cast<const float4*>(cs + col);
                        const float4 c23 = *reinterpret_cast<const float4*>(cs + col + 2);
                        const float2 cc[4] = {make_float2(c01.x, c01.y), make_float2(c01.z, c01.w),
                                              make_float2(c23.x, c23.y), make_float2(c23.z, c23.w)};
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            if (full || col + e < l2) o[e] = bs_vals(__fmul_rn(v[e], a.invT), rs, cc[e]).out;
                    }
                    st4g(orow + col, o, pol_out);
                }
            }
            __syncthreads();
            cl_next(rg, k, kfail);
        }
    }
    cluster_sync();   // no CTA leaves while another may still read its shared memory
    cl_drain(rg, kfail);
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
template <typename T, typename G, int VPL>
__global__ void __launch_bounds__(kBwdWarps * 32, 2) bs_bwd_cluster_kernel(ClArgs a) {
    constexpr int NW = kBwdWarps, S = kBwdStages, NT = NW * 32;
    constexpr int WPR = WL<VPL>::WPR, VPLW = WL<VPL>::VPLW, NC = WL<VPL>::NC, SLOTS = NW / WPR;
    extern __shared__ __align__(128) unsigned char smem[];
    float2* cs = reinterpret_cast<float2*>(smem + size_t(S) * kStage);   // [kMaxL2] column statistics
    float* cd = reinterpret_cast<float*>(cs + kMaxL2);                    // [kMaxL2] cdot
    __shared__ __align__(8) uint64_t bars[S];
    __shared__ float s_rp[64][WPR];   // per-row partial sums of the row's warps

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int slot = wid / WPR, cpart = wid % WPR;
    const int64_t cbase = int64_t(cpart) * 128 * VPLW;
    const int64_t L1 = a.L1, L2 = a.L2;
    const uint32_t rank = cluster_rank();
    ClRing<S> rg = cl_ring_init<S>(a, bars, smem);
    const int64_t c0 = min(L2, int64_t(rank) * a.cols_per), c1 = min(L2, c0 + a.cols_per);
    const uint64_t pol_out = l2_policy_evict_first();
    G* gsim = static_cast<G*>(a.gsim);
    int kfail = -1;
    int k = 0;
    for (int64_t b = rg.cid; b < a.B; b += rg.ncl) {
        int64_t l1, l2;
        window(a.lengths, b, L1, L2, l1, l2);
        const bool full = l2 == L2;
        for (int64_t col = tid; col < L2; col += NT) cs[col] = __ldcg(a.cstat + b * L2 + col);
        __syncthreads();

        // ---- pass 1: rdot and column partials of q ----
        float C[NC];
#pragma unroll
        for (int e = 0; e < NC; ++e) C[e] = 0.0f;
        float* cp = nullptr;
        int kcp = -1;
        for (int j = 0; j < rg.nb; ++j, ++k) {
            const bool ok = cl_wait(rg, k, kfail);
            const T* xs = reinterpret_cast<const T*>(rg.stage(k));
            const float* gs = reinterpret_cast<const float*>(rg.stage(k) + a.tile_off1);
            const int rows = rg.rows_in(j);
            for (int il = slot; ok && il < rows; il += SLOTS) {
                const int64_t i = rg.r0 + int64_t(j) * a.R + il;
                float rd = 0.0f;
                if (i < l1) {
                    const float2 rs = __ldcg(a.rstat + b * L1 + i);
#pragma unroll
                    for (int p = 0; p < VPLW; ++p) {
                        const int64_t col = cbase + 4 * lane + 128 * p;
                        if (col < l2) {
                            float v[4], g[4];
                            ld4s(xs + il * L2 + col, v);
                            ld4s(gs + il * L2 + col, g);
                            const float4 c01 = *reinterpret_cast<const float4*>(cs + col);
                            const float4 c23 = *reinterpret_cast<const float4*>(cs + col + 2);
                            const float2 cc[4] = {make_float2(c01.x, c01.y), make_float2(c01.z, c01.w),
                                                  make_float2(c23.x, c23.y), make_float2(c23.z, c23.w)};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                if (full || col + e < l2) {
                                    const BsVals q = bs_vals(__fmul_rn(v[e], a.invT), rs, cc[e]);
                                    const float qq = (g[e] * 0.5f) * q.iout * q.rc;
                                    rd += qq;
                                    C[4 * p + e] += qq;
                                }
                            }
                        }
                    }
                }
                rd = warp_sum<32>(rd);
                if (lane == 0) s_rp[il][cpart] = rd;
            }
            __syncthreads();
            if (ok && tid < rows) {
                float rd = 0.0f;
#pragma unroll
                for (int c = 0; c < WPR; ++c) rd += s_rp[tid][c];
                a.rdot[b * L1 + rg.r0 + int64_t(j) * a.R + tid] = rd;
            }
            if (j == rg.nb - 1) {
                float* mb = reinterpret_cast<float*>(rg.stage(k));   // [SLOTS][L2] <= 16 KB
#pragma unroll
                for (int p = 0; p < VPLW; ++p) {
                    const int64_t col = cbase + 4 * lane + 128 * p;
                    if (col < L2) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) mb[slot * L2 + col + e] = C[4 * p + e];
                    }
                }
                __syncthreads();
                for (int64_t col = tid; col < L2; col += NT) {
                    float sum = 0.0f;
#pragma unroll
                    for (int q = 0; q < SLOTS; ++q) sum += mb[q * L2 + col];
                    mb[col] = sum;   // only this thread reads column col
                }
                cp = mb;
                kcp = k;
            } else {
                cl_next(rg, k, kfail);
            }
        }
        float* cpx = cp != nullptr ? cp : reinterpret_cast<float*>(rg.stage(0));
        if (rg.nb == 0)
            for (int64_t col = tid; col < L2; col += NT) cpx[col] = 0.0f;
        cluster_sync();

        // ---- column reduction ----
        for (int64_t col = c0 + tid; col < c1; col += NT) {
            float sum = 0.0f;
            for (uint32_t rr = 0; rr < kC; ++rr) sum += ld_dsmem(dsmem(cpx + col, rr));
            cd[col] = sum;
        }
        cluster_sync();
        if (kcp >= 0) {
            fence_proxy_async_smem();
            __syncthreads();
            cl_next(rg, kcp, kfail);
        }
        for (int64_t col = tid; col < L2; col += NT) {
            const uint32_t owner = uint32_t(col / a.cols_per);
            if (owner != rank) cd[col] = ld_dsmem(dsmem(cd + col, owner));
        }
        __syncthreads();

        // ---- pass 2: gradient ----
        for (int j = 0; j < rg.nb; ++j, ++k) {
            const bool ok = cl_wait(rg, k, kfail);
            const T* xs = reinterpret_cast<const T*>(rg.stage(k));
            const float* gs = reinterpret_cast<const float*>(rg.stage(k) + a.tile_off1);
            const int rows = rg.rows_in(j);
            for (int il = slot; ok && il < rows; il += SLOTS) {
                const int64_t i = rg.r0 + int64_t(j) * a.R + il;
                const float2 rs = __ldcg(a.rstat + b * L1 + i);
                const float rd = __ldcg(a.rdot + b * L1 + i);
                G* grow = gsim + (b * L1 + i) * L2;
                const bool live = i < l1;
                float acc = 0.0f;
#pragma unroll
                for (int p = 0; p < VPLW; ++p) {
                    const int64_t col = cbase + 4 * lane + 128 * p;
                    if (col >= L2) continue;
                    float gr[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    if (live && col < l2) {
                        float v[4], g[4];
                        ld4s(xs + il * L2 + col, v);
                        ld4s(gs + il * L2 + col, g);
                        const float4 c01 = *reinterpret_cast<const float4*>(cs + col);
                        const float4 c23 = *reinterpret_cast<const float4*>(cs + col + 2);
                        const float4 d4 = *reinterpret_cast<const float4*>(cd + col);
                        const float2 cc[4] = {make_float2(c01.x, c01.y), make_float2(c01.z, c01.w),
                                              make_float2(c23.x, c23.y), make_float2(c23.z, c23.w)};
                        const float cdv[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            if (full || col + e < l2) {
                                const BsVals q = bs_vals(__fmul_rn(v[e], a.invT), rs, cc[e]);
                                const float qq = (g[e] * 0.5f) * q.iout * q.rc;
                                gr[e] = (2.0f * qq - rd * q.row - cdv[e] * q.col) * a.invT;
                                acc = fmaf(gr[e], v[e] * a.invT, acc);
                            }
                        }
                    }
                    st4g(grow + col, gr, pol_out);
                }
                if (a.tau_row != nullptr) {
                    acc = warp_sum<32>(acc);
                    if (lane == 0) s_rp[il][cpart] = acc;
                }
            }
            __syncthreads();
            if (a.tau_row != nullptr && ok && tid < rows) {
                float acc = 0.0f;
#pragma unroll
                for (int c = 0; c < WPR; ++c) acc += s_rp[tid][c];
                a.tau_row[b * L1 + rg.r0 + int64_t(j) * a.R + tid] = acc;
            }
            cl_next(rg, k, kfail);
        }
    }
    cluster_sync();
    cl_drain(rg, kfail);
}

__global__ void bsf_batch_sum_kernel(const float* __restrict__ row_part, float* __restrict__ outv, int64_t B,
                                     int64_t n, float scale) {
    const int lane = threadIdx.x & 31;
    const int64_t b = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= B) return;
    float acc = 0.0f;
    for (int64_t i = lane; i < n; i += 32) acc += row_part[b * n + i];
    acc = warp_sum<32>(acc);
    if (lane == 0) outv[b] = acc * scale;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
int vpl_of(int64_t L2) { return L2 <= 128 ? 1 : L2 <= 256 ? 2 : L2 <= 512 ? 4 : 8; }

// Rows per ring block: as many as fit one stage, a multiple of the warp
// count, at most 64.
int rows_per_block(int64_t row_bytes_total, int nw) {
    int64_t r = kStage / row_bytes_total;
    r = std::min<int64_t>(r, 64);
    r = (r / nw) * nw;
    return int(std::max<int64_t>(r, 1));
}

// DOT_B200_BS_SMEM_PAD_KB adds dynamic shared memory per CTA (tuning runs:
// fewer resident CTAs, hence fewer problems in flight).
size_t smem_pad() {
    static size_t v = [] {
        const char* e = std::getenv("DOT_B200_BS_SMEM_PAD_KB");
        const long kb = e ? std::atol(e) : 0;
        return size_t(kb > 0 && kb < 128 ? kb : 0) << 10;
    }();
    return v;
}
size_t fwd_smem() { return size_t(kFwdStages) * kStage + kMaxL2 * sizeof(float2) + smem_pad(); }
size_t bwd_smem() {
    return size_t(kBwdStages) * kStage + kMaxL2 * sizeof(float2) + kMaxL2 * sizeof(float) + smem_pad();
}

// Row slots of a CTA (warps / warps per row).
int slots_for(int64_t L2, int nw) { return vpl_of(L2) >= 8 ? nw / 2 : nw; }

cudaLaunchConfig_t cluster_config(int grid, int threads, size_t smem, cudaStream_t st, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(grid));
    cfg.blockDim = dim3(unsigned(threads));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kC;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

// Persistent grid: as many clusters as the GPU holds at once, at most B.
template <typename K>
int cluster_grid(K kernel, int threads, size_t smem, int64_t B, cudaStream_t st) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cluster_config(kC, threads, smem, st, attr);
    int ncl = 0;
    if (cudaOccupancyMaxActiveClusters(&ncl, kernel, &cfg) != cudaSuccess || ncl < 1) {
        cudaGetLastError();
        ncl = 1;
    }
    return int(std::min<int64_t>(ncl, B)) * kC;
}

ClArgs base_args(const void* sim, int esz, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau,
                 int nw, bool with_grad) {
    ClArgs a{};
    a.src[0] = static_cast<const unsigned char*>(sim);
    a.row_bytes[0] = uint32_t(L2 * esz);
    a.nsrc = 1;
    const int64_t row_total = L2 * esz + (with_grad ? L2 * 4 : 0);
    a.R = rows_per_block(row_total, slots_for(L2, nw));
    if (with_grad) {
        a.nsrc = 2;
        a.row_bytes[1] = uint32_t(L2 * 4);
        a.tile_off1 = uint32_t((int64_t(a.R) * L2 * esz + 127) / 128 * 128);
    }
    a.lengths = lengths;
    a.B = B;
    a.L1 = L1;
    a.L2 = L2;
    a.rows_per = (L1 + kC - 1) / kC;
    a.cols_per = (L2 + kC - 1) / kC;
    a.invT = 1.0f / tau;
    return a;
}

template <typename T, int VPL>
int fwd_impl(const T* sim, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau, float* out,
             float2* rstat, float2* cstat, void* ws, cudaStream_t st) {
    ClArgs a = base_args(sim, sizeof(T), lengths, B, L1, L2, tau, kFwdWarps, false);
    a.rstat = rstat;
    a.cstat = cstat;
    a.out = out;
    a.err = static_cast<int32_t*>(ws);
    cudaMemsetAsync(a.err, 0, sizeof(int32_t), st);
    const int grid = cluster_grid(bs_fwd_cluster_kernel<T, VPL>, kFwdWarps * 32, fwd_smem(), B, st);
    {
        ProfScope ps(DOT_K_BS_FWD, st);
        cudaLaunchAttribute attr[1];
        cudaLaunchConfig_t cfg = cluster_config(grid, kFwdWarps * 32, fwd_smem(), st, attr);
        cudaLaunchKernelEx(&cfg, bs_fwd_cluster_kernel<T, VPL>, a);
    }
    return check_launch("bidirectional softmax forward (cluster)");
}

template <typename T, typename G, int VPL>
int bwd_impl(const T* sim, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau, const float2* rstat,
             const float2* cstat, const float* gout, G* gsim, float* gtau, void* ws, cudaStream_t st) {
    ClArgs a = base_args(sim, sizeof(T), lengths, B, L1, L2, tau, kBwdWarps, true);
    a.src[1] = reinterpret_cast<const unsigned char*>(gout);
    a.rstat = const_cast<float2*>(rstat);
    a.cstat = const_cast<float2*>(cstat);
    a.gsim = gsim;
    Carve cv(ws);
    a.err = cv.take<int32_t>(1);
    a.rdot = cv.take<float>(size_t(B * L1));
    float* tau_row = cv.take<float>(size_t(B * L1));
    a.tau_row = gtau ? tau_row : nullptr;
    cudaMemsetAsync(a.err, 0, sizeof(int32_t), st);
    const int grid = cluster_grid(bs_bwd_cluster_kernel<T, G, VPL>, kBwdWarps * 32, bwd_smem(), B, st);
    {
        ProfScope ps(DOT_K_BS_BWD, st);
        cudaLaunchAttribute attr[1];
        cudaLaunchConfig_t cfg = cluster_config(grid, kBwdWarps * 32, bwd_smem(), st, attr);
        cudaLaunchKernelEx(&cfg, bs_bwd_cluster_kernel<T, G, VPL>, a);
    }
    if (gtau != nullptr) {
        ProfScope ps(DOT_K_BS_BWD, st);
        bsf_batch_sum_kernel<<<unsigned(ceil_div(B, 8)), 256, 0, st>>>(tau_row, gtau, B, L1, -1.0f);
    }
    return check_launch("bidirectional softmax backward (cluster)");
}

template <typename T>
int fwd_dispatch(const T* sim, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau, float* out,
                 float2* rs, float2* cs, void* ws, cudaStream_t st) {
    switch (vpl_of(L2)) {
        case 1: return fwd_impl<T, 1>(sim, lengths, B, L1, L2, tau, out, rs, cs, ws, st);
        case 2: return fwd_impl<T, 2>(sim, lengths, B, L1, L2, tau, out, rs, cs, ws, st);
        case 4: return fwd_impl<T, 4>(sim, lengths, B, L1, L2, tau, out, rs, cs, ws, st);
        default: return fwd_impl<T, 8>(sim, lengths, B, L1, L2, tau, out, rs, cs, ws, st);
    }
}

template <typename T, typename G>
int bwd_dispatch(const T* sim, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau, const float2* rs,
                 const float2* cs, const float* gout, G* gsim, float* gtau, void* ws, cudaStream_t st) {
    switch (vpl_of(L2)) {
        case 1: return bwd_impl<T, G, 1>(sim, lengths, B, L1, L2, tau, rs, cs, gout, gsim, gtau, ws, st);
        case 2: return bwd_impl<T, G, 2>(sim, lengths, B, L1, L2, tau, rs, cs, gout, gsim, gtau, ws, st);
        case 4: return bwd_impl<T, G, 4>(sim, lengths, B, L1, L2, tau, rs, cs, gout, gsim, gtau, ws, st);
        default: return bwd_impl<T, G, 8>(sim, lengths, B, L1, L2, tau, rs, cs, gout, gsim, gtau, ws, st);
    }
}

}  // namespace

// dst: out (forward, fp32) or grad_sim (backward, dst_dtype); gout non-null
// for the backward.
bool bsf_supported(int64_t B, int64_t L1, int64_t L2, int dtype, const void* sim, const void* gout, const void* dst,
                   int dst_dtype) {
    auto aligned = [](const void* p, uintptr_t a) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) % a) == 0; };
    if (L2 < 4 || L2 > kMaxL2 || L1 < 1 || B < 1) return false;
    if (dtype == DOT_F32 ? (L2 % 4) != 0 : (L2 % 8) != 0) return false;
    const int64_t esz = dtype == DOT_F32 ? 4 : 2;
    const int R = gout ? rows_per_block(L2 * (esz + 4), slots_for(L2, kBwdWarps))
                       : rows_per_block(L2 * esz, slots_for(L2, kFwdWarps));
    // the block sequence index of a CTA is 32-bit
    const int64_t nb = ((L1 + kC - 1) / kC + R - 1) / R;
    if (2 * nb * B >= (int64_t(1) << 31)) return false;
    return aligned(sim, 16) && aligned(gout, 16) && aligned(dst, dst_dtype == DOT_F32 ? 16 : 8);
}

size_t bsf_fwd_ws(int64_t, int64_t, int64_t) { return 256; }

size_t bsf_bwd_ws(int64_t B, int64_t L1, int64_t) {
    Carve c(nullptr);
    c.take<int32_t>(1);
    c.take<float>(size_t(B * L1));
    c.take<float>(size_t(B * L1));
    return c.size();
}

int bsf_fwd(const void* sim, int dtype, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau,
            float* out, float* row_stats, float* col_stats, void* ws, cudaStream_t st) {
    float2* rs = reinterpret_cast<float2*>(row_stats);
    float2* cs = reinterpret_cast<float2*>(col_stats);
    if (dtype == DOT_F32)
        return fwd_dispatch(static_cast<const float*>(sim), lengths, B, L1, L2, tau, out, rs, cs, ws, st);
    return fwd_dispatch(static_cast<const __nv_bfloat16*>(sim), lengths, B, L1, L2, tau, out, rs, cs, ws, st);
}

int bsf_bwd(const void* sim, int dtype, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau,
            const float* row_stats, const float* col_stats, const float* gout, void* gsim, int gdtype, float* gtau,
            void* ws, cudaStream_t st) {
    const float2* rs = reinterpret_cast<const float2*>(row_stats);
    const float2* cs = reinterpret_cast<const float2*>(col_stats);
    if (dtype == DOT_F32) {
        const float* s = static_cast<const float*>(sim);
        if (gdtype == DOT_F32)
            return bwd_dispatch(s, lengths, B, L1, L2, tau, rs, cs, gout, static_cast<float*>(gsim), gtau, ws, st);
        return bwd_dispatch(s, lengths, B, L1, L2, tau, rs, cs, gout, static_cast<__nv_bfloat16*>(gsim), gtau, ws, st);
    }
    const __nv_bfloat16* s = static_cast<const __nv_bfloat16*>(sim);
    if (gdtype == DOT_F32)
        return bwd_dispatch(s, lengths, B, L1, L2, tau, rs, cs, gout, static_cast<float*>(gsim), gtau, ws, st);
    return bwd_dispatch(s, lengths, B, L1, L2, tau, rs, cs, gout, static_cast<__nv_bfloat16*>(gsim), gtau, ws, st);
}

}  // namespace dotb

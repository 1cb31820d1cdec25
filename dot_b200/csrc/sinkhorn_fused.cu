// Fused single-pass Sinkhorn iterations for m <= 1024 (m % 4 == 0).
//
// One kernel launch per iteration reads the B x n x m matrix once (the
// streaming two-kernel path in sinkhorn_stream.cu reads it twice):
//
//   forward   for each row i of the CTA's rows:   u_i = la_i - LSE_j(K_ij + v_j)
//             then, with the fresh u, per-column partials of LSE_i(K_ij + u_i)
//   backward  lambda_i = (sum_k P G - sum_k P_ik mu_k) / max(sum_k P, 1e-12)
//             then per-column partials of sum_i P_ik lambda_i
//
// This is exactly the reference's Gauss-Seidel order (u from the previous v,
// v from the new u: src/sinkhorn/torch_cuda.cpp:200-223; lambda from the
// previous mu, mu from the new lambda: kernels.cu:1715-1718).
//
// Work decomposition: grid (nseg, B); a CTA owns a segment of consecutive
// rows of one problem and streams it through shared memory in row blocks of
// R rows (R*m <= 8192 floats, 32 KB) with double-buffered 1-D bulk copies
// (cp.async.bulk, the TMA engine) completing on mbarriers.  Warp per row; each
// lane owns fixed columns, so after its row's reduction it folds the same
// registers into its columns' running partials (no second pass over shared
// memory).  At the end of its segment a CTA merges its warps' partials and
// publishes them; the last CTA of the problem to finish (atomic arrival
// counter, no waiting) merges the nseg partials in segment order and writes v
// (or mu), so results are deterministic.  The next launch consumes them.
#include <cmath>

#include "common.cuh"
#include "internal.h"
#include "sinkhorn.h"
#include "tma.cuh"

namespace dotb {

namespace {

constexpr int kFT = 256;              // threads per CTA
constexpr int kFW = kFT / 32;         // warps per CTA
constexpr int kTileFloats = 8192;     // one row-block buffer (32 KB)
constexpr size_t kFusedSmem = 2 * kTileFloats * sizeof(float);

template <int VPL>
struct FCfg {
    static constexpr int R = 64 / VPL;    // rows per block (R * 128 * VPL floats = 32 KB)
    static constexpr int RPW = R / kFW;   // rows per warp per block
};

struct FusedCommon {
    const float* data;   // X (forward) or P (backward), [B, n, m]
    int64_t n, m;
    int64_t seg_rows;    // rows per segment (multiple of R)
    int nseg;
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
    float2* part;        // [B, nseg, m] column (max, sum) partials
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
    float* part;         // [B, nseg, m] column sums
};

// Double-buffered row-block stream of one CTA's segment.
struct BlockStream {
    float* buf0;         // buffer k at buf0 + k * kTileFloats
    uint64_t* bar;
    const float* src;    // first row of the segment
    int64_t rows, m;
    int R;

    __device__ int nblk() const { return int((rows + R - 1) / R); }
    __device__ int rows_in(int j) const { return int(min(int64_t(R), rows - int64_t(j) * R)); }
    __device__ float* buf(int j) const { return buf0 + (j & 1) * kTileFloats; }
    __device__ void issue(int j) const {   // one thread
        const uint32_t bytes = uint32_t(rows_in(j)) * uint32_t(m) * 4u;
        uint64_t* b = bar + (j & 1);
        mbar_arrive_expect_tx(b, bytes);
        bulk_g2s(buf(j), src + int64_t(j) * R * m, bytes, b);
    }
};

// Shared prologue: barriers, first two copies.
__device__ __forceinline__ BlockStream stream_begin(const FusedCommon& c, int R, uint64_t* bars,
                                                    unsigned char* smem) {
    BlockStream s;
    s.buf0 = reinterpret_cast<float*>(smem);
    s.bar = bars;
    const int64_t b = blockIdx.y;
    const int64_t r0 = int64_t(blockIdx.x) * c.seg_rows;
    s.rows = min(c.n, r0 + c.seg_rows) - r0;
    s.m = c.m;
    s.R = R;
    s.src = c.data + (b * c.n + r0) * c.m;
    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        s.issue(0);
        if (s.nblk() > 1) s.issue(1);
    }
    return s;
}

// After a failed wait: wait (bounded) for copies still in flight into this
// CTA's shared memory before the CTA exits.
__device__ __forceinline__ void stream_drain(const BlockStream& s, int j, int32_t* err) {
    if (threadIdx.x == 0) {
        for (int k = j; k < s.nblk() && k < j + 2; ++k) mbar_wait(s.bar + (k & 1), (k >> 1) & 1, err);
    }
    __syncthreads();
}

// Arrival at the end of a segment; returns true (to every thread) in the CTA
// that arrived last for its problem.
__device__ __forceinline__ bool arrive_last(int32_t* cnt, int nseg, int* s_flag) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *s_flag = (atomicAdd(cnt + blockIdx.y, 1) == nseg - 1) ? 1 : 0;
    __syncthreads();
    const bool last = *s_flag != 0;
    if (last) __threadfence();
    return last;
}

// ---------------------------------------------------------------------------
// Row-owner layout shared by both kernels: warp w takes rows w, w+8, ... of
// each row block; lane l takes columns 4l + 128p (p < VPL) of every row it
// touches.  Each lane therefore sees the same columns in every row and keeps
// their column partials in registers for the whole segment; the 8 warps'
// partials are merged once, at the end of the segment, through shared memory
// (the row-block buffers, free by then).
// ---------------------------------------------------------------------------

// Cross-warp merge buffer layout: [kFW][m] entries of T (float2 or float).
template <typename T>
__device__ __forceinline__ T* merge_slot(unsigned char* smem, int w, int64_t m, int64_t col) {
    return reinterpret_cast<T*>(smem) + int64_t(w) * m + col;
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

template <int VPL, bool FULL>
__global__ void __launch_bounds__(kFT, (VPL >= 8 ? 2 : 3)) skf_fwd_iter_kernel(FwdIter a) {
    using Cfg = FCfg<VPL>;
    constexpr int R = Cfg::R, RPW = Cfg::RPW;
    constexpr int NC = 4 * VPL;   // columns per lane
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ float s_dmax[kFW];
    __shared__ int s_flag;
    __shared__ int s_nfix;
    __shared__ int s_fix[1024];

    if (a.delta != nullptr) {   // device-side early stop (tol > 0)
        if (*reinterpret_cast<volatile int32_t*>(a.status + 2) != 0) return;
        if (a.iter > 0 && a.delta[a.iter - 1] < a.tol) {
            if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) {
                a.status[0] = a.iter;
                a.status[1] = 1;
                a.status[2] = 1;
            }
            return;
        }
    }
    const FusedCommon& c = a.c;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int64_t b = blockIdx.y, m = c.m;
    const int64_t row0 = b * c.n + int64_t(blockIdx.x) * c.seg_rows;   // global row of local row 0
    if (tid == 0) s_nfix = 0;
    BlockStream st = stream_begin(c, R, bars, smem);

    auto live = [&](int p) -> bool { return FULL || (4 * lane + 128 * p) < m; };
    float vr[NC];
#pragma unroll
    for (int p = 0; p < VPL; ++p) {
        const int64_t col = 4 * lane + 128 * p;
        const float4 v4 = live(p) ? *reinterpret_cast<const float4*>(a.v2 + b * m + col) : make_float4(0, 0, 0, 0);
        vr[4 * p + 0] = v4.x;
        vr[4 * p + 1] = v4.y;
        vr[4 * p + 2] = v4.z;
        vr[4 * p + 3] = v4.w;
    }
    float cS[NC];
#pragma unroll
    for (int e = 0; e < NC; ++e) cS[e] = 0.0f;
    float A = kNegBig;   // warp-wide column reference (uniform across the warp)
    float dmax = 0.0f;

    const int nblk = st.nblk();
    for (int j = 0; j < nblk; ++j) {
        const bool ok = mbar_wait(st.bar + (j & 1), (j >> 1) & 1, c.err);
        if (!__syncthreads_and(ok)) {
            stream_drain(st, j, c.err);
            return;
        }
        const float* xs = st.buf(j);
        const int rj = st.rows_in(j);
        auto do_row = [&](int i) {
            float t[NC];
            float mx = kNegBig;
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                if (live(p)) {
                    const float4 x = *reinterpret_cast<const float4*>(xs + i * int(m) + 4 * lane + 128 * p);
                    t[4 * p + 0] = kplus(x.x, a.kinv, vr[4 * p + 0]);
                    t[4 * p + 1] = kplus(x.y, a.kinv, vr[4 * p + 1]);
                    t[4 * p + 2] = kplus(x.z, a.kinv, vr[4 * p + 2]);
                    t[4 * p + 3] = kplus(x.w, a.kinv, vr[4 * p + 3]);
                } else {
                    t[4 * p + 0] = t[4 * p + 1] = t[4 * p + 2] = t[4 * p + 3] = -INFINITY;
                }
            }
#pragma unroll
            for (int e = 0; e < NC; ++e) mx = fmaxf(mx, t[e]);
            // row LSE, max pass then sum pass (the reference's two-pass order)
            mx = warp_max<32>(mx);
#pragma unroll
            for (int e = 0; e < NC; ++e) t[e] = exp_shift(t[e] - mx);   // t now holds E_ij
            const float s = warp_sum<32>(tree_sum(t));
            const int64_t grow = row0 + int64_t(j) * R + i;
            const float unew = (a.la ? a.la[grow] : a.la_def) - lse_finish(mx, s);
            if (lane == 0) {
                if (a.delta != nullptr) dmax = fmaxf(dmax, fabsf(unew - a.u2[grow]));
                a.u2[grow] = unew;
            }
            const float ai = mx + unew;
            if (ai > A + kRaise) {            // warp-uniform
                const float sc = exp_shift(A - ai);
#pragma unroll
                for (int e = 0; e < NC; ++e) cS[e] *= sc;
                A = ai;
            }
            const float w = exp_shift(ai - A);
#pragma unroll
            for (int e = 0; e < NC; ++e) cS[e] = fmaf(t[e], w, cS[e]);
        };
        if (rj == R) {
#pragma unroll
            for (int q = 0; q < RPW; ++q) do_row(wid + kFW * q);
        } else {
            for (int q = 0; q < RPW; ++q)
                if (wid + kFW * q < rj) do_row(wid + kFW * q);
        }
        __syncthreads();   // buffer (j & 1) is free again
        if (tid == 0 && j + 2 < nblk) st.issue(j + 2);
    }

    if (a.delta != nullptr) {
        if (lane == 0) s_dmax[wid] = dmax;
    }
    // cross-warp merge of the column partials through the (now idle) buffers
#pragma unroll
    for (int p = 0; p < VPL; ++p) {
        if (live(p)) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                *merge_slot<float2>(smem, wid, m, 4 * lane + 128 * p + e) =
                    make_float2(A - vr[4 * p + e], cS[4 * p + e]);
        }
    }
    __syncthreads();
    if (a.delta != nullptr && tid == 0) {
        float mx = 0.0f;
#pragma unroll
        for (int w = 0; w < kFW; ++w) mx = fmaxf(mx, s_dmax[w]);
        atomic_max_nonneg(a.delta + a.iter, mx);
    }
    // Finalise one column from its merged (max, sum); flag it for the exact
    // path when the shared-reference sum is too small to trust.
    auto finish = [&](int64_t col, float mm, float ss) {
        if (ss < kTinySum) {
            s_fix[atomicAdd(&s_nfix, 1)] = int(col);
        } else {
            a.v2[b * m + col] = (a.lb ? a.lb[b * m + col] : a.lb_def) - lse_finish(mm, ss);
        }
    };
    float2* mypart = a.part + (b * c.nseg + blockIdx.x) * m;
    for (int64_t col = tid; col < m; col += kFT) {
        float mm = kNegBig, ss = 0.0f;
#pragma unroll
        for (int w = 0; w < kFW; ++w) {
            const float2 pw = *merge_slot<float2>(smem, w, m, col);
            lse_merge(mm, ss, pw.x, pw.y);
        }
        if (c.nseg == 1) finish(col, mm, ss);
        else mypart[col] = make_float2(mm, ss);
    }
    if (c.nseg > 1) {
        if (!arrive_last(c.cnt, c.nseg, &s_flag)) return;
        for (int64_t col = tid; col < m; col += kFT) {
            float mm = kNegBig, ss = 0.0f;
            for (int sg = 0; sg < c.nseg; ++sg) {
                const float2 pp = __ldcg(a.part + (b * c.nseg + sg) * m + col);
                lse_merge(mm, ss, pp.x, pp.y);
            }
            finish(col, mm, ss);
        }
        if (tid == 0) c.cnt[b] = 0;
    } else {
        __threadfence();   // this CTA's u rows are read back by exact_column
    }
    __syncthreads();
    const int nfix = s_nfix;
    for (int k = wid; k < nfix; k += kFW) {
        const int64_t col = s_fix[k];
        const float lse = exact_column(c.data, a.u2, a.kinv, b, c.n, m, col);
        if (lane == 0) a.v2[b * m + col] = (a.lb ? a.lb[b * m + col] : a.lb_def) - lse;
    }
}

// ---------------------------------------------------------------------------
// backward (adjoint) iteration
// ---------------------------------------------------------------------------
template <int VPL, bool FULL>
__global__ void __launch_bounds__(kFT, (VPL >= 8 ? 2 : 3)) skf_bwd_iter_kernel(BwdIter a) {
    using Cfg = FCfg<VPL>;
    constexpr int R = Cfg::R, RPW = Cfg::RPW;
    constexpr int NC = 4 * VPL;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ int s_flag;

    const FusedCommon& c = a.c;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int64_t b = blockIdx.y, m = c.m;
    const int64_t row0 = b * c.n + int64_t(blockIdx.x) * c.seg_rows;
    BlockStream st = stream_begin(c, R, bars, smem);

    auto live = [&](int p) -> bool { return FULL || (4 * lane + 128 * p) < m; };
    float mr[NC];
#pragma unroll
    for (int p = 0; p < VPL; ++p) {
        const int64_t col = 4 * lane + 128 * p;
        const float4 u4 = live(p) ? *reinterpret_cast<const float4*>(a.mu + b * m + col) : make_float4(0, 0, 0, 0);
        mr[4 * p + 0] = u4.x;
        mr[4 * p + 1] = u4.y;
        mr[4 * p + 2] = u4.z;
        mr[4 * p + 3] = u4.w;
    }
    float acc[NC];
#pragma unroll
    for (int e = 0; e < NC; ++e) acc[e] = 0.0f;

    const int nblk = st.nblk();
    for (int j = 0; j < nblk; ++j) {
        const int rj = st.rows_in(j);
        float2 ri[RPW];   // row invariants, loaded before waiting on the block
#pragma unroll
        for (int q = 0; q < RPW; ++q) {
            const int i = wid + kFW * q;
            ri[q] = i < rj ? a.rinv[row0 + int64_t(j) * R + i] : make_float2(0.0f, 1.0f);
        }
        const bool ok = mbar_wait(st.bar + (j & 1), (j >> 1) & 1, c.err);
        if (!__syncthreads_and(ok)) {
            stream_drain(st, j, c.err);
            return;
        }
        const float* ps = st.buf(j);
#pragma unroll
        for (int q = 0; q < RPW; ++q) {
            const int i = wid + kFW * q;
            if (i >= rj) break;
            float pv[NC];
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                if (live(p)) {
                    const float4 x = *reinterpret_cast<const float4*>(ps + int64_t(i) * m + 4 * lane + 128 * p);
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
            const int64_t grow = row0 + int64_t(j) * R + i;
            const float l = (ri[q].x - s) / fmaxf(ri[q].y, kSumFloor);
            if (lane == 0) a.lam[grow] = l;
#pragma unroll
            for (int e = 0; e < NC; ++e) acc[e] += pv[e] * l;
        }
        __syncthreads();
        if (tid == 0 && j + 2 < nblk) st.issue(j + 2);
    }

#pragma unroll
    for (int p = 0; p < VPL; ++p) {
        if (live(p)) {
#pragma unroll
            for (int e = 0; e < 4; ++e) *merge_slot<float>(smem, wid, m, 4 * lane + 128 * p + e) = acc[4 * p + e];
        }
    }
    __syncthreads();
    float* mypart = a.part + (b * c.nseg + blockIdx.x) * m;
    for (int64_t col = tid; col < m; col += kFT) {
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < kFW; ++w) sum += *merge_slot<float>(smem, w, m, col);
        if (c.nseg == 1) {
            const float2 ci = a.cinv[b * m + col];
            a.mu[b * m + col] = (ci.x - sum) / fmaxf(ci.y, kSumFloor);
        } else {
            mypart[col] = sum;
        }
    }
    if (c.nseg == 1) return;
    if (!arrive_last(c.cnt, c.nseg, &s_flag)) return;
    for (int64_t col = tid; col < m; col += kFT) {
        float sum = 0.0f;
        for (int sg = 0; sg < c.nseg; ++sg) sum += __ldcg(a.part + (b * c.nseg + sg) * m + col);
        const float2 ci = a.cinv[b * m + col];
        a.mu[b * m + col] = (ci.x - sum) / fmaxf(ci.y, kSumFloor);
    }
    if (tid == 0) c.cnt[b] = 0;
}

int vpl_for(int64_t m) { return m <= 128 ? 1 : m <= 256 ? 2 : m <= 512 ? 4 : 8; }
int rows_per_block(int64_t m) { return 64 / vpl_for(m); }

template <typename K>
int blocks_per_sm(K kernel) {
    int nb = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kernel, kFT, kFusedSmem);
    return nb > 0 ? nb : 1;
}

int sm_count() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

// Segments per problem: minimise (CTA waves) x (rows per CTA + merge cost).
int choose_nseg(int64_t B, int64_t n, int64_t m, int slots) {
    const int64_t R = rows_per_block(m);
    const int64_t nblk = (n + R - 1) / R;
    int best = 1;
    double best_cost = 1e300;
    for (int64_t blocks_per_seg = 1; blocks_per_seg <= nblk; ++blocks_per_seg) {
        const int64_t nseg = (nblk + blocks_per_seg - 1) / blocks_per_seg;
        if (nseg > 4096) continue;
        const double waves = std::ceil(double(B * nseg) / slots);
        const double cost = waves * double(blocks_per_seg * R + (nseg > 1 ? 3 : 0));
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = int(nseg);
        }
    }
    return best;
}

template <int VPL>
void set_smem_attrs() {
    cudaFuncSetAttribute(skf_fwd_iter_kernel<VPL, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kFusedSmem));
    cudaFuncSetAttribute(skf_bwd_iter_kernel<VPL, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kFusedSmem));
    cudaFuncSetAttribute(skf_fwd_iter_kernel<VPL, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kFusedSmem));
    cudaFuncSetAttribute(skf_bwd_iter_kernel<VPL, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kFusedSmem));
}

void ensure_attrs() {
    // Per-device attribute; cheap enough to set on every call.
    set_smem_attrs<1>();
    set_smem_attrs<2>();
    set_smem_attrs<4>();
    set_smem_attrs<8>();
}

template <int VPL>
void launch_fwd(const FwdIter& a, dim3 grid, cudaStream_t st) {
    if (a.c.m == 128 * VPL) skf_fwd_iter_kernel<VPL, true><<<grid, kFT, kFusedSmem, st>>>(a);
    else skf_fwd_iter_kernel<VPL, false><<<grid, kFT, kFusedSmem, st>>>(a);
}
template <int VPL>
void launch_bwd(const BwdIter& a, dim3 grid, cudaStream_t st) {
    if (a.c.m == 128 * VPL) skf_bwd_iter_kernel<VPL, true><<<grid, kFT, kFusedSmem, st>>>(a);
    else skf_bwd_iter_kernel<VPL, false><<<grid, kFT, kFusedSmem, st>>>(a);
}

}  // namespace

bool sk_fused_supported(int64_t n, int64_t m, const void* data) {
    return n >= 1 && m >= 4 && m <= 1024 && (m % 4) == 0 && (reinterpret_cast<uintptr_t>(data) & 15u) == 0;
}

FusedPlan sk_fused_plan(int64_t B, int64_t n, int64_t m) {
    FusedPlan p;
    const int R = rows_per_block(m);
    ensure_attrs();
    int per_sm = 1;
    switch (vpl_for(m)) {
        case 1: per_sm = blocks_per_sm(skf_fwd_iter_kernel<1, false>); break;
        case 2: per_sm = blocks_per_sm(skf_fwd_iter_kernel<2, false>); break;
        case 4: per_sm = blocks_per_sm(skf_fwd_iter_kernel<4, false>); break;
        default: per_sm = blocks_per_sm(skf_fwd_iter_kernel<8, false>); break;
    }
    const int slots = sm_count() * per_sm;
    p.nseg = choose_nseg(B, n, m, slots);
    const int64_t nblk = (n + R - 1) / R;
    const int64_t bps = (nblk + p.nseg - 1) / p.nseg;
    p.seg_rows = bps * R;
    p.nseg = int((n + p.seg_rows - 1) / p.seg_rows);
    return p;
}

int sk_fused_fwd_iter(const SkFwdArgs& a, const FusedPlan& p, float2* part, int32_t* cnt, float* delta,
                      int iter, cudaStream_t st) {
    ensure_attrs();
    FwdIter f{};
    f.c.data = a.X;
    f.c.n = a.n;
    f.c.m = a.m;
    f.c.seg_rows = p.seg_rows;
    f.c.nseg = p.nseg;
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
    const dim3 grid(unsigned(p.nseg), unsigned(a.B));
    switch (vpl_for(a.m)) {
        case 1: launch_fwd<1>(f, grid, st); break;
        case 2: launch_fwd<2>(f, grid, st); break;
        case 4: launch_fwd<4>(f, grid, st); break;
        default: launch_fwd<8>(f, grid, st); break;
    }
    return DOT_OK;
}

int sk_fused_bwd_iter(const SkBwdArgs& a, const FusedPlan& p, const float2* rinv, const float2* cinv,
                      float* lam, float* mu, float* part, int32_t* cnt, int32_t* err, cudaStream_t st) {
    ensure_attrs();
    BwdIter f{};
    f.c.data = a.P;
    f.c.n = a.n;
    f.c.m = a.m;
    f.c.seg_rows = p.seg_rows;
    f.c.nseg = p.nseg;
    f.c.cnt = cnt;
    f.c.err = err;
    f.rinv = rinv;
    f.cinv = cinv;
    f.lam = lam;
    f.mu = mu;
    f.part = part;
    const dim3 grid(unsigned(p.nseg), unsigned(a.B));
    switch (vpl_for(a.m)) {
        case 1: launch_bwd<1>(f, grid, st); break;
        case 2: launch_bwd<2>(f, grid, st); break;
        case 4: launch_bwd<4>(f, grid, st); break;
        default: launch_bwd<8>(f, grid, st); break;
    }
    return DOT_OK;
}

}  // namespace dotb

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
// (cp.async.bulk, the TMA engine) completing on mbarriers.  Row pass: warp per
// row, lane-strided float4 columns.  Column pass: thread per column, walking
// the block's rows.  At the end of its segment a CTA publishes its column
// partials; the last CTA of the problem to finish (atomic arrival counter,
// no waiting) merges the nseg partials in segment order and writes v (or mu),
// so results are deterministic.  The next launch consumes them.
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
    static constexpr int R = 64 / VPL;                        // rows per block
    static constexpr int RPW = R / kFW;                       // rows per warp (row pass)
    static constexpr int CPT = (128 * VPL + kFT - 1) / kFT;   // columns per thread (column pass)
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
// forward iteration
// ---------------------------------------------------------------------------
template <int VPL>
__global__ void __launch_bounds__(kFT, 3) skf_fwd_iter_kernel(FwdIter a) {
    using Cfg = FCfg<VPL>;
    constexpr int R = Cfg::R, RPW = Cfg::RPW, CPT = Cfg::CPT;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ float u_s[R];
    __shared__ float s_dmax[kFW];
    __shared__ int s_flag;

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
    BlockStream st = stream_begin(c, R, bars, smem);

    float4 vr[VPL];
#pragma unroll
    for (int p = 0; p < VPL; ++p) {
        const int64_t col = 4 * lane + 128 * p;
        vr[p] = col < m ? *reinterpret_cast<const float4*>(a.v2 + b * m + col) : make_float4(0, 0, 0, 0);
    }
    float cM[CPT], cS[CPT];
#pragma unroll
    for (int k = 0; k < CPT; ++k) { cM[k] = kNegBig; cS[k] = 0.0f; }
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
        // ---- row pass: warp per row -------------------------------------
#pragma unroll
        for (int q = 0; q < RPW; ++q) {
            const int i = wid + kFW * q;
            if (i < rj) {
                float t[4 * VPL];
                float mx = kNegBig;
#pragma unroll
                for (int p = 0; p < VPL; ++p) {
                    const int col = 4 * lane + 128 * p;
                    if (col < m) {
                        const float4 x = *reinterpret_cast<const float4*>(xs + int64_t(i) * m + col);
                        t[4 * p + 0] = kplus(x.x, a.kinv, vr[p].x);
                        t[4 * p + 1] = kplus(x.y, a.kinv, vr[p].y);
                        t[4 * p + 2] = kplus(x.z, a.kinv, vr[p].z);
                        t[4 * p + 3] = kplus(x.w, a.kinv, vr[p].w);
                    } else {
                        t[4 * p + 0] = t[4 * p + 1] = t[4 * p + 2] = t[4 * p + 3] = -INFINITY;
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) mx = fmaxf(mx, t[4 * p + e]);
                }
                mx = warp_max<32>(mx);
                float s = 0.0f;
#pragma unroll
                for (int e = 0; e < 4 * VPL; ++e) s += exp_shift(t[e] - mx);
                s = warp_sum<32>(s);
                const int64_t grow = row0 + int64_t(j) * R + i;
                const float unew = (a.la ? a.la[grow] : a.la_def) - lse_finish(mx, s);
                if (lane == 0) {
                    if (a.delta != nullptr) dmax = fmaxf(dmax, fabsf(unew - a.u2[grow]));
                    a.u2[grow] = unew;
                    u_s[i] = unew;
                }
            }
        }
        __syncthreads();
        // ---- column pass: thread per column -----------------------------
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            const int col = tid + kFT * k;
            if (col < m) {
                for (int i0 = 0; i0 < rj; i0 += 8) {
                    float t8[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int i = i0 + e;
                        t8[e] = i < rj ? kplus(xs[int64_t(i) * m + col], a.kinv, u_s[i]) : -INFINITY;
                    }
                    lse_push<8>(cM[k], cS[k], t8);
                }
            }
        }
        __syncthreads();   // buffer (j & 1) and u_s are free again
        if (tid == 0 && j + 2 < nblk) st.issue(j + 2);
    }

    if (a.delta != nullptr) {
        if (lane == 0) s_dmax[wid] = dmax;
        __syncthreads();
        if (tid == 0) {
            float mx = 0.0f;
#pragma unroll
            for (int w = 0; w < kFW; ++w) mx = fmaxf(mx, s_dmax[w]);
            atomic_max_nonneg(a.delta + a.iter, mx);
        }
    }

    if (c.nseg == 1) {
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            const int64_t col = tid + kFT * k;
            if (col < m) a.v2[b * m + col] = (a.lb ? a.lb[b * m + col] : a.lb_def) - lse_finish(cM[k], cS[k]);
        }
        return;
    }
    float2* mypart = a.part + (b * c.nseg + blockIdx.x) * m;
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
        const int64_t col = tid + kFT * k;
        if (col < m) mypart[col] = make_float2(cM[k], cS[k]);
    }
    if (!arrive_last(c.cnt, c.nseg, &s_flag)) return;
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
        const int64_t col = tid + kFT * k;
        if (col < m) {
            float mm = kNegBig, ss = 0.0f;
            for (int sg = 0; sg < c.nseg; ++sg) {
                const float2 p = __ldcg(a.part + (b * c.nseg + sg) * m + col);
                lse_merge(mm, ss, p.x, p.y);
            }
            a.v2[b * m + col] = (a.lb ? a.lb[b * m + col] : a.lb_def) - lse_finish(mm, ss);
        }
    }
    if (tid == 0) c.cnt[b] = 0;
}

// ---------------------------------------------------------------------------
// backward (adjoint) iteration
// ---------------------------------------------------------------------------
template <int VPL>
__global__ void __launch_bounds__(kFT, 3) skf_bwd_iter_kernel(BwdIter a) {
    using Cfg = FCfg<VPL>;
    constexpr int R = Cfg::R, RPW = Cfg::RPW, CPT = Cfg::CPT;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ float l_s[R];
    __shared__ int s_flag;

    const FusedCommon& c = a.c;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int64_t b = blockIdx.y, m = c.m;
    const int64_t row0 = b * c.n + int64_t(blockIdx.x) * c.seg_rows;
    BlockStream st = stream_begin(c, R, bars, smem);

    float4 mr[VPL];
#pragma unroll
    for (int p = 0; p < VPL; ++p) {
        const int64_t col = 4 * lane + 128 * p;
        mr[p] = col < m ? *reinterpret_cast<const float4*>(a.mu + b * m + col) : make_float4(0, 0, 0, 0);
    }
    float acc[CPT];
#pragma unroll
    for (int k = 0; k < CPT; ++k) acc[k] = 0.0f;

    const int nblk = st.nblk();
    for (int j = 0; j < nblk; ++j) {
        const bool ok = mbar_wait(st.bar + (j & 1), (j >> 1) & 1, c.err);
        if (!__syncthreads_and(ok)) {
            stream_drain(st, j, c.err);
            return;
        }
        const float* ps = st.buf(j);
        const int rj = st.rows_in(j);
#pragma unroll
        for (int q = 0; q < RPW; ++q) {
            const int i = wid + kFW * q;
            if (i < rj) {
                float s = 0.0f;
#pragma unroll
                for (int p = 0; p < VPL; ++p) {
                    const int col = 4 * lane + 128 * p;
                    if (col < m) {
                        const float4 pv = *reinterpret_cast<const float4*>(ps + int64_t(i) * m + col);
                        s += pv.x * mr[p].x + pv.y * mr[p].y + pv.z * mr[p].z + pv.w * mr[p].w;
                    }
                }
                s = warp_sum<32>(s);
                const int64_t grow = row0 + int64_t(j) * R + i;
                if (lane == 0) {
                    const float2 ri = a.rinv[grow];
                    const float l = (ri.x - s) / fmaxf(ri.y, kSumFloor);
                    a.lam[grow] = l;
                    l_s[i] = l;
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            const int col = tid + kFT * k;
            if (col < m) {
                float s = acc[k];
                for (int i = 0; i < rj; ++i) s += ps[int64_t(i) * m + col] * l_s[i];
                acc[k] = s;
            }
        }
        __syncthreads();
        if (tid == 0 && j + 2 < nblk) st.issue(j + 2);
    }

    if (c.nseg == 1) {
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            const int64_t col = tid + kFT * k;
            if (col < m) {
                const float2 ci = a.cinv[b * m + col];
                a.mu[b * m + col] = (ci.x - acc[k]) / fmaxf(ci.y, kSumFloor);
            }
        }
        return;
    }
    float* mypart = a.part + (b * c.nseg + blockIdx.x) * m;
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
        const int64_t col = tid + kFT * k;
        if (col < m) mypart[col] = acc[k];
    }
    if (!arrive_last(c.cnt, c.nseg, &s_flag)) return;
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
        const int64_t col = tid + kFT * k;
        if (col < m) {
            float s = 0.0f;
            for (int sg = 0; sg < c.nseg; ++sg) s += __ldcg(a.part + (b * c.nseg + sg) * m + col);
            const float2 ci = a.cinv[b * m + col];
            a.mu[b * m + col] = (ci.x - s) / fmaxf(ci.y, kSumFloor);
        }
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
    cudaFuncSetAttribute(skf_fwd_iter_kernel<VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kFusedSmem));
    cudaFuncSetAttribute(skf_bwd_iter_kernel<VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kFusedSmem));
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
    skf_fwd_iter_kernel<VPL><<<grid, kFT, kFusedSmem, st>>>(a);
}
template <int VPL>
void launch_bwd(const BwdIter& a, dim3 grid, cudaStream_t st) {
    skf_bwd_iter_kernel<VPL><<<grid, kFT, kFusedSmem, st>>>(a);
}

}  // namespace

bool sk_fused_supported(int64_t n, int64_t m, const void* data) {
    return n >= 1 && m >= 4 && m <= 1024 && (m % 4) == 0 && (reinterpret_cast<uintptr_t>(data) & 15u) == 0;
}

FusedPlan sk_fused_plan(int64_t B, int64_t n, int64_t m) {
    FusedPlan p;
    const int R = rows_per_block(m);
    const int slots = sm_count() * 3;
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

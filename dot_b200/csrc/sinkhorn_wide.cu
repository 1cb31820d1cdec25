// Fused single-pass Sinkhorn iterations for wide rows (8192 <= m <= 65536,
// m % 32 == 0): one launch per iteration reads the B x n x m matrix once.
//
//   u_i = la_i - LSE_j(K_ij + v_j),  then column partials of LSE_i(K_ij + u_i)
//   with the new u (Gauss-Seidel order, src/sinkhorn/torch_cuda.cpp:200-223).
//
// A row does not fit one CTA's registers, so a thread-block cluster of kWC
// CTAs shares every row: CTA r of a cluster owns columns [r*mc, (r+1)*mc),
// mc = m / kWC, and keeps v and its columns' running partials in registers
// (thread t: columns 4t + 2048q, q < NQ).  The clusters split the B*nbat row
// batches (kWR rows each) into equal contiguous ranges.  Per batch, every CTA
//   pass A   streams its slice of the batch's rows into shared memory (1-D
//            bulk copies on a 3-stage mbarrier ring), forms t = K + v, a
//            warp-wide max, E = exp(t - max) (written back in place) and the
//            warp sums, merges its warps into one (max, sum) per row and
//            stores that pair into every CTA of the cluster (distributed
//            shared memory), then arrives on the cluster barrier;
//   pass B   of the previous batch runs while the barrier completes: the
//            column partials S_j += E_ij * exp(max_i + u_i - A) (one FFMA per
//            element, A a warp-wide reference, as in sinkhorn_fused.cu);
//   merge    after the barrier, each CTA combines the kWC pairs of every row
//            in rank order (all CTAs get the same LSE) into u_i.
// When its range leaves a problem, a CTA publishes its columns' partials;
// the CTA that arrives last among the same-rank CTAs of every cluster that
// touched the problem merges that column slice in cluster order (atomic
// arrival counter, no waiting) and writes v -- or, for a row shard of a
// larger problem, the merged (max, sum) pairs for the cross-GPU combine.
// Columns whose merged sum is too small to trust are recomputed exactly.
#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "common.cuh"
#include "internal.h"
#include "sinkhorn.h"
#include "tma.cuh"

namespace dotb {

namespace {

constexpr int kWC = 8;                 // CTAs per cluster
constexpr int kWS = 3;                 // ring stages
constexpr int kWMaxR = 4;              // rows per batch (at most)

// CTA shapes: (A) 512 threads, 64 KB stages, one CTA per SM; (B) 256
// threads, 32 KB stages, two CTAs per SM (one CTA computes while the other
// waits at its cluster barrier; clusters also pack onto more SMs).
template <int T_, int STAGE_, int MINB_>
struct WCfg {
    static constexpr int T = T_;
    static constexpr int W = T_ / 32;
    static constexpr int STAGE = STAGE_;
    static constexpr int MINB = MINB_;
};
using WideA = WCfg<512, 65536, 1>;
using WideB = WCfg<256, 32768, 2>;
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
__device__ __forceinline__ void w_st_remote(const void* local, uint32_t rank, float2 v) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(local)), "r"(rank));
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(a), "f"(v.x), "f"(v.y) : "memory");
}

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

// Exact column LSE over all n rows of problem b (max pass, then sum pass);
// one warp, strided reads; only for columns flagged by the merge.
__device__ float w_exact_column(const float* X, const float* u2, float kinv, int64_t b, int64_t n, int64_t m,
                                int64_t col) {
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

template <class CFG, int NQ, bool FULL>
__global__ void __launch_bounds__(CFG::T, CFG::MINB) skw_iter_kernel(WideArgs a) {
    constexpr int NC = 4 * NQ, kWT = CFG::T, kWW = CFG::W, kWStage = CFG::STAGE;
    extern __shared__ __align__(128) unsigned char smem[];
    float2* xch = reinterpret_cast<float2*>(smem + size_t(kWS) * kWStage);   // [2][kWC][kWMaxR]
    __shared__ __align__(8) uint64_t bars[kWS];
    __shared__ float2 s_wp[kWW][kWMaxR];   // warp (max, sum) per row
    __shared__ float s_u[2][kWMaxR];       // u of the rows of a batch, by batch parity
    __shared__ int s_flag, s_nfix;
    __shared__ int s_fix[kWFix];

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const uint32_t rank = w_rank(), cid = w_cid();
    const int64_t n = a.n, m = a.m, mc = a.mc;
    const int64_t cbase = int64_t(rank) * mc;
    const int g0 = w_q(a, int(cid)), g1 = w_q(a, int(cid) + 1);
    auto live = [&](int q) -> bool { return FULL || (4 * tid + 4 * kWT * q) < mc; };
    auto stage = [&](int g) -> float* { return reinterpret_cast<float*>(smem + size_t((g - g0) % kWS) * kWStage); };
    auto rows_of = [&](int g) -> int {
        const int jb = g % a.nbat;
        return int(min(int64_t(a.R), n - int64_t(jb) * a.R));
    };
    auto issue = [&](int g) {   // one thread
        const int b = g / a.nbat, jb = g - b * a.nbat;
        const int rows = rows_of(g);
        const uint32_t bytes = uint32_t(mc) * 4u;
        uint64_t* bb = &bars[(g - g0) % kWS];
        mbar_arrive_expect_tx(bb, bytes * uint32_t(rows));
        const float* src = a.X + (int64_t(b) * n + int64_t(jb) * a.R) * m + cbase;
        for (int r = 0; r < rows; ++r) bulk_g2s(stage(g) + int64_t(r) * mc, src + int64_t(r) * m, bytes, bb);
    };

    if (tid == 0) {
#pragma unroll
        for (int k = 0; k < kWS; ++k) mbar_init(&bars[k], 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (tid == 0)
        for (int g = g0; g < g1 && g < g0 + kWS; ++g) issue(g);

    float vr[NC], cS[NC];
    float A = kNegBig;              // warp-wide column reference
    float tmc[kWMaxR], tmp[kWMaxR]; // warp row maxima: current batch, pending batch
    int cur = -1, pend = -1, kfail = -1;

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

    // column update of a batch whose E and u are ready; frees its stage
    auto pass_b = [&](int gp) {
        const float* es = stage(gp);
        const int rows = rows_of(gp);
        if (kfail < 0) {
            for (int ir = 0; ir < rows; ++ir) {
                const float ai = tmp[ir] + s_u[gp & 1][ir];   // warp-uniform
                if (ai > A + kRaiseW) {
                    const float sc = exp_shift(A - ai);
#pragma unroll
                    for (int e = 0; e < NC; ++e) cS[e] *= sc;
                    A = ai;
                }
                const float w = exp_shift(ai - A);
#pragma unroll
                for (int q = 0; q < NQ; ++q) {
                    if (live(q)) {
                        const float4 e4 = *reinterpret_cast<const float4*>(es + int64_t(ir) * mc + 4 * tid + 4 * kWT * q);
                        cS[4 * q + 0] = fmaf(e4.x, w, cS[4 * q + 0]);
                        cS[4 * q + 1] = fmaf(e4.y, w, cS[4 * q + 1]);
                        cS[4 * q + 2] = fmaf(e4.z, w, cS[4 * q + 2]);
                        cS[4 * q + 3] = fmaf(e4.w, w, cS[4 * q + 3]);
                    }
                }
            }
        }
        fence_proxy_async_smem();   // E was written with generic stores; the stage is refilled by a bulk copy
        __syncthreads();
        if (tid == 0 && kfail < 0 && gp + kWS < g1) issue(gp + kWS);
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
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            s_flag = (atomicAdd(a.cnt + int64_t(b) * kWC + rank, 1) == nseg - 1) ? 1 : 0;
            s_nfix = 0;
        }
        __syncthreads();
        if (s_flag == 0) return;
        __threadfence();
        for (int64_t lc = tid; lc < mc; lc += kWT) {
            float mm = kNegBig, ss = 0.0f;
            for (int sg = 0; sg < nseg; ++sg) {
                const float2 pp = __ldcg(a.part + (int64_t(b) * a.maxseg + sg) * m + cbase + lc);
                lse_merge(mm, ss, pp.x, pp.y);
            }
            const int64_t col = cbase + lc;
            if (a.pairs != nullptr) {
                a.pairs[int64_t(b) * m + col] = make_float2(mm, ss);
            } else if (ss < kTinyW) {
                const int k = atomicAdd(&s_nfix, 1);
                if (k < kWFix) s_fix[k] = int(lc);
                else a.v2[int64_t(b) * m + col] = (a.lb ? a.lb[int64_t(b) * m + col] : a.lb_def) - lse_finish(mm, ss);
            } else {
                a.v2[int64_t(b) * m + col] = (a.lb ? a.lb[int64_t(b) * m + col] : a.lb_def) - lse_finish(mm, ss);
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

    for (int g = g0; g < g1; ++g) {
        const int b = g / a.nbat, jb = g - b * a.nbat;
        if (b != cur) {
            if (pend >= 0) {
                pass_b(pend);
                pend = -1;
            }
            if (cur >= 0) flush(cur);
            cur = b;
            load_v(b);
        }
        const int rows = rows_of(g);
        const bool ok = kfail < 0 && __syncthreads_and(mbar_wait_sleep(&bars[(g - g0) % kWS],
                                                                       uint32_t(((g - g0) / kWS) & 1), a.err));
        if (kfail < 0 && !ok) kfail = g;

        // ---- pass A: row partials of this CTA's columns ----
        float* xs = stage(g);
        for (int ir = 0; ir < rows; ++ir) {
            float mx = kNegBig, s = 0.0f;
            if (ok) {
                float t[NC];
#pragma unroll
                for (int q = 0; q < NQ; ++q) {
                    if (live(q)) {
                        const float4 x = *reinterpret_cast<const float4*>(xs + int64_t(ir) * mc + 4 * tid + 4 * kWT * q);
                        t[4 * q + 0] = kplus(x.x, a.kinv, vr[4 * q + 0]);
                        t[4 * q + 1] = kplus(x.y, a.kinv, vr[4 * q + 1]);
                        t[4 * q + 2] = kplus(x.z, a.kinv, vr[4 * q + 2]);
                        t[4 * q + 3] = kplus(x.w, a.kinv, vr[4 * q + 3]);
                    } else {
                        t[4 * q + 0] = t[4 * q + 1] = t[4 * q + 2] = t[4 * q + 3] = -INFINITY;
                    }
                }
#pragma unroll
                for (int e = 0; e < NC; ++e) mx = fmaxf(mx, t[e]);
                mx = warp_max<32>(mx);
#pragma unroll
                for (int e = 0; e < NC; ++e) t[e] = exp_shift(t[e] - mx);
                s = warp_sum<32>(tree_sum(t));
#pragma unroll
                for (int q = 0; q < NQ; ++q) {
                    if (live(q))
                        *reinterpret_cast<float4*>(xs + int64_t(ir) * mc + 4 * tid + 4 * kWT * q) =
                            make_float4(t[4 * q + 0], t[4 * q + 1], t[4 * q + 2], t[4 * q + 3]);
                }
            }
            tmc[ir] = mx;
            if (lane == 0) s_wp[wid][ir] = make_float2(mx, s);
        }
        __syncthreads();
        if (tid < rows * kWC) {   // this CTA's (max, sum) of each row, to every CTA of the cluster
            const int ir = tid / kWC, peer = tid % kWC;
            float mm = kNegBig, ss = 0.0f;
#pragma unroll
            for (int w = 0; w < kWW; ++w) lse_merge(mm, ss, s_wp[w][ir].x, s_wp[w][ir].y);
            w_st_remote(xch + ((g & 1) * kWC + rank) * kWMaxR + ir, uint32_t(peer), make_float2(mm, ss));
        }
        w_arrive();
        if (pend >= 0) pass_b(pend);   // overlaps the exchange
        w_wait();

        // ---- merge: u of this batch's rows (identical in every CTA) ----
        if (tid < rows) {
            float mm = kNegBig, ss = 0.0f;
#pragma unroll
            for (int r = 0; r < kWC; ++r) {
                const float2 q = xch[((g & 1) * kWC + r) * kWMaxR + tid];
                lse_merge(mm, ss, q.x, q.y);
            }
            const int64_t grow = int64_t(b) * n + int64_t(jb) * a.R + tid;
            const float unew = (a.la ? a.la[grow] : a.la_def) - lse_finish(mm, ss);
            s_u[g & 1][tid] = unew;
            a.u2[grow] = unew;   // every rank writes the same value: ordered before its own arrival
        }
        __syncthreads();
#pragma unroll
        for (int ir = 0; ir < kWMaxR; ++ir) tmp[ir] = tmc[ir];
        pend = g;
    }
    if (pend >= 0) pass_b(pend);
    if (cur >= 0) flush(cur);
    if (kfail >= 0 && tid == 0)   // copies still in flight after a failed wait
        for (int g = kfail; g < g1 && g < kfail + kWS; ++g)
            mbar_wait_sleep(&bars[(g - g0) % kWS], uint32_t(((g - g0) / kWS) & 1), nullptr);
}

template <class CFG>
size_t wide_smem() { return size_t(kWS) * CFG::STAGE + 2 * kWC * kWMaxR * sizeof(float2); }

template <class CFG>
cudaLaunchConfig_t wide_config(int grid, cudaStream_t st, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(grid));
    cfg.blockDim = dim3(CFG::T);
    cfg.dynamicSmemBytes = wide_smem<CFG>();
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kWC;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

// DOT_B200_WIDE_CTAS=1 or 2 selects the CTA shape (tuning runs); 2 by
// default where the slice fits it (mc <= 4096), else 1.
int wide_ctas_pref() {
    static int v = [] {
        const char* e = std::getenv("DOT_B200_WIDE_CTAS");
        const int x = e ? std::atoi(e) : 2;
        return x == 1 ? 1 : 2;
    }();
    return v;
}
bool use_b(int64_t mc) { return wide_ctas_pref() == 2 && mc <= 4096; }

template <class CFG>
int nq_of(int64_t mc) {
    const int64_t per = 4 * CFG::T;
    return mc <= per ? 1 : mc <= 2 * per ? 2 : mc <= 4 * per ? 4 : 8;
}

template <class CFG, int NQ>
void launch_nq(const WideArgs& a, cudaStream_t st) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = wide_config<CFG>(a.G * kWC, st, attr);
    if (a.mc == 4 * CFG::T * NQ) cudaLaunchKernelEx(&cfg, skw_iter_kernel<CFG, NQ, true>, a);
    else cudaLaunchKernelEx(&cfg, skw_iter_kernel<CFG, NQ, false>, a);
}

template <class CFG, int NQ>
void set_attr_nq() {
    cudaFuncSetAttribute(skw_iter_kernel<CFG, NQ, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(wide_smem<CFG>()));
    cudaFuncSetAttribute(skw_iter_kernel<CFG, NQ, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(wide_smem<CFG>()));
}

void launch_any(const WideArgs& a, cudaStream_t st) {
    if (use_b(a.mc)) {
        switch (nq_of<WideB>(a.mc)) {
            case 1: launch_nq<WideB, 1>(a, st); break;
            case 2: launch_nq<WideB, 2>(a, st); break;
            default: launch_nq<WideB, 4>(a, st); break;
        }
    } else {
        switch (nq_of<WideA>(a.mc)) {
            case 1: launch_nq<WideA, 1>(a, st); break;
            case 2: launch_nq<WideA, 2>(a, st); break;
            default: launch_nq<WideA, 4>(a, st); break;
        }
    }
}

int max_clusters(bool b_shape) {
    static int cached[2][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const int k = b_shape ? 1 : 0;
    if (dev >= 0 && dev < 64 && cached[k][dev] > 0) return cached[k][dev];
    set_attr_nq<WideA, 1>();
    set_attr_nq<WideA, 2>();
    set_attr_nq<WideA, 4>();
    set_attr_nq<WideB, 1>();
    set_attr_nq<WideB, 2>();
    set_attr_nq<WideB, 4>();
    cudaLaunchAttribute attr[1];
    int ncl = 0;
    cudaError_t e;
    if (b_shape) {
        cudaLaunchConfig_t cfg = wide_config<WideB>(kWC, nullptr, attr);
        e = cudaOccupancyMaxActiveClusters(&ncl, skw_iter_kernel<WideB, 4, true>, &cfg);
    } else {
        cudaLaunchConfig_t cfg = wide_config<WideA>(kWC, nullptr, attr);
        e = cudaOccupancyMaxActiveClusters(&ncl, skw_iter_kernel<WideA, 2, true>, &cfg);
    }
    if (e != cudaSuccess || ncl < 1) {
        cudaGetLastError();
        ncl = 1;
    }
    if (dev >= 0 && dev < 64) cached[k][dev] = ncl;
    return ncl;
}

// Rows per batch: as many rows of the CTA's slice as one stage holds (<= 4).
int wide_rows(int64_t mc) {
    const int64_t stage = use_b(mc) ? WideB::STAGE : WideA::STAGE;
    return int(std::max<int64_t>(1, std::min<int64_t>(kWMaxR, stage / (mc * 4))));
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
    p.G = int(std::min<int64_t>(max_clusters(use_b(p.mc)), p.TB));
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
                       const float* v2, float* u2, float2* pairs, void* ws, cudaStream_t st) {
    const WidePlan p = wide_plan(B, n, m);
    if (p.maxseg > wide_seg_bound(B, n, m))
        return fail(DOT_ERR_WORKSPACE, "wide Sinkhorn: more row segments than the workspace holds");
    Carve c(ws);
    WideArgs w{};
    w.part = c.take<float2>(size_t(B * wide_seg_bound(B, n, m) * m));
    w.cnt = c.take<int32_t>(size_t(B * kWC));
    cudaMemsetAsync(w.cnt, 0, sizeof(int32_t) * size_t(B * kWC), st);
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
    w.err = nullptr;
    ProfScope ps(DOT_K_SK_FWD_ITER, st);
    launch_any(w, st);
    return check_launch("sinkhorn rows + column pairs (wide rows)");
}

}  // namespace dotb

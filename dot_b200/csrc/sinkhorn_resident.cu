// On-chip resident Sinkhorn solvers for small problems: one CTA per problem.
//
// The problem's n x m tile is copied into shared memory once with a 1-D bulk
// copy (cp.async.bulk, the TMA engine) and every iteration runs on it, so HBM
// is read once per call instead of once per iteration.  Used for tol == 0
// (the reference's tol > 0 criterion is global over the batch, which
// independent CTAs cannot evaluate without waiting on one another) when
// n*m*4 fits the shared-memory budget and m % 4 == 0.
//
// Layout: W warps; a warp is split into G = 32/LPR lane groups of LPR lanes,
// each group owning one row at a time; lane l of a group owns columns
// 4*l + 4*LPR*p (p < VPL) of every row it touches.  Per iteration:
//   row pass   t_ij = K_ij + v_j, u_i = la_i - LSE_j t_ij (max then sum,
//              reduced across the group's lanes), and the column sums
//              S_j += E_ij * exp(a_i - A) with E_ij = exp(t_ij - max_i),
//              a_i = max_i + u_i, A a warp-wide reference (see
//              sinkhorn_fused.cu: one exponential per element);
//   merge      per column over the W warps: v_j = lb_j - (A* - v_j + log S_j),
//              with an exact max-based column LSE from shared memory when the
//              merged sum is too small to trust.
// The backward keeps the plan tile resident and runs the Gauss-Seidel adjoint
// sweeps on it (reference: src/sinkhorn/kernels.cu:965-1098).
#include <cmath>

#include "common.cuh"
#include "internal.h"
#include "pack.cuh"
#include "sinkhorn.h"
#include "tma.cuh"

namespace dotb {

namespace {

constexpr float kRaiseR = 60.0f;
constexpr float kTinyR = 8.077935669463161e-28f;   // 2^-90
constexpr int kMaxSmemTile = 160 * 1024;           // bytes of the resident tile

template <int LPR_, int VPL_, int W_, int MINB_>
struct RCfg {
    static constexpr int MINB = MINB_;           // CTAs per SM the launch bounds target
    static constexpr int LPR = LPR_;             // lanes per row
    static constexpr int VPL = VPL_;             // float4 per lane per row
    static constexpr int W = W_;                 // warps
    static constexpr int G = 32 / LPR;           // row groups per warp
    static constexpr int NC = 4 * VPL;           // columns per lane
    static constexpr int CW = 4 * LPR * VPL;     // columns covered
    static constexpr int ROWS_PER_SLOT = W * G;  // rows per pass over the warps
    static constexpr int T = W * 32;
};

// Dynamic shared memory: tile [n*m] | part [W*CW] | v [CW] | aw [W] | sc [W] |
// u [n] | fix [CW] | nfix.  tile, part and v start 16-byte aligned (n*m, W*CW
// and CW are multiples of 4 floats) for float4 access.
template <typename C>
struct RSmem {
    float* tile;
    float* part;   // per-warp column partial sums
    float* u;
    float* v;
    float* aw;     // per-warp reference (forward) ; scratch
    float* sc;     // per-warp scale factors
    int* fix;      // flagged columns
    int* nfix;
    static size_t bytes(int64_t n, int64_t m) {
        size_t b = size_t(n * m) * 4;
        b += size_t(C::W) * C::CW * 4;
        b += size_t(n) * 4 + size_t(C::CW) * 4 + 2 * C::W * 4 + size_t(C::CW) * 4 + 16;
        return (b + 127) & ~size_t(127);
    }
    __device__ static RSmem carve(unsigned char* base, int64_t n, int64_t m) {
        RSmem s;
        float* f = reinterpret_cast<float*>(base);
        s.tile = f;
        f += n * m;
        s.part = f;
        f += C::W * C::CW;
        s.v = f;
        f += C::CW;
        s.aw = f;
        f += C::W;
        s.sc = f;
        f += C::W;
        s.u = f;
        f += n;
        s.fix = reinterpret_cast<int*>(f);
        s.nfix = s.fix + C::CW;
        return s;
    }
};

template <int LPR>
__device__ __forceinline__ float group_max(float v) {
#pragma unroll
    for (int off = LPR / 2; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}
template <int LPR>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int off = LPR / 2; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}
// Reduce across the G groups of a warp (lanes with the same lane % LPR).
template <int LPR>
__device__ __forceinline__ float across_groups_sum(float v) {
#pragma unroll
    for (int off = LPR; off < 32; off <<= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}
template <int LPR>
__device__ __forceinline__ float across_groups_max(float v) {
#pragma unroll
    for (int off = LPR; off < 32; off <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

// Load the b-th n x m tile of src into shared memory with one bulk copy.
__device__ __forceinline__ bool load_tile(float* tile, const float* src, int64_t n, int64_t m, uint64_t* bar,
                                          int32_t* err) {
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t bytes = uint32_t(n * m * 4);
        mbar_arrive_expect_tx(bar, bytes);
        bulk_g2s(tile, src, bytes, bar);
    }
    const bool ok = mbar_wait(bar, 0, err);
    return __syncthreads_and(ok) != 0;
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
// FULL: every row slot holds rows (n % ROWS_PER_SLOT == 0) and the lanes'
// columns are the row (m == CW), so the sweep needs no row or column checks.
template <typename C, bool FULL>
__global__ void __launch_bounds__(C::T, C::MINB) skr_fwd_kernel(SkFwdArgs a) {
    constexpr int LPR = C::LPR, VPL = C::VPL, W = C::W, G = C::G, NC = C::NC;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ float s_red[W];
    const int64_t n = a.n, m = a.m, b = blockIdx.x;
    RSmem<C> S = RSmem<C>::carve(smem, n, m);
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int grp = lane / LPR, gl = lane % LPR;
    int32_t* err = a.status + 3;

    for (int64_t j = tid; j < C::CW; j += C::T) S.v[j] = 0.0f;
    if (!load_tile(S.tile, a.X + b * n * m, n, m, &bar, err)) return;
    // the tile holds K = X * kinv from here on (rounded once, as the reference
    // materialises log_K); the cost epilogue re-reads X
    for (int64_t q = tid; q < (n * m) >> 2; q += C::T) {
        const float4 x = reinterpret_cast<float4*>(S.tile)[q];
        const float2 lo = mul2(make_float2(x.x, x.y), splat2(a.kinv)), hi = mul2(make_float2(x.z, x.w), splat2(a.kinv));
        reinterpret_cast<float4*>(S.tile)[q] = make_float4(lo.x, lo.y, hi.x, hi.y);
    }
    __syncthreads();

    auto colof = [&](int p) { return 4 * gl + 4 * LPR * p; };
    const int nslots = int((n + C::ROWS_PER_SLOT - 1) / C::ROWS_PER_SLOT);
    const float* la = a.la ? a.la + b * n : nullptr;
    const float* lb = a.lb ? a.lb + b * m : nullptr;

    for (int it = 0; it < a.n_iters; ++it) {
        // packed two-lane arithmetic (pack.cuh): element pairs (2k, 2k+1)
        float2 vr[NC / 2];
#pragma unroll
        for (int p = 0; p < VPL; ++p) {
            const float4 v4 = *reinterpret_cast<const float4*>(S.v + colof(p));
            vr[2 * p] = make_float2(v4.x, v4.y);
            vr[2 * p + 1] = make_float2(v4.z, v4.w);
        }
        float2 cs[NC / 2];
#pragma unroll
        for (int k = 0; k < NC / 2; ++k) cs[k] = make_float2(0.0f, 0.0f);
        float A = kNegBig;
        for (int sl = 0; sl < nslots; ++sl) {
            const int64_t i = int64_t(sl) * C::ROWS_PER_SLOT + wid * G + grp;
            const bool rok = FULL || i < n;
            float2 t[NC / 2];
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                const int col = colof(p);
                if (FULL || (rok && col < m)) {
                    const float4 k4 = *reinterpret_cast<const float4*>(S.tile + i * m + col);
                    t[2 * p] = add2(make_float2(k4.x, k4.y), vr[2 * p]);
                    t[2 * p + 1] = add2(make_float2(k4.z, k4.w), vr[2 * p + 1]);
                } else {
                    t[2 * p] = t[2 * p + 1] = make_float2(-INFINITY, -INFINITY);
                }
            }
            const float mx = group_max<LPR>(max_of(t));
            // exp(t - mx) as 2^(t*log2e - mL) in one FFMA, mL = mx*log2e rounded;
            // every term carries 2^cr, cr = mx*log2e - mL exactly (FMA
            // remainder), taken out of the row LSE and the column weight
            const float mxc = fmaxf(mx, -1.0e37f);   // a row of -inf terms keeps mL finite
            const float mL = mxc * kLog2e;
            const float cr = fmaf(mxc, kLog2e, -mL);
            const float2 l2 = splat2(kLog2e), nm = splat2(-mL);
#pragma unroll
            for (int k = 0; k < NC / 2; ++k) {
                const float2 e = fma2(t[k], l2, nm);
                t[k] = make_float2(ex2(e.x), ex2(e.y));
            }
            const float2 s2 = tree_sum2(t);
            const float s = group_sum<LPR>(s2.x + s2.y);
            float ai = -INFINITY;
            if (rok) {
                const float unew = (la ? la[i] : a.la_def) - (mx + (fast_log(fmaxf(s, kSumFloor)) - cr * kLn2));
                if (gl == 0) S.u[i] = unew;
                ai = mx + unew;
            }
            const float amax = across_groups_max<LPR>(ai);
            if (amax > A + kRaiseR) {          // warp-uniform
                const float2 sc = splat2(exp_shift(A - amax));
#pragma unroll
                for (int k = 0; k < NC / 2; ++k) cs[k] = mul2(cs[k], sc);
                A = amax;
            }
            const float2 w = splat2(ex2(fmaf(ai - A, kLog2e, -cr)));   // exp(ai - A) / 2^cr
#pragma unroll
            for (int k = 0; k < NC / 2; ++k) cs[k] = fma2(t[k], w, cs[k]);
        }
#pragma unroll
        for (int k = 0; k < NC / 2; ++k) {
            cs[k].x = across_groups_sum<LPR>(cs[k].x);
            cs[k].y = across_groups_sum<LPR>(cs[k].y);
        }
        if (grp == 0) {
#pragma unroll
            for (int p = 0; p < VPL; ++p)
                *reinterpret_cast<float4*>(S.part + wid * C::CW + colof(p)) =
                    make_float4(cs[2 * p].x, cs[2 * p].y, cs[2 * p + 1].x, cs[2 * p + 1].y);
        }
        if (lane == 0) S.aw[wid] = A;
        __syncthreads();
        if (wid == 0) {
            const float aw = lane < W ? S.aw[lane] : kNegBig;
            const float amax = warp_max<32>(aw);
            if (lane < W) S.sc[lane] = exp_shift(aw - amax);
            if (lane == 0) s_red[0] = amax;
        }
        if (tid == 0) *S.nfix = 0;
        __syncthreads();
        const float amax = s_red[0];
        for (int64_t j = tid; j < m; j += C::T) {
            float sum = 0.0f;
#pragma unroll
            for (int w = 0; w < W; ++w) sum = fmaf(S.part[w * C::CW + j], S.sc[w], sum);
            if (sum < kTinyR) {
                S.fix[atomicAdd(S.nfix, 1)] = int(j);
            } else {
                S.v[j] = (lb ? lb[j] : a.lb_def) - (amax - S.v[j] + logf(sum));
            }
        }
        __syncthreads();
        const int nfix = *S.nfix;
        for (int k = wid; k < nfix; k += W) {   // exact column LSE from the resident tile
            const int64_t j = S.fix[k];
            float mx = kNegBig;
            for (int64_t i = lane; i < n; i += 32) mx = fmaxf(mx, __fadd_rn(S.tile[i * m + j], S.u[i]));
            mx = warp_max<32>(mx);
            float sm = 0.0f;
            for (int64_t i = lane; i < n; i += 32) sm += exp_shift(__fadd_rn(S.tile[i * m + j], S.u[i]) - mx);
            sm = warp_sum<32>(sm);
            if (lane == 0) S.v[j] = (lb ? lb[j] : a.lb_def) - lse_finish(mx, sm);
        }
        if (nfix > 0) __syncthreads();
    }

    // epilogue: potentials, plan (P = safe_exp((K + u_i) + v_j)) and cost
    for (int64_t i = tid; i < n; i += C::T) a.u2[b * n + i] = a.n_iters > 0 ? S.u[i] : 0.0f;
    for (int64_t j = tid; j < m; j += C::T) a.v2[b * m + j] = S.v[j];
    if (a.n_iters == 0)
        for (int64_t i = tid; i < n; i += C::T) S.u[i] = 0.0f;
    __syncthreads();
    float acc = 0.0f;
    float* outb = a.out + b * n * m;
    const float4* xg = reinterpret_cast<const float4*>(a.X + b * n * m);
    const int64_t nm4 = (n * m) >> 2;
    for (int64_t q = tid; q < nm4; q += C::T) {
        const int64_t e0 = q * 4;
        const int64_t i = e0 / m, j = e0 - i * m;
        const float4 k4 = *reinterpret_cast<const float4*>(S.tile + e0);
        const float uu = S.u[i];
        const float t0 = __fadd_rn(__fadd_rn(k4.x, uu), S.v[j + 0]);
        const float t1 = __fadd_rn(__fadd_rn(k4.y, uu), S.v[j + 1]);
        const float t2 = __fadd_rn(__fadd_rn(k4.z, uu), S.v[j + 2]);
        const float t3 = __fadd_rn(__fadd_rn(k4.w, uu), S.v[j + 3]);
        float4 o;
        if (a.out_mode == 0) {
            o = make_float4(safe_expf(t0), safe_expf(t1), safe_expf(t2), safe_expf(t3));
            if (a.cost != nullptr) {
                const float4 x = __ldg(xg + q);
                acc += o.x * x.x + o.y * x.y + o.z * x.z + o.w * x.w;
            }
        } else {
            o = make_float4(t0, t1, t2, t3);
        }
        reinterpret_cast<float4*>(outb)[q] = o;
    }
    if (a.cost != nullptr) {
        acc = warp_sum<32>(acc);
        if (lane == 0) s_red[wid] = acc;
        __syncthreads();
        if (tid == 0) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < W; ++w) tot += s_red[w];
            a.cost[b] = tot;
        }
    }
}

// ---------------------------------------------------------------------------
// backward (implicit adjoint on the resident plan tile)
// ---------------------------------------------------------------------------
template <typename C>
__global__ void __launch_bounds__(C::T, C::MINB) skr_bwd_kernel(SkBwdArgs a, int32_t* err) {
    constexpr int LPR = C::LPR, VPL = C::VPL, W = C::W, G = C::G, NC = C::NC;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ float s_red[W];
    const int64_t n = a.n, m = a.m, b = blockIdx.x;
    RSmem<C> S = RSmem<C>::carve(smem, n, m);
    // reuse of the carve: u -> lambda [n], v -> mu [CW]; the row invariants
    // (sum P G, sum P) live in registers of their row's group, the column
    // invariants in `colinv` below.
    float* lam = S.u;
    float* mu = S.v;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int grp = lane / LPR, gl = lane % LPR;
    auto colof = [&](int p) { return 4 * gl + 4 * LPR * p; };
    const int nslots = int((n + C::ROWS_PER_SLOT - 1) / C::ROWS_PER_SLOT);
    constexpr int MAXSLOTS = 8;
    const float gc = a.gcost ? a.gcost[b] : 0.0f;
    const float* Xb = a.X + b * n * m;
    const float* gPb = a.gP ? a.gP + b * n * m : nullptr;

    for (int64_t j = tid; j < C::CW; j += C::T) mu[j] = 0.0f;
    if (!load_tile(S.tile, a.P + b * n * m, n, m, &bar, err)) return;

    auto G_at = [&](int64_t idx) -> float {   // G = grad_cost_b * X + grad_P (autograd's rounding)
        float g = __fmul_rn(gc, __ldg(Xb + idx));
        if (gPb) g = __fadd_rn(g, __ldg(gPb + idx));
        return g;
    };

    // ---- invariants: row (sum_k P G, sum_k P), column (sum_i P G, sum_i P)
    float rPG[MAXSLOTS], rP[MAXSLOTS];   // rP: 1 / max(sum_k P, 1e-12)
    float cPG[NC], cP[NC];
#pragma unroll
    for (int e = 0; e < NC; ++e) { cPG[e] = 0.0f; cP[e] = 0.0f; }
#pragma unroll
    for (int sl = 0; sl < MAXSLOTS; ++sl) {
        rPG[sl] = 0.0f;
        rP[sl] = 1.0f;
        if (sl >= nslots) continue;
        const int64_t i = int64_t(sl) * C::ROWS_PER_SLOT + wid * G + grp;
        float spg = 0.0f, sp = 0.0f;
        if (i < n) {
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                const int col = colof(p);
                if (col < m) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float pv = S.tile[i * m + col + e];
                        const float gv = G_at(i * m + col + e);
                        spg += pv * gv;
                        sp += pv;
                        cPG[4 * p + e] += pv * gv;
                        cP[4 * p + e] += pv;
                    }
                }
            }
        }
        rPG[sl] = group_sum<LPR>(spg);
        rP[sl] = 1.0f / fmaxf(group_sum<LPR>(sp), kSumFloor);   // reciprocal of the row denominator
    }
    // column invariants: reduce over groups, then over warps through S.part
    float* cinv_pg = S.part;
#pragma unroll
    for (int e = 0; e < NC; ++e) {
        cPG[e] = across_groups_sum<LPR>(cPG[e]);
        cP[e] = across_groups_sum<LPR>(cP[e]);
    }
    // two rounds through the per-warp partial buffer: first sum P G, then sum P
    __shared__ float s_cpg[C::CW];
    __shared__ float s_cp[C::CW];
    if (grp == 0) {
#pragma unroll
        for (int p = 0; p < VPL; ++p)
#pragma unroll
            for (int e = 0; e < 4; ++e) cinv_pg[wid * C::CW + colof(p) + e] = cPG[4 * p + e];
    }
    __syncthreads();
    for (int j = tid; j < C::CW; j += C::T) {
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < W; ++w) s += cinv_pg[w * C::CW + j];
        s_cpg[j] = s;
    }
    __syncthreads();
    if (grp == 0) {
#pragma unroll
        for (int p = 0; p < VPL; ++p)
#pragma unroll
            for (int e = 0; e < 4; ++e) cinv_pg[wid * C::CW + colof(p) + e] = cP[4 * p + e];
    }
    __syncthreads();
    for (int j = tid; j < C::CW; j += C::T) {
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < W; ++w) s += cinv_pg[w * C::CW + j];
        s_cp[j] = 1.0f / fmaxf(s, kSumFloor);   // reciprocal of the column denominator
    }
    __syncthreads();

    // ---- Gauss-Seidel sweeps (packed two-lane arithmetic, pairs of columns)
    for (int it = 0; it < a.bwd_iters; ++it) {
        float2 mr[NC / 2], acc[NC / 2];
#pragma unroll
        for (int p = 0; p < VPL; ++p) {
            const float4 u4 = *reinterpret_cast<const float4*>(mu + colof(p));
            mr[2 * p] = make_float2(u4.x, u4.y);
            mr[2 * p + 1] = make_float2(u4.z, u4.w);
        }
#pragma unroll
        for (int k = 0; k < NC / 2; ++k) acc[k] = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int sl = 0; sl < MAXSLOTS; ++sl) {
            if (sl >= nslots) break;
            const int64_t i = int64_t(sl) * C::ROWS_PER_SLOT + wid * G + grp;
            const bool rok = i < n;
            float2 pv[NC / 2];
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                const int col = colof(p);
                if (rok && col < m) {
                    const float4 x = *reinterpret_cast<const float4*>(S.tile + i * m + col);
                    pv[2 * p] = make_float2(x.x, x.y);
                    pv[2 * p + 1] = make_float2(x.z, x.w);
                } else {
                    pv[2 * p] = pv[2 * p + 1] = make_float2(0.0f, 0.0f);
                }
            }
            float2 sq[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};   // four independent chains
#pragma unroll
            for (int k = 0; k < NC / 2; ++k) sq[k & 1] = fma2(pv[k], mr[k], sq[k & 1]);
            const float2 sq2 = add2(sq[0], sq[1]);
            const float s = group_sum<LPR>(sq2.x + sq2.y);
            const float l = rok ? (rPG[sl] - s) * rP[sl] : 0.0f;
            if (rok && gl == 0) lam[i] = l;
            const float2 l2 = splat2(l);
#pragma unroll
            for (int k = 0; k < NC / 2; ++k) acc[k] = fma2(pv[k], l2, acc[k]);
        }
#pragma unroll
        for (int k = 0; k < NC / 2; ++k) {
            acc[k].x = across_groups_sum<LPR>(acc[k].x);
            acc[k].y = across_groups_sum<LPR>(acc[k].y);
        }
        if (grp == 0) {
#pragma unroll
            for (int p = 0; p < VPL; ++p)
                *reinterpret_cast<float4*>(S.part + wid * C::CW + colof(p)) =
                    make_float4(acc[2 * p].x, acc[2 * p].y, acc[2 * p + 1].x, acc[2 * p + 1].y);
        }
        __syncthreads();
        for (int64_t j = tid; j < m; j += C::T) {
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < W; ++w) s += S.part[w * C::CW + j];
            mu[j] = (s_cpg[j] - s) * s_cp[j];
        }
        __syncthreads();
    }
    if (a.bwd_iters == 0)
        for (int64_t i = tid; i < n; i += C::T) lam[i] = 0.0f;
    __syncthreads();

    // ---- gradient epilogue
    float accT = 0.0f;
    const int64_t nm = n * m;
    for (int64_t idx = tid; idx < nm; idx += C::T) {
        const int64_t i = idx / m, j = idx - i * m;
        const float x = __ldg(Xb + idx);
        const float p = S.tile[idx];
        const float centred = G_at(idx) - lam[i] - mu[j];
        const float g = p * centred / a.tau;
        a.gX[b * nm + idx] = __fadd_rn(a.sign * g, __fmul_rn(gc, p));
        accT += g * (a.sign * x);
    }
    if (a.gtau != nullptr) {
        accT = warp_sum<32>(accT);
        if (lane == 0) s_red[wid] = accT;
        __syncthreads();
        if (tid == 0) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < W; ++w) tot += s_red[w];
            a.gtau[b] = tot * (-1.0f / a.tau);
        }
    }
}

// ---------------------------------------------------------------------------
// configurations
// ---------------------------------------------------------------------------
using CfgS = RCfg<8, 2, 8, 4>;    // m <= 64,  32 rows per slot
using CfgM = RCfg<8, 4, 8, 3>;    // m <= 128, 32 rows per slot
using CfgL = RCfg<16, 4, 8, 2>;   // m <= 256, 16 rows per slot

template <typename C>
bool fits(int64_t n, int64_t m) {
    if (m > C::CW || n > int64_t(C::ROWS_PER_SLOT) * 8) return false;
    return RSmem<C>::bytes(n, m) <= size_t(kMaxSmemTile) + 32 * 1024 && n * m * 4 <= kMaxSmemTile;
}

enum class RKind { None, S, M, L };

RKind pick(int64_t n, int64_t m) {
    if (m % 4 != 0 || n < 1) return RKind::None;
    if (m <= 64 && fits<CfgS>(n, m)) return RKind::S;
    if (m <= 128 && fits<CfgM>(n, m)) return RKind::M;
    if (m <= 256 && fits<CfgL>(n, m)) return RKind::L;
    return RKind::None;
}

template <typename C>
int launch_fwd(const SkFwdArgs& a, cudaStream_t st) {
    const size_t sm = RSmem<C>::bytes(a.n, a.m);
    ProfScope ps(DOT_K_SK_RESIDENT, st);
    if (a.n % C::ROWS_PER_SLOT == 0 && a.m == C::CW) {
        cudaFuncSetAttribute(skr_fwd_kernel<C, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
        skr_fwd_kernel<C, true><<<unsigned(a.B), C::T, sm, st>>>(a);
    } else {
        cudaFuncSetAttribute(skr_fwd_kernel<C, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
        skr_fwd_kernel<C, false><<<unsigned(a.B), C::T, sm, st>>>(a);
    }
    return check_launch("sinkhorn forward (resident)");
}

template <typename C>
int launch_bwd(const SkBwdArgs& a, int32_t* err, cudaStream_t st) {
    const size_t sm = RSmem<C>::bytes(a.n, a.m);
    cudaFuncSetAttribute(skr_bwd_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
    ProfScope ps(DOT_K_SK_RESIDENT, st);
    skr_bwd_kernel<C><<<unsigned(a.B), C::T, sm, st>>>(a, err);
    return check_launch("sinkhorn backward (resident)");
}

__global__ void skr_status_kernel(int32_t* status, int n_iters) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        status[0] = n_iters;
        status[1] = 0;
    }
}

}  // namespace

bool sk_resident_supported(int64_t n, int64_t m) { return pick(n, m) != RKind::None; }

size_t sk_resident_fwd_ws(int64_t, int64_t, int64_t, bool) { return 0; }
size_t sk_resident_bwd_ws(int64_t, int64_t, int64_t) { return 256; }

int sk_resident_fwd(const SkFwdArgs& a, void* ws, cudaStream_t st) {
    if ((reinterpret_cast<uintptr_t>(a.X) & 15u) != 0) return sk_stream_fwd(a, ws, st);
    cudaMemsetAsync(a.status, 0, sizeof(int32_t) * 4, st);
    int rc;
    switch (pick(a.n, a.m)) {
        case RKind::S: rc = launch_fwd<CfgS>(a, st); break;
        case RKind::M: rc = launch_fwd<CfgM>(a, st); break;
        case RKind::L: rc = launch_fwd<CfgL>(a, st); break;
        default: return fail(DOT_ERR_UNSUPPORTED, "resident solver: shape not supported");
    }
    if (rc) return rc;
    skr_status_kernel<<<1, 32, 0, st>>>(a.status, a.n_iters);
    return check_launch("sinkhorn status");
}

int sk_resident_bwd(const SkBwdArgs& a, void* ws, cudaStream_t st) {
    if ((reinterpret_cast<uintptr_t>(a.P) & 15u) != 0) return sk_stream_bwd(a, ws, st);
    int32_t* err = static_cast<int32_t*>(ws);
    cudaMemsetAsync(err, 0, sizeof(int32_t), st);
    switch (pick(a.n, a.m)) {
        case RKind::S: return launch_bwd<CfgS>(a, err, st);
        case RKind::M: return launch_bwd<CfgM>(a, err, st);
        case RKind::L: return launch_bwd<CfgL>(a, err, st);
        default: return fail(DOT_ERR_UNSUPPORTED, "resident solver: shape not supported");
    }
}

}  // namespace dotb

// Cluster-resident Sinkhorn solvers for mid-size problems: one thread-block
// cluster of CL CTAs per problem, the problem's rows spread over the CTAs'
// shared memory (CTA r holds rows [r*rpc, (r+1)*rpc)), every iteration on
// chip.  HBM is read once per call (the cost, or the plan in the backward)
// instead of once per iteration; what remains per iteration is the
// exponential unit (forward) and one exchange of column partials inside the
// cluster.
//
// Forward iteration (the reference's Gauss-Seidel order,
// src/sinkhorn/torch_cuda.cpp:200-223; row/column updates kernels.cu:503-545,
// 629-671):
//   row pass   every warp takes rows of its CTA: t = K + v (K = X * kinv,
//              converted once in shared memory), u_i = la_i - LSE_j t (max,
//              then the sum of exp(t - max)), and the column sums
//              S_j += E_ij * exp(a_i - A) with E_ij = exp(t_ij - max_i),
//              a_i = max_i + u_i, A a warp-wide reference (one exponential per
//              element, as in the streaming kernels);
//   CTA merge  per column over the warps: the CTA's pair (A* - v_j, S*_j);
//   exchange   column j belongs to CTA j / cpo of the cluster: every CTA
//              stores its pair into the owner's shared memory with st.async
//              (the bytes complete a transaction on the owner's mbarrier); the
//              owner merges the CL pairs in CTA order (max, then the rescaled
//              sums), writes v_j = lb_j - LSE and stores v_j into every CTA of
//              the cluster the same way; a column whose merged sum is too
//              small to trust is recomputed exactly (max-based LSE over all n
//              rows, read from the CTAs' tiles through distributed shared
//              memory).
// Backward: the plan tile stays resident and the Gauss-Seidel adjoint sweeps
// (kernels.cu:965-1098) run on it, with the same exchange for the column
// sums of P * lambda.
//
// Every mbarrier wait is bounded; a CTA whose wait expires records 0x100 in
// the error word, stops waiting and leaves the loop with the rest of its CTA
// at the next CTA barrier; every CTA arrives at the final cluster barrier.
#include <cmath>

#include "cluster.cuh"
#include "common.cuh"
#include "internal.h"
#include "pack.cuh"
#include "sinkhorn.h"
#include "tma.cuh"

namespace dotb {

namespace {

constexpr float kRaiseC = 60.0f;
constexpr float kTinyC = 8.077935669463161e-28f;   // 2^-90

template <int CL_, int VPL_, int W_>
struct CCfg {
    static constexpr int CL = CL_;            // CTAs per cluster, one problem per cluster
    static constexpr int VPL = VPL_;          // float4 per lane per row (a warp covers 128 * VPL columns)
    static constexpr int W = W_;              // warps per CTA
    static constexpr int NC = 4 * VPL;        // columns per lane
    static constexpr int NP = NC / 2;         // float2 pairs per lane
    static constexpr int CW = 128 * VPL;      // columns covered (>= m)
    static constexpr int T = 32 * W;
    static constexpr int MINB = T <= 256 ? 2 : 1;   // CTAs per SM the launch bounds target
};

// Shared-memory carve (dynamic part): tile [rpc*m] | part [W*CW] | v [CW] |
// u [rpc] | in [CL*cpo] float2 | cinv [cpo] float2 | rinv [rpc] float2 |
// red [CL] | aw [W].  tile, part and v are 16-byte aligned.
template <class C>
struct CSmem {
    float* tile;
    float* part;
    float* v;
    float* u;
    float2* in;
    float2* cinv;
    float2* rinv;
    float* red;
    float* aw;
    static size_t bytes(int rpc, int64_t m, int cpo) {
        size_t b = size_t(rpc) * size_t(m) * 4;
        b += size_t(C::W) * C::CW * 4 + size_t(C::CW) * 4;
        b += (size_t(rpc) * 4 + 7) & ~size_t(7);
        b += size_t(C::CL) * cpo * 8 + size_t(cpo) * 8 + size_t(rpc) * 8;
        b += size_t(C::CL) * 4 + size_t(C::W) * 4;
        return (b + 127) & ~size_t(127);
    }
    __device__ static CSmem carve(unsigned char* base, int rpc, int64_t m, int cpo) {
        CSmem s;
        float* f = reinterpret_cast<float*>(base);
        s.tile = f;
        f += int64_t(rpc) * m;
        s.part = f;
        f += C::W * C::CW;
        s.v = f;
        f += C::CW;
        s.u = f;
        f += (rpc + 1) & ~1;
        s.in = reinterpret_cast<float2*>(f);
        s.cinv = s.in + C::CL * cpo;
        s.rinv = s.cinv + cpo;
        s.red = reinterpret_cast<float*>(s.rinv + rpc);
        s.aw = s.red + C::CL;
        return s;
    }
};

struct ClusterGeom {
    int rpc;   // rows per CTA
    int cpo;   // columns owned per CTA (exchange)
};

// Exact column (max, sum) over all n rows of the cluster's problem, read from
// every CTA's tile and u through distributed shared memory; one thread.
template <class C>
__device__ float2 exact_pair_dsmem(const CSmem<C>& S, int64_t n, int64_t m, int rpc, int64_t j) {
    float mx = kNegBig;
    for (int64_t i = 0; i < n; ++i) {
        const uint32_t r = uint32_t(i / rpc);
        const int64_t lr = i - int64_t(r) * rpc;
        const float k = ld_cluster_f32(cluster_map(S.tile + lr * m + j, r));
        const float uu = ld_cluster_f32(cluster_map(S.u + lr, r));
        mx = fmaxf(mx, __fadd_rn(k, uu));
    }
    float sm = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        const uint32_t r = uint32_t(i / rpc);
        const int64_t lr = i - int64_t(r) * rpc;
        const float k = ld_cluster_f32(cluster_map(S.tile + lr * m + j, r));
        const float uu = ld_cluster_f32(cluster_map(S.u + lr, r));
        sm += exp_shift(__fadd_rn(k, uu) - mx);
    }
    return make_float2(mx, sm);
}

// Per-warp column partials (group lanes hold different rows of the same
// columns only when several rows share a warp; here a warp is one row) into
// the CTA merge buffer.
template <class C>
__device__ __forceinline__ void store_part(const CSmem<C>& S, int wid, int lane, const float2 (&cs)[C::NP]) {
#pragma unroll
    for (int p = 0; p < C::VPL; ++p)
        *reinterpret_cast<float4*>(S.part + wid * C::CW + 4 * lane + 128 * p) =
            make_float4(cs[2 * p].x, cs[2 * p].y, cs[2 * p + 1].x, cs[2 * p + 1].y);
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
template <class C>
__global__ void __launch_bounds__(C::T, C::MINB) skc_fwd_kernel(SkFwdArgs a, ClusterGeom geo) {
    constexpr int W = C::W, VPL = C::VPL, NP = C::NP, CL = C::CL, T = C::T;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bar_tile, bar_in, bar_v;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int rpc = geo.rpc, cpo = geo.cpo;
    const uint32_t rank = cl_rank();
    const int64_t b = cl_id();
    const int64_t n = a.n, m = a.m;
    const int64_t r0 = int64_t(rank) * rpc;
    const int nr = int(max(int64_t(0), min(int64_t(rpc), n - r0)));
    const int64_t o0 = int64_t(rank) * cpo;
    const int owned = int(max(int64_t(0), min(int64_t(cpo), m - o0)));
    const CSmem<C> S = CSmem<C>::carve(smem, rpc, m, cpo);
    int32_t* err = a.status + 3;
    auto live = [&](int p) -> bool { return 4 * lane + 128 * p < m; };

    if (tid == 0) {
        mbar_init(&bar_tile, 1);
        mbar_init(&bar_in, 1);
        mbar_init(&bar_v, 1);
        mbar_fence_init();
    }
    for (int j = tid; j < C::CW; j += T) S.v[j] = 0.0f;
    __syncthreads();
    if (tid == 0) {
        if (nr > 0) {
            const uint32_t bytes = uint32_t(nr) * uint32_t(m) * 4u;
            mbar_arrive_expect_tx(&bar_tile, bytes);
            bulk_g2s(S.tile, a.X + (b * n + r0) * m, bytes, &bar_tile);
        }
        if (a.n_iters > 0) {
            mbar_arrive_expect_tx(&bar_in, uint32_t(CL * owned * 8));
            mbar_arrive_expect_tx(&bar_v, uint32_t(m * 4));
        }
    }
    bool failed = false;
    if (nr > 0) failed = !mbar_wait_sleep(&bar_tile, 0, err);
    failed = __syncthreads_or(failed) != 0;
    if (!failed) {   // the tile holds K = X * kinv from here on (rounded once, as the reference's log_K)
        const float2 k2 = splat2(a.kinv);
        float4* t4 = reinterpret_cast<float4*>(S.tile);
        for (int q = tid; q < (nr * int(m)) >> 2; q += T) {
            const float4 x = t4[q];
            const float2 lo = mul2(make_float2(x.x, x.y), k2), hi = mul2(make_float2(x.z, x.w), k2);
            t4[q] = make_float4(lo.x, lo.y, hi.x, hi.y);
        }
    }
    // every CTA's barriers are armed and its tile converted before any
    // exchange or distributed read
    cl_sync();

    const float* la = a.la ? a.la + b * n + r0 : nullptr;
    const float* lb = a.lb ? a.lb + b * m : nullptr;
    const int nslots = (nr + W - 1) / W;
    for (int it = 0; it < a.n_iters; ++it) {
        const uint32_t par = uint32_t(it & 1);
        float2 vr[NP], cs[NP];
#pragma unroll
        for (int p = 0; p < VPL; ++p) {
            const float4 v4 = *reinterpret_cast<const float4*>(S.v + 4 * lane + 128 * p);
            vr[2 * p] = make_float2(v4.x, v4.y);
            vr[2 * p + 1] = make_float2(v4.z, v4.w);
        }
#pragma unroll
        for (int k = 0; k < NP; ++k) cs[k] = make_float2(0.0f, 0.0f);
        float A = kNegBig;
        for (int sl = 0; sl < nslots; ++sl) {
            const int lr = sl * W + wid;
            if (lr >= nr) break;   // warp-uniform
            float2 t[NP];
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                if (live(p)) {
                    const float4 k4 = *reinterpret_cast<const float4*>(S.tile + int64_t(lr) * m + 4 * lane + 128 * p);
                    t[2 * p] = add2(make_float2(k4.x, k4.y), vr[2 * p]);
                    t[2 * p + 1] = add2(make_float2(k4.z, k4.w), vr[2 * p + 1]);
                } else {
                    t[2 * p] = t[2 * p + 1] = make_float2(-INFINITY, -INFINITY);
                }
            }
            const float mx = warp_max<32>(max_of(t));
            // exp(t - mx) as 2^(t*log2e - mL) in one FFMA, mL = mx*log2e
            // rounded; every term carries 2^cr, cr = mx*log2e - mL exactly
            // (FMA remainder), taken out of the row LSE and the column weight
            const float mxc = fmaxf(mx, -1.0e37f);
            const float mL = mxc * kLog2e;
            const float cr = fmaf(mxc, kLog2e, -mL);
            const float2 l2 = splat2(kLog2e), nm = splat2(-mL);
#pragma unroll
            for (int k = 0; k < NP; ++k) {
                const float2 e = fma2(t[k], l2, nm);
                t[k] = make_float2(ex2(e.x), ex2(e.y));
            }
            const float2 s2 = tree_sum2(t);
            const float s = warp_sum<32>(s2.x + s2.y);
            const float unew = (la ? __ldg(la + lr) : a.la_def) - (mx + (fast_log(fmaxf(s, kSumFloor)) - cr * kLn2));
            if (lane == 0) S.u[lr] = unew;
            const float ai = mx + unew;
            if (ai > A + kRaiseC) {   // warp-uniform
                const float2 sc = splat2(exp_shift(A - ai));
#pragma unroll
                for (int k = 0; k < NP; ++k) cs[k] = mul2(cs[k], sc);
                A = ai;
            }
            const float2 w = splat2(ex2(fmaf(ai - A, kLog2e, -cr)));   // exp(ai - A) / 2^cr
#pragma unroll
            for (int k = 0; k < NP; ++k) cs[k] = fma2(t[k], w, cs[k]);
        }
        store_part<C>(S, wid, lane, cs);
        if (lane == 0) S.aw[wid] = A;
        if (__syncthreads_or(failed)) break;

        // CTA merge over the warps (fixed order), then the pair to the column's owner
        {
            const float awl = lane < W ? S.aw[lane] : kNegBig;
            const float amax = warp_max<32>(awl);
            const float scl = lane < W ? exp_shift(awl - amax) : 0.0f;
            float scw[W];
#pragma unroll
            for (int w = 0; w < W; ++w) scw[w] = __shfl_sync(0xffffffffu, scl, w);
            for (int j = tid; j < m; j += T) {
                float sj = 0.0f;
#pragma unroll
                for (int w = 0; w < W; ++w) sj = fmaf(S.part[w * C::CW + j], scw[w], sj);
                const uint32_t o = uint32_t(j / cpo);
                const int jl = j - int(o) * cpo;
                st_async_f2(cluster_map(S.in + int(rank) * cpo + jl, o), cluster_map(&bar_in, o),
                            make_float2(amax - S.v[j], sj));
            }
        }
        // owner: merge the CL pairs of each owned column, broadcast v
        if (!failed && !mbar_wait_cluster(&bar_in, par, err)) failed = true;
        if (tid == 0 && it + 1 < a.n_iters) mbar_arrive_expect_tx(&bar_in, uint32_t(CL * owned * 8));
        for (int jl = tid; jl < owned; jl += T) {
            float2 q[CL];
            float mm = kNegBig;
#pragma unroll
            for (int r = 0; r < CL; ++r) {
                q[r] = S.in[r * cpo + jl];
                mm = fmaxf(mm, q[r].x);
            }
            float ss = 0.0f;
#pragma unroll
            for (int r = 0; r < CL; ++r) ss = fmaf(q[r].y, exp_shift(q[r].x - mm), ss);
            const int64_t j = o0 + jl;
            if (ss < kTinyC) {
                const float2 e = exact_pair_dsmem<C>(S, n, m, rpc, j);
                mm = e.x;
                ss = e.y;
            }
            const float vj = (lb ? __ldg(lb + j) : a.lb_def) - lse_finish(mm, ss);
#pragma unroll
            for (int r = 0; r < CL; ++r) st_async_f32(cluster_map(S.v + j, uint32_t(r)), cluster_map(&bar_v, uint32_t(r)), vj);
        }
        if (!failed && !mbar_wait_cluster(&bar_v, par, err)) failed = true;
        if (tid == 0 && it + 1 < a.n_iters) mbar_arrive_expect_tx(&bar_v, uint32_t(m * 4));
    }

    // epilogue: potentials, plan (P = safe_exp((K + u_i) + v_j)) and cost
    __syncthreads();
    if (a.n_iters == 0)
        for (int lr = tid; lr < nr; lr += T) S.u[lr] = 0.0f;
    __syncthreads();
    for (int lr = tid; lr < nr; lr += T) a.u2[b * n + r0 + lr] = S.u[lr];
    if (rank == 0)
        for (int j = tid; j < m; j += T) a.v2[b * m + j] = S.v[j];
    float acc = 0.0f;
    float* outb = a.out + (b * n + r0) * m;
    const float4* xg = reinterpret_cast<const float4*>(a.X + (b * n + r0) * m);
    const int m4 = int(m >> 2);
    for (int q = tid; q < nr * m4; q += T) {
        const int lr = q / m4, j = (q - lr * m4) * 4;
        const float4 k4 = *reinterpret_cast<const float4*>(S.tile + int64_t(lr) * m + j);
        const float uu = S.u[lr];
        const float4 v4 = *reinterpret_cast<const float4*>(S.v + j);
        const float t0 = __fadd_rn(__fadd_rn(k4.x, uu), v4.x);
        const float t1 = __fadd_rn(__fadd_rn(k4.y, uu), v4.y);
        const float t2 = __fadd_rn(__fadd_rn(k4.z, uu), v4.z);
        const float t3 = __fadd_rn(__fadd_rn(k4.w, uu), v4.w);
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
        __syncthreads();
        if (lane == 0) S.part[wid] = acc;
        __syncthreads();
        if (tid == 0) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < W; ++w) tot += S.part[w];
            st_cluster_f32(cluster_map(S.red + rank, 0), tot);
        }
    }
    cl_sync();   // no CTA leaves while another may still read or store its shared memory
    if (a.cost != nullptr && rank == 0 && tid == 0) {
        float tot = 0.0f;
        for (int r = 0; r < CL; ++r) tot += S.red[r];
        a.cost[b] = tot;
    }
}

// ---------------------------------------------------------------------------
// backward (implicit adjoint on the resident plan tile)
// ---------------------------------------------------------------------------
template <class C>
__global__ void __launch_bounds__(C::T, C::MINB) skc_bwd_kernel(SkBwdArgs a, ClusterGeom geo, int32_t* err) {
    constexpr int W = C::W, VPL = C::VPL, NP = C::NP, CL = C::CL, T = C::T;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bar_tile, bar_in, bar_v;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int rpc = geo.rpc, cpo = geo.cpo;
    const uint32_t rank = cl_rank();
    const int64_t b = cl_id();
    const int64_t n = a.n, m = a.m;
    const int64_t r0 = int64_t(rank) * rpc;
    const int nr = int(max(int64_t(0), min(int64_t(rpc), n - r0)));
    const int64_t o0 = int64_t(rank) * cpo;
    const int owned = int(max(int64_t(0), min(int64_t(cpo), m - o0)));
    const CSmem<C> S = CSmem<C>::carve(smem, rpc, m, cpo);
    float* lam = S.u;
    float* mu = S.v;
    auto live = [&](int p) -> bool { return 4 * lane + 128 * p < m; };
    const float gc = a.gcost ? __ldg(a.gcost + b) : 0.0f;
    const float* Xr = a.X + (b * n + r0) * m;
    const float* gPr = a.gP ? a.gP + (b * n + r0) * m : nullptr;
    auto G_at = [&](int64_t idx) -> float {   // G = grad_cost_b * X + grad_P (autograd's rounding)
        float g = __fmul_rn(gc, __ldg(Xr + idx));
        if (gPr) g = __fadd_rn(g, __ldg(gPr + idx));
        return g;
    };

    if (tid == 0) {
        mbar_init(&bar_tile, 1);
        mbar_init(&bar_in, 1);
        mbar_init(&bar_v, 1);
        mbar_fence_init();
    }
    for (int j = tid; j < C::CW; j += T) mu[j] = 0.0f;
    __syncthreads();
    if (tid == 0) {
        if (nr > 0) {
            const uint32_t bytes = uint32_t(nr) * uint32_t(m) * 4u;
            mbar_arrive_expect_tx(&bar_tile, bytes);
            bulk_g2s(S.tile, a.P + (b * n + r0) * m, bytes, &bar_tile);
        }
        mbar_arrive_expect_tx(&bar_in, uint32_t(CL * owned * 8));   // phase 0: column invariants
        if (a.bwd_iters > 0) mbar_arrive_expect_tx(&bar_v, uint32_t(m * 4));
    }
    cl_sync();
    bool failed = false;
    if (nr > 0) failed = !mbar_wait_sleep(&bar_tile, 0, err);
    failed = __syncthreads_or(failed) != 0;

    // ---- invariants: rows (sum_k P G, sum_k P) kept in rinv; columns
    // (sum_i P G, sum_i P) summed per CTA, then by the owners in CTA order
    {
        float2 cpg[NP], cp[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) cpg[k] = cp[k] = make_float2(0.0f, 0.0f);
        for (int lr = wid; lr < nr && !failed; lr += W) {
            float spg = 0.0f, sp = 0.0f;
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                if (!live(p)) continue;
                const int64_t e0 = int64_t(lr) * m + 4 * lane + 128 * p;
                const float4 p4 = *reinterpret_cast<const float4*>(S.tile + e0);
                const float pv[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float gv = G_at(e0 + e);
                    spg += pv[e] * gv;
                    sp += pv[e];
                    float2& a2 = cpg[2 * p + e / 2];
                    float2& b2 = cp[2 * p + e / 2];
                    if (e & 1) {
                        a2.y += pv[e] * gv;
                        b2.y += pv[e];
                    } else {
                        a2.x += pv[e] * gv;
                        b2.x += pv[e];
                    }
                }
            }
            spg = warp_sum<32>(spg);
            sp = warp_sum<32>(sp);
            if (lane == 0) S.rinv[lr] = make_float2(spg, sp);
        }
        // per-warp column partials through the merge buffer, two rounds
        store_part<C>(S, wid, lane, cpg);
        __syncthreads();
        constexpr int CPT = (C::CW + T - 1) / T;   // columns per thread
        float colpg[CPT];
#pragma unroll
        for (int q = 0; q < CPT; ++q) {
            const int j = tid + q * T;
            float s = 0.0f;
            if (j < m) {
#pragma unroll
                for (int w = 0; w < W; ++w) s += S.part[w * C::CW + j];
            }
            colpg[q] = s;
        }
        __syncthreads();
        store_part<C>(S, wid, lane, cp);
        __syncthreads();
#pragma unroll
        for (int q = 0; q < CPT; ++q) {
            const int j = tid + q * T;
            if (j >= m) break;
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < W; ++w) s += S.part[w * C::CW + j];
            const uint32_t o = uint32_t(j / cpo);
            const int jl = j - int(o) * cpo;
            st_async_f2(cluster_map(S.in + int(rank) * cpo + jl, o), cluster_map(&bar_in, o),
                        make_float2(colpg[q], s));
        }
        if (!failed && !mbar_wait_cluster(&bar_in, 0, err)) failed = true;
        if (tid == 0 && a.bwd_iters > 0) mbar_arrive_expect_tx(&bar_in, uint32_t(CL * owned * 8));
        for (int jl = tid; jl < owned; jl += T) {
            float pg = 0.0f, pp = 0.0f;
#pragma unroll
            for (int r = 0; r < CL; ++r) {
                const float2 q = S.in[r * cpo + jl];
                pg += q.x;
                pp += q.y;
            }
            S.cinv[jl] = make_float2(pg, fmaxf(pp, kSumFloor));
        }
    }
    __syncthreads();   // rinv / cinv visible; the merge buffer is free

    // ---- Gauss-Seidel sweeps
    for (int it = 0; it < a.bwd_iters; ++it) {
        const uint32_t pin = uint32_t((it + 1) & 1), pv = uint32_t(it & 1);
        float2 mr[NP], acc[NP];
#pragma unroll
        for (int p = 0; p < VPL; ++p) {
            const float4 u4 = *reinterpret_cast<const float4*>(mu + 4 * lane + 128 * p);
            mr[2 * p] = make_float2(u4.x, u4.y);
            mr[2 * p + 1] = make_float2(u4.z, u4.w);
        }
#pragma unroll
        for (int k = 0; k < NP; ++k) acc[k] = make_float2(0.0f, 0.0f);
        for (int lr = wid; lr < nr; lr += W) {
            float2 p2[NP];
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                if (live(p)) {
                    const float4 x = *reinterpret_cast<const float4*>(S.tile + int64_t(lr) * m + 4 * lane + 128 * p);
                    p2[2 * p] = make_float2(x.x, x.y);
                    p2[2 * p + 1] = make_float2(x.z, x.w);
                } else {
                    p2[2 * p] = p2[2 * p + 1] = make_float2(0.0f, 0.0f);
                }
            }
            float2 dq[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};   // four independent chains
#pragma unroll
            for (int k = 0; k < NP; ++k) dq[k & 1] = fma2(p2[k], mr[k], dq[k & 1]);
            const float2 d2 = add2(dq[0], dq[1]);
            const float s = warp_sum<32>(d2.x + d2.y);
            const float2 ri = S.rinv[lr];
            const float l = (ri.x - s) / fmaxf(ri.y, kSumFloor);
            if (lane == 0) lam[lr] = l;
            const float2 l2 = splat2(l);
#pragma unroll
            for (int k = 0; k < NP; ++k) acc[k] = fma2(p2[k], l2, acc[k]);
        }
        store_part<C>(S, wid, lane, acc);
        if (__syncthreads_or(failed)) break;
        for (int j = tid; j < m; j += T) {
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < W; ++w) s += S.part[w * C::CW + j];
            const uint32_t o = uint32_t(j / cpo);
            const int jl = j - int(o) * cpo;
            st_async_f2(cluster_map(S.in + int(rank) * cpo + jl, o), cluster_map(&bar_in, o), make_float2(s, 0.0f));
        }
        if (!failed && !mbar_wait_cluster(&bar_in, pin, err)) failed = true;
        if (tid == 0 && it + 1 < a.bwd_iters) mbar_arrive_expect_tx(&bar_in, uint32_t(CL * owned * 8));
        for (int jl = tid; jl < owned; jl += T) {
            float s = 0.0f;
#pragma unroll
            for (int r = 0; r < CL; ++r) s += S.in[r * cpo + jl].x;
            const float2 ci = S.cinv[jl];
            const float muj = (ci.x - s) / ci.y;
            const int64_t j = o0 + jl;
#pragma unroll
            for (int r = 0; r < CL; ++r) st_async_f32(cluster_map(mu + j, uint32_t(r)), cluster_map(&bar_v, uint32_t(r)), muj);
        }
        if (!failed && !mbar_wait_cluster(&bar_v, pv, err)) failed = true;
        if (tid == 0 && it + 1 < a.bwd_iters) mbar_arrive_expect_tx(&bar_v, uint32_t(m * 4));
    }
    __syncthreads();
    if (a.bwd_iters == 0)
        for (int lr = tid; lr < nr; lr += T) lam[lr] = 0.0f;
    __syncthreads();

    // ---- gradient epilogue for this CTA's rows
    float accT = 0.0f;
    float* gXr = a.gX + (b * n + r0) * m;
    for (int64_t idx = tid; idx < int64_t(nr) * m; idx += T) {
        const int64_t lr = idx / m, j = idx - lr * m;
        const float x = __ldg(Xr + idx);
        const float p = S.tile[idx];
        const float centred = G_at(idx) - lam[lr] - mu[j];
        const float g = p * centred / a.tau;
        gXr[idx] = __fadd_rn(a.sign * g, __fmul_rn(gc, p));
        accT += g * (a.sign * x);
    }
    if (a.gtau != nullptr) {
        accT = warp_sum<32>(accT);
        if (lane == 0) S.part[wid] = accT;
        __syncthreads();
        if (tid == 0) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < W; ++w) tot += S.part[w];
            st_cluster_f32(cluster_map(S.red + rank, 0), tot);
        }
    }
    cl_sync();
    if (a.gtau != nullptr && rank == 0 && tid == 0) {
        float tot = 0.0f;
        for (int r = 0; r < CL; ++r) tot += S.red[r];
        a.gtau[b] = tot * (-1.0f / a.tau);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// One 8-CTA cluster per problem, 16 warps per CTA, one CTA per SM: rows of up
// to 1024 columns, the tile at most kTileBudget bytes per CTA.
constexpr int kCL = 8;
constexpr int kW = 16;
constexpr size_t kTileBudget = 168 * 1024;

template <int VPL>
using CfgV = CCfg<kCL, VPL, kW>;

int vpl_of(int64_t m) { return m <= 256 ? 2 : m <= 512 ? 4 : 8; }

ClusterGeom geom_of(int64_t n, int64_t m) {
    ClusterGeom g;
    g.rpc = int((n + kCL - 1) / kCL);
    g.cpo = int((m + kCL - 1) / kCL);
    return g;
}

template <int VPL>
size_t smem_bytes(const ClusterGeom& g, int64_t m) { return CSmem<CfgV<VPL>>::bytes(g.rpc, m, g.cpo); }

size_t smem_of(const ClusterGeom& g, int64_t m) {
    switch (vpl_of(m)) {
        case 2: return smem_bytes<2>(g, m);
        case 4: return smem_bytes<4>(g, m);
        default: return smem_bytes<8>(g, m);
    }
}

template <class C>
cudaLaunchConfig_t cluster_config(int64_t B, size_t sm, cudaStream_t st, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(B * C::CL));
    cfg.blockDim = dim3(C::T);
    cfg.dynamicSmemBytes = sm;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C::CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

// Clusters of this kernel with `sm` bytes of dynamic shared memory the
// device holds at once (0: none fits), cached per device, kernel and size;
// sets the kernel's shared-memory attribute as a side effect.
template <class C, int WHICH, typename K>
int resident_clusters(K kernel, size_t sm) {
    constexpr int kMaxDev = 64;
    static size_t c_sm[kMaxDev] = {};   // one cache per configuration and direction
    static int c_ncl[kMaxDev] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < kMaxDev && c_sm[dev] == sm) return c_ncl[dev];
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
    if (C::CL > 8) cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cluster_config<C>(1, sm, nullptr, attr);
    int ncl = 0;
    if (cudaOccupancyMaxActiveClusters(&ncl, kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();
        ncl = 0;
    }
    if (dev >= 0 && dev < kMaxDev) {
        c_sm[dev] = sm;
        c_ncl[dev] = ncl;
    }
    return ncl;
}
template <class C, int WHICH, typename K>
bool can_launch(K kernel, size_t sm) { return resident_clusters<C, WHICH>(kernel, sm) >= 1; }

template <int VPL>
int fwd_v(const SkFwdArgs& a, const ClusterGeom& g, cudaStream_t st) {
    using C = CfgV<VPL>;
    const size_t sm = smem_bytes<VPL>(g, a.m);
    if (!can_launch<C, 0>(skc_fwd_kernel<C>, sm)) return DOT_ERR_UNSUPPORTED;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cluster_config<C>(a.B, sm, st, attr);
    ProfScope ps(DOT_K_SK_RESIDENT, st);
    cudaLaunchKernelEx(&cfg, skc_fwd_kernel<C>, a, g);
    return DOT_OK;
}

template <int VPL>
int bwd_v(const SkBwdArgs& a, const ClusterGeom& g, int32_t* err, cudaStream_t st) {
    using C = CfgV<VPL>;
    const size_t sm = smem_bytes<VPL>(g, a.m);
    if (!can_launch<C, 1>(skc_bwd_kernel<C>, sm)) return DOT_ERR_UNSUPPORTED;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cluster_config<C>(a.B, sm, st, attr);
    ProfScope ps(DOT_K_SK_RESIDENT, st);
    cudaLaunchKernelEx(&cfg, skc_bwd_kernel<C>, a, g, err);
    return DOT_OK;
}

__global__ void skc_status_kernel(int32_t* status, int n_iters) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        status[0] = n_iters;
        status[1] = 0;
    }
}

}  // namespace

int sk_cluster_capacity(int64_t n, int64_t m) {
    const ClusterGeom g = geom_of(n, m);
    switch (vpl_of(m)) {
        case 2: return resident_clusters<CfgV<2>, 0>(skc_fwd_kernel<CfgV<2>>, smem_bytes<2>(g, m));
        case 4: return resident_clusters<CfgV<4>, 0>(skc_fwd_kernel<CfgV<4>>, smem_bytes<4>(g, m));
        default: return resident_clusters<CfgV<8>, 0>(skc_fwd_kernel<CfgV<8>>, smem_bytes<8>(g, m));
    }
}

bool sk_cluster_supported(int64_t B, int64_t n, int64_t m, const void* data) {
    if (B < 1 || n < 1 || m < 4 || m > 1024 || (m % 4) != 0) return false;
    if ((reinterpret_cast<uintptr_t>(data) & 15u) != 0) return false;
    if (B * kCL > int64_t(0x7fffffff)) return false;
    const ClusterGeom g = geom_of(n, m);
    if (size_t(g.rpc) * size_t(m) * 4 > kTileBudget) return false;
    return smem_of(g, m) <= 227 * 1024 - 64;
}

constexpr int64_t kClusterWaves = 8;

bool sk_cluster_preferred(int64_t B, int64_t n, int64_t m, const void* data) {
    return sk_cluster_supported(B, n, m, data) && B <= kClusterWaves * int64_t(sk_cluster_capacity(n, m));
}

int sk_cluster_fwd(const SkFwdArgs& a, cudaStream_t st) {
    const ClusterGeom g = geom_of(a.n, a.m);
    cudaMemsetAsync(a.status, 0, sizeof(int32_t) * 4, st);   // the fall-back path clears it again
    int rc;
    switch (vpl_of(a.m)) {
        case 2: rc = fwd_v<2>(a, g, st); break;
        case 4: rc = fwd_v<4>(a, g, st); break;
        default: rc = fwd_v<8>(a, g, st); break;
    }
    if (rc != DOT_OK) return rc;
    skc_status_kernel<<<1, 32, 0, st>>>(a.status, a.n_iters);
    return check_launch("sinkhorn forward (cluster-resident)");
}

int sk_cluster_bwd(const SkBwdArgs& a, int32_t* err, cudaStream_t st) {
    const ClusterGeom g = geom_of(a.n, a.m);
    cudaMemsetAsync(err, 0, sizeof(int32_t), st);
    int rc;
    switch (vpl_of(a.m)) {
        case 2: rc = bwd_v<2>(a, g, err, st); break;
        case 4: rc = bwd_v<4>(a, g, err, st); break;
        default: rc = bwd_v<8>(a, g, err, st); break;
    }
    if (rc != DOT_OK) return rc;
    return check_launch("sinkhorn backward (cluster-resident)");
}

}  // namespace dotb

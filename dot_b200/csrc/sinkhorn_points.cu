// Sinkhorn on point clouds: the cost C_bij = scale * |x_bi - y_bj|^2 is built
// inside the iterations from x [B,n,d] and y [B,m,d] instead of being read
// from a materialised B x n x m matrix.  For low-dimensional clouds (d <= 4;
// the squared-distance costs of the reference's usage, e.g. 32768 points in
// 3-D) an iteration then moves no matrix bytes at all, and its bound is the
// exponential unit instead of HBM.
//
// A Sinkhorn half-step on points is symmetric in the two sides,
//     u_i = la_i - LSE_j(K_ij + v_j)      (rows: side a = x, side b = y)
//     v_j = lb_j - LSE_i(K_ij + u_i)      (columns: side a = y, side b = x)
// with K_ij = -C_ij / tau, so one kernel serves both (skp_half_kernel): a lane
// owns one point of side a (its coordinates and running (max, sum) in
// registers) and sweeps a chunk of side b's points, which every lane of the
// warp reads at once (one broadcast load of a packed point and one of its
// potential per 32 elements).  Per element: the distance (packed f32x2 on
// column pairs), K + w, an online max (the sum is rescaled only when a lane's
// maximum grows, warp-uniform branch) and one ex2.  Chunks of side b spread
// the work over the grid; skp_merge_kernel merges each point's chunk partials
// in chunk order and writes the potential.  Each half-step reads the other
// side's potentials as they are, so the iteration keeps the reference's
// Gauss-Seidel order (src/sinkhorn/torch_cuda.cpp:200-223).
//
// The plan / cost epilogue (skp_plan_kernel) builds the entries the same way.
// Shapes the point kernels do not take (d > 4, tol > 0) materialise C once
// with the same arithmetic (dot_sq_dist) and run the matrix solvers.  The
// reference builds such costs in Python (torch.cdist(x, y) ** 2) and hands the
// matrix to sinkhorn(); this path has no counterpart there.
#include <algorithm>
#include <cmath>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "pack.cuh"
#include "sinkhorn.h"

namespace dotb {
namespace {

constexpr int kPRows = 8;   // rows per CTA (one warp per row)

// C[row, j] for one row per warp, lanes over the columns.
__global__ void __launch_bounds__(kPRows * 32)
skp_sqdist_kernel(const float* __restrict__ x, const float* __restrict__ y, int64_t rows, int64_t n, int64_t m,
                  int d, float scale, float* __restrict__ C) {
    const int lane = threadIdx.x & 31;
    const int64_t row = int64_t(blockIdx.x) * kPRows + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float* xr = x + row * d;
    const float* yb = y + (row / n) * m * d;
    float* cr = C + row * m;
    for (int64_t j = lane; j < m; j += 32) cr[j] = sq_dist_n(xr, yb + j * d, d, scale);
}

// Side-b operand of skp_half_kernel: the points of one side in column-pair
// records, so that each packed f32x2 operand arrives in adjacent registers of
// one 16-byte load.  Record of pair (j, j+1), 2 (d + 1) floats padded to a
// multiple of 4: {-p_0(j), -p_0(j+1), ..., -p_{d-1}(j), -p_{d-1}(j+1),
// w(j), w(j+1)} with w the side's potential (x + (-y) is the rounded x - y).
// Points are padded to a multiple of kHU with p = 0, w = -inf (their terms
// are exactly 0), so the sweep needs no bounds checks.
constexpr int kHW = 4;              // warps per CTA
constexpr int kHRows = 32 * kHW;    // side-a points per CTA (one per lane)
constexpr int kHU = 16;             // side-b padding and chunk granularity (a multiple of every step)

__host__ __device__ constexpr int rec_f4(int d) { return (2 * (d + 1) + 3) / 4; }   // float4 per record
__host__ __device__ inline int64_t padded_points(int64_t nb) { return (nb + kHU - 1) / kHU * kHU; }

// One thread per pair of points; w = 0 for real points.
__global__ void skp_pack_kernel(const float* __restrict__ p, int64_t B, int64_t np, int d,
                                float* __restrict__ rec) {
    const int64_t npair = padded_points(np) / 2;
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= B * npair) return;
    const int64_t b = idx / npair, pr = idx - b * npair;
    const int nf = 4 * rec_f4(d);
    float* r = rec + idx * nf;
    for (int h = 0; h < 2; ++h) {
        const int64_t j = 2 * pr + h;
        const bool real = j < np;
        for (int k = 0; k < d; ++k) r[2 * k + h] = real ? -__ldg(p + (b * np + j) * d + k) : 0.0f;
        r[2 * d + h] = real ? 0.0f : -INFINITY;
    }
    for (int f = 2 * (d + 1); f < nf; ++f) r[f] = 0.0f;
}

struct HalfArgs {
    const float* pa;     // [B][na][PD] points of the side being updated
    const float4* rb;    // [B][padded nb / 2][rec_f4(PD)] records of the other side
    int64_t na, nb;
    int64_t ch;          // side-b points per chunk (a multiple of kHU)
    int nchunk;
    float kfold;         // cost_scale * (-1 / tau): K = s * kfold for s = |x - y|^2
    float2* part;        // [B][nchunk][na] (max, sum) partials
};

// One chunk of one half-step: each lane's RL points i of side a against
// side-b points [j0, j1): (max, sum) of t_j = K_ij + w_j, with
//   s = sq_dist's sum of squares (packed, per column pair), t = fma(s, kfold, w)
//   (one rounding; C * kinv with C = s * scale for scale 1 exactly),
//   sum of exp(t - m) as 2^(t log2e - mL), mL = m log2e rounded and the
//   remainder 2^-(m log2e - mL) taken out at the end (as the matrix kernels do).
// The RL points of a lane share every record load and give the warp RL
// independent dependency chains.  Measured on 32768 x 32768 3-D clouds (one
// half-step, ms): 1 point per lane 0.59 (0.55 with the next step's records
// loaded one step ahead), 2 points 0.39, 4 points 0.38 (10 elements per clock
// per SM; steps of 2 or 8 pairs 0.40), 8 points 0.44 (spills) -- kRL = 4,
// kNP = 4.
template <int PD, int RL, int NP>
__global__ void __launch_bounds__(kHW * 32) skp_half_kernel(HalfArgs h, int64_t b0) {
    static_assert(kHU % (2 * NP) == 0, "a step must divide the chunk granularity");
    constexpr int R4 = rec_f4(PD);
    const int64_t b = b0 + blockIdx.z;
    const int64_t i0 = int64_t(blockIdx.x) * (kHRows * RL) + threadIdx.x;   // points i0 + r * kHRows
    const int chunk = int(blockIdx.y);
    const int64_t nbp = padded_points(h.nb);
    const int j0 = int(int64_t(chunk) * h.ch / 2);                     // pair indices
    const int j1 = int(min(nbp, int64_t(chunk) * h.ch + h.ch) / 2);
    float2 xs[RL][PD];
#pragma unroll
    for (int r = 0; r < RL; ++r) {
        const int64_t i = i0 + r * kHRows;
#pragma unroll
        for (int k = 0; k < PD; ++k) xs[r][k] = splat2(i < h.na ? __ldg(h.pa + (b * h.na + i) * PD + k) : 0.0f);
    }
    const float4* rb = h.rb + b * (nbp / 2) * R4;
    const float2 kf = splat2(h.kfold), l2 = splat2(kLog2e);
    float m[RL], mL[RL];
    float2 s2[RL];
#pragma unroll
    for (int r = 0; r < RL; ++r) {
        m[r] = kNegBig;
        mL[r] = fmaxf(m[r], -1.0e37f) * kLog2e;
        s2[r] = make_float2(0.0f, 0.0f);
    }
    auto step = [&](const float4 (&q)[NP][R4]) {
        float2 t[RL][NP];
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            float rv[4 * R4];
#pragma unroll
            for (int c = 0; c < R4; ++c) {
                rv[4 * c + 0] = q[p][c].x;
                rv[4 * c + 1] = q[p][c].y;
                rv[4 * c + 2] = q[p][c].z;
                rv[4 * c + 3] = q[p][c].w;
            }
#pragma unroll
            for (int r = 0; r < RL; ++r) {
                float2 d = add2(xs[r][0], make_float2(rv[0], rv[1]));
                float2 sq = mul2(d, d);
#pragma unroll
                for (int k = 1; k < PD; ++k) {
                    d = add2(xs[r][k], make_float2(rv[2 * k], rv[2 * k + 1]));
                    sq = fma2(d, d, sq);
                }
                t[r][p] = fma2(sq, kf, make_float2(rv[2 * PD], rv[2 * PD + 1]));
            }
        }
        float mx[RL];
        bool grew = false;
#pragma unroll
        for (int r = 0; r < RL; ++r) {
            mx[r] = max_of(t[r]);
            grew = grew || mx[r] > m[r];
        }
        if (__any_sync(0xffffffffu, grew)) {   // some maximum grew: rescale (factor 1 elsewhere)
#pragma unroll
            for (int r = 0; r < RL; ++r) {
                const float mn = fmaxf(m[r], mx[r]);
                const float mLn = fmaxf(mn, -1.0e37f) * kLog2e;
                s2[r] = mul2(s2[r], splat2(ex2(mL[r] - mLn)));
                m[r] = mn;
                mL[r] = mLn;
            }
        }
#pragma unroll
        for (int r = 0; r < RL; ++r) {
            const float2 nm = splat2(-mL[r]);
#pragma unroll
            for (int p = 0; p < NP; ++p) {
                const float2 a = fma2(t[r][p], l2, nm);
                s2[r] = add2(s2[r], make_float2(ex2(a.x), ex2(a.y)));
            }
        }
    };
    auto load = [&](float4 (&q)[NP][R4], int jp) {
#pragma unroll
        for (int p = 0; p < NP; ++p)
#pragma unroll
            for (int c = 0; c < R4; ++c) q[p][c] = __ldg(rb + (jp + p) * R4 + c);
    };
    for (int jp = j0; jp < j1; jp += NP) {
        float4 q[NP][R4];
        load(q, jp);
        step(q);
    }
#pragma unroll
    for (int r = 0; r < RL; ++r) {
        const int64_t i = i0 + r * kHRows;
        if (i < h.na) {
            const float cr = fmaf(fmaxf(m[r], -1.0e37f), kLog2e, -mL[r]);   // exact remainder of the rounded mL
            h.part[(b * h.nchunk + chunk) * h.na + i] = make_float2(m[r], (s2[r].x + s2[r].y) * ex2(-cr));
        }
    }
}

// Potential of every side-a point from its chunk partials, merged in chunk
// order: max pass, then the rescaled sums; pot = l - (max + log(sum)), also
// written into the point's record slot for the next half-step.
__global__ void skp_merge_kernel(const float2* __restrict__ part, int nchunk, int64_t B, int64_t na, int d,
                                 const float* __restrict__ l, float l_def, float* __restrict__ pot,
                                 float* __restrict__ rec_a) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= B * na) return;
    const int64_t b = idx / na, i = idx - b * na;
    const float2* pc = part + b * nchunk * na + i;
    float mm = kNegBig;
    for (int c = 0; c < nchunk; ++c) mm = fmaxf(mm, pc[int64_t(c) * na].x);
    float ss = 0.0f;
    for (int c = 0; c < nchunk; ++c) {
        const float2 q = pc[int64_t(c) * na];
        ss = fmaf(q.y, exp_shift(q.x - mm), ss);
    }
    const float v = (l ? l[idx] : l_def) - lse_finish(mm, ss);
    pot[idx] = v;
    rec_a[((b * (padded_points(na) / 2) + (i >> 1)) * rec_f4(d)) * 4 + 2 * d + (i & 1)] = v;
}

// Row shards: each column's chunk partials over this shard's rows merged
// into one (max, sum) pair (the column half-step's skp_merge_kernel without
// the log), for the cross-shard exchange.
__global__ void skp_pairs_kernel(const float2* __restrict__ part, int nchunk, int64_t B, int64_t m,
                                 float2* __restrict__ pairs) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= B * m) return;
    const int64_t b = idx / m, j = idx - b * m;
    const float2* pc = part + b * nchunk * m + j;
    float mm = kNegBig;
    for (int c = 0; c < nchunk; ++c) mm = fmaxf(mm, pc[int64_t(c) * m].x);
    float ss = 0.0f;
    for (int c = 0; c < nchunk; ++c) {
        const float2 q = pc[int64_t(c) * m];
        ss = fmaf(q.y, exp_shift(q.x - mm), ss);
    }
    pairs[idx] = make_float2(mm, ss);
}

// v from the gathered pairs [nranks][B][m], merged in rank order (max pass,
// then the rescaled sums), written to pot_v and to y's records; every rank
// computes the same v.
__global__ void skp_rank_merge_kernel(const float2* __restrict__ pairs, int nranks, int64_t B, int64_t m, int d,
                                      const float* __restrict__ lb, float lb_def, float* __restrict__ pot_v,
                                      float* __restrict__ rec_y) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= B * m) return;
    const int64_t b = idx / m, j = idx - b * m;
    float mm = kNegBig;
    for (int r = 0; r < nranks; ++r) mm = fmaxf(mm, pairs[int64_t(r) * B * m + idx].x);
    float ss = 0.0f;
    for (int r = 0; r < nranks; ++r) {
        const float2 q = pairs[int64_t(r) * B * m + idx];
        ss = fmaf(q.y, exp_shift(q.x - mm), ss);
    }
    const float v = (lb ? lb[idx] : lb_def) - lse_finish(mm, ss);
    pot_v[idx] = v;
    rec_y[((b * (padded_points(m) / 2) + (j >> 1)) * rec_f4(d)) * 4 + 2 * d + (j & 1)] = v;
}

__global__ void skp_empty_pairs_kernel(float2* pairs, int64_t count) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < count) pairs[i] = make_float2(kNegBig, 0.0f);
}

// Plan P = safe_exp((K + u_i) + v_j) with K = C * kinv, C built from the
// points (out may be null: cost only), and per-row cost partials
// sum_j P_ij C_ij -- the arithmetic of the matrix epilogue (sk_plan_kernel)
// on sq_dist()'s entries.  One warp per row, four columns per lane.
template <int PD>
__global__ void __launch_bounds__(kPRows * 32)
skp_plan_kernel(const float* __restrict__ x, const float* __restrict__ y, float scale, float kinv,
                const float* __restrict__ u2, const float* __restrict__ v2, float* __restrict__ out,
                float* __restrict__ cost_row, int64_t rows, int64_t n, int64_t m) {
    const int lane = threadIdx.x & 31;
    const int64_t row = int64_t(blockIdx.x) * kPRows + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int64_t b = row / n;
    float xi[PD];
#pragma unroll
    for (int k = 0; k < PD; ++k) xi[k] = __ldg(x + row * PD + k);
    const float* yb = y + b * m * PD;
    const float* vb = v2 + b * m;
    float* orow = out != nullptr ? out + row * m : nullptr;
    const float uu = u2[row];
    float acc = 0.0f;
    const bool vec = (m & 3) == 0 && aligned16(yb) && aligned16(vb) && (orow == nullptr || aligned16(orow));
    if (vec) {
        for (int64_t q = lane; q < (m >> 2); q += 32) {
            float yv[4 * PD];
#pragma unroll
            for (int k = 0; k < PD; ++k) {
                const float4 f = __ldg(reinterpret_cast<const float4*>(yb + 4 * q * PD) + k);
                yv[4 * k + 0] = f.x;
                yv[4 * k + 1] = f.y;
                yv[4 * k + 2] = f.z;
                yv[4 * k + 3] = f.w;
            }
            const float4 v = __ldg(reinterpret_cast<const float4*>(vb) + q);
            const float vv[4] = {v.x, v.y, v.z, v.w};
            float o[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float yc[PD];
#pragma unroll
                for (int k = 0; k < PD; ++k) yc[k] = yv[c * PD + k];
                const float cij = sq_dist<PD>(xi, yc, scale);
                o[c] = safe_expf(__fadd_rn(kplus(cij, kinv, uu), vv[c]));
                acc = fmaf(o[c], cij, acc);
            }
            if (orow != nullptr) reinterpret_cast<float4*>(orow)[q] = make_float4(o[0], o[1], o[2], o[3]);
        }
    } else {
        for (int64_t j = lane; j < m; j += 32) {
            float yc[PD];
#pragma unroll
            for (int k = 0; k < PD; ++k) yc[k] = __ldg(yb + j * PD + k);
            const float cij = sq_dist<PD>(xi, yc, scale);
            const float p = safe_expf(__fadd_rn(kplus(cij, kinv, uu), __ldg(vb + j)));
            if (orow != nullptr) orow[j] = p;
            acc = fmaf(p, cij, acc);
        }
    }
    if (cost_row != nullptr) {
        acc = warp_sum<32>(acc);
        if (lane == 0) cost_row[row] = acc;
    }
}

// cost_b = sum_i cost_row[b, i] in a fixed order; one warp per problem.
__global__ void skp_cost_sum_kernel(const float* __restrict__ cost_row, float* __restrict__ cost, int64_t B,
                                    int64_t n) {
    const int lane = threadIdx.x & 31;
    const int64_t b = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= B) return;
    float acc = 0.0f;
    for (int64_t i = lane; i < n; i += 32) acc += cost_row[b * n + i];
    acc = warp_sum<32>(acc);
    if (lane == 0) cost[b] = acc;
}

// status = {n_iters, 0 (fixed iterations: not converged by a test), -, -}
__global__ void skp_status_kernel(int32_t* status, int n_iters) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        status[0] = n_iters;
        status[1] = 0;
    }
}

template <int PD>
void launch_plan(const float* x, const float* y, float scale, float kinv, const float* u2, const float* v2,
                 float* out, float* cost_row, int64_t rows, int64_t n, int64_t m, cudaStream_t st) {
    skp_plan_kernel<PD><<<unsigned(ceil_div(rows, kPRows)), kPRows * 32, 0, st>>>(x, y, scale, kinv, u2, v2, out,
                                                                                  cost_row, rows, n, m);
}

// Point-cloud kernels: up to four coordinates, fixed iteration count.
bool points_fused(int64_t d, float tol) { return tol == 0.0f && d >= 1 && d <= 4; }

// Chunks of side b for a half-step over na points of side a: enough CTAs for
// about two full waves of 16 resident CTAs per SM, chunks of at least 256
// points, a multiple of kHU points each.
struct HalfPlan {
    int nchunk;
    int64_t ch;
};
// Points of side a per lane and side-b pairs per step of the half-step kernel.
constexpr int kRL = 4;
constexpr int kNP = 4;

int sm_count_cached() {
    static int cached[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) {
        cudaGetLastError();
        n = 148;
    }
    if (dev >= 0 && dev < 64) cached[dev] = n;
    return n;
}

HalfPlan half_plan(int64_t B, int64_t na, int64_t nb) {
    const int64_t base = ceil_div(na, kHRows * kRL) * B;
    int64_t chunks = ceil_div(int64_t(2 * 16) * sm_count_cached(), base);
    chunks = std::max<int64_t>(1, std::min<int64_t>(chunks, ceil_div(nb, 256)));
    HalfPlan hp;
    hp.ch = ceil_div(ceil_div(nb, chunks), kHU) * kHU;
    hp.nchunk = int(ceil_div(nb, hp.ch));
    return hp;
}

struct PointsWs {
    float* recx;    // records of x (side b of the column half-steps)
    float* recy;    // records of y (side b of the row half-steps)
    float2* part;   // partials of the larger half-step
    float* cost_row;
};

PointsWs carve_points(Carve& c, int64_t B, int64_t n, int64_t m, int d, bool want_cost) {
    PointsWs w{};
    w.recx = c.take<float>(size_t(B * (padded_points(n) / 2) * 4 * rec_f4(d)));
    w.recy = c.take<float>(size_t(B * (padded_points(m) / 2) * 4 * rec_f4(d)));
    const HalfPlan hr = half_plan(B, n, m), hc = half_plan(B, m, n);
    w.part = c.take<float2>(size_t(std::max(B * hr.nchunk * n, B * hc.nchunk * m)));
    w.cost_row = want_cost ? c.take<float>(size_t(B * n)) : nullptr;
    return w;
}

template <int PD>
void launch_half(const HalfArgs& h, int64_t B, cudaStream_t st) {
    for (int64_t b0 = 0; b0 < B; b0 += kMaxGridZ) {
        const dim3 grid(unsigned(ceil_div(h.na, kHRows * kRL)), unsigned(h.nchunk),
                        unsigned(std::min<int64_t>(kMaxGridZ, B - b0)));
        skp_half_kernel<PD, kRL, kNP><<<grid, kHW * 32, 0, st>>>(h, b0);
    }
}

// One half-step: pot_a = l_a - LSE_b(K + w_b) for every point of side a, also
// stored into rec_a (side a's records) for the other half-step.
void half_step(const float* pa, float* rec_a, const float* rec_b, int64_t B, int64_t na, int64_t nb, int d,
               float kfold, float2* part, const float* la, float la_def, float* pot_a, cudaStream_t st) {
    const HalfPlan hp = half_plan(B, na, nb);
    HalfArgs h{pa, reinterpret_cast<const float4*>(rec_b), na, nb, hp.ch, hp.nchunk, kfold, part};
    switch (d) {
        case 1: launch_half<1>(h, B, st); break;
        case 2: launch_half<2>(h, B, st); break;
        case 3: launch_half<3>(h, B, st); break;
        default: launch_half<4>(h, B, st); break;
    }
    skp_merge_kernel<<<unsigned(ceil_div(B * na, 256)), 256, 0, st>>>(part, hp.nchunk, B, na, d, la, la_def, pot_a,
                                                                       rec_a);
}

bool bad_float(float v) { return !std::isfinite(v); }

// Row-shard workspace: the records of the shard's x (n rows) and of y, the
// partials of the larger half-step, the cost rows.
PointsWs carve_shard(Carve& c, int64_t B, int64_t n, int64_t m, int d) {
    return carve_points(c, B, n > 0 ? n : 1, m, d, true);
}

}  // namespace

size_t skp_shard_ws(int64_t B, int64_t n, int64_t m, int d) {
    Carve c(nullptr);
    carve_shard(c, B, n, m, d);
    return c.size();
}

int skp_shard_begin(const float* x, const float* y, int64_t B, int64_t n, int64_t m, int d, float* pot_u,
                    float* pot_v, void* ws, cudaStream_t st) {
    Carve c(ws);
    const PointsWs w = carve_shard(c, B, n, m, d);
    if (n > 0) cudaMemsetAsync(pot_u, 0, sizeof(float) * size_t(B * n), st);
    cudaMemsetAsync(pot_v, 0, sizeof(float) * size_t(B * m), st);
    ProfScope ps(DOT_K_SK_FWD_EPI, st);
    if (n > 0)
        skp_pack_kernel<<<unsigned(ceil_div(B * padded_points(n) / 2, 256)), 256, 0, st>>>(x, B, n, d, w.recx);
    skp_pack_kernel<<<unsigned(ceil_div(B * padded_points(m) / 2, 256)), 256, 0, st>>>(y, B, m, d, w.recy);
    return check_launch("point-cloud row shard set-up");
}

int skp_shard_rows_pairs(const float* x, const float* y, const float* la, float la_def, int64_t B, int64_t n,
                         int64_t m, int d, float kfold, float* pot_u, float2* pairs, void* ws, cudaStream_t st) {
    Carve c(ws);
    const PointsWs w = carve_shard(c, B, n, m, d);
    if (n == 0) {
        ProfScope ps(DOT_K_SK_EXCHANGE, st);
        skp_empty_pairs_kernel<<<unsigned(ceil_div(B * m, 256)), 256, 0, st>>>(pairs, B * m);
        return check_launch("point-cloud row shard (no rows)");
    }
    {
        ProfScope ps(DOT_K_SK_FWD_ITER, st, 2 * int(ceil_div(B, kMaxGridZ) + 1));
        half_step(x, w.recx, w.recy, B, n, m, d, kfold, w.part, la, la_def, pot_u, st);   // u of the shard's rows
        // column partials over the shard's rows with the new u: side a = y, side b = x
        const HalfPlan hp = half_plan(B, m, n);
        HalfArgs h{y, reinterpret_cast<const float4*>(w.recx), m, n, hp.ch, hp.nchunk, kfold, w.part};
        switch (d) {
            case 1: launch_half<1>(h, B, st); break;
            case 2: launch_half<2>(h, B, st); break;
            case 3: launch_half<3>(h, B, st); break;
            default: launch_half<4>(h, B, st); break;
        }
        skp_pairs_kernel<<<unsigned(ceil_div(B * m, 256)), 256, 0, st>>>(w.part, hp.nchunk, B, m, pairs);
    }
    return check_launch("point-cloud row shard half-steps");
}

int skp_shard_col_merge(const float2* gathered, int nranks, const float* lb, float lb_def, int64_t B, int64_t n,
                        int64_t m, int d, float* pot_v, void* ws, cudaStream_t st) {
    Carve c(ws);
    const PointsWs w = carve_shard(c, B, n, m, d);
    ProfScope ps(DOT_K_SK_EXCHANGE, st);
    skp_rank_merge_kernel<<<unsigned(ceil_div(B * m, 256)), 256, 0, st>>>(gathered, nranks, B, m, d, lb, lb_def,
                                                                          pot_v, w.recy);
    return check_launch("point-cloud column merge");
}

int skp_shard_plan(const float* x, const float* y, int64_t B, int64_t n, int64_t m, int d, float cost_scale,
                   float kinv, const float* pot_u, const float* pot_v, float* plan, float* cost, void* ws,
                   cudaStream_t st) {
    Carve c(ws);
    const PointsWs w = carve_shard(c, B, n, m, d);
    ProfScope ps(DOT_K_SK_FWD_EPI, st);
    if (n == 0) {
        if (cost != nullptr) cudaMemsetAsync(cost, 0, sizeof(float) * size_t(B), st);
        return check_launch("point-cloud row shard plan");
    }
    const int64_t rows = B * n;
    float* crow = cost != nullptr ? w.cost_row : nullptr;
    switch (d) {
        case 1: launch_plan<1>(x, y, cost_scale, kinv, pot_u, pot_v, plan, crow, rows, n, m, st); break;
        case 2: launch_plan<2>(x, y, cost_scale, kinv, pot_u, pot_v, plan, crow, rows, n, m, st); break;
        case 3: launch_plan<3>(x, y, cost_scale, kinv, pot_u, pot_v, plan, crow, rows, n, m, st); break;
        default: launch_plan<4>(x, y, cost_scale, kinv, pot_u, pot_v, plan, crow, rows, n, m, st); break;
    }
    if (cost != nullptr) skp_cost_sum_kernel<<<unsigned(ceil_div(B, 8)), 256, 0, st>>>(w.cost_row, cost, B, n);
    return check_launch("point-cloud row shard plan");
}

}  // namespace dotb

using namespace dotb;

extern "C" {

int dot_sq_dist(const float* x, const float* y, int64_t B, int64_t n, int64_t m, int d, float cost_scale, float* C,
                void* stream) {
    clear_error();
    if (B < 0 || n < 0 || m < 0) return fail(DOT_ERR_INVALID, "negative dimension");
    if (d < 1) return fail(DOT_ERR_INVALID, "point dimension must be >= 1");
    if (bad_float(cost_scale)) return fail(DOT_ERR_INVALID, "cost_scale must be finite");
    if (B == 0 || n == 0 || m == 0) return DOT_OK;
    if (!x || !y || !C) return fail(DOT_ERR_INVALID, "null tensor pointer");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t rows = B * n;
    {
        ProfScope ps(DOT_K_SK_FWD_EPI, st);
        skp_sqdist_kernel<<<unsigned(ceil_div(rows, kPRows)), kPRows * 32, 0, st>>>(x, y, rows, n, m, d, cost_scale,
                                                                                     C);
    }
    return check_launch("squared distances");
}

size_t dot_sinkhorn_points_fwd_workspace_bytes(int64_t B, int64_t n, int64_t m, int d, int n_iters, float tol,
                                               int want_plan, int want_cost) {
    if (B <= 0 || n <= 0 || m <= 0 || d <= 0) return 0;
    Carve c(nullptr);
    if (points_fused(d, tol)) {
        carve_points(c, B, n, m, d, want_cost != 0);
        return c.size();
    }
    c.take<float>(size_t(B * n * m));                  // the materialised cost
    if (!want_plan) c.take<float>(size_t(B * n * m));  // a plan for the matrix solvers to write
    c.take<char>(dot_sinkhorn_fwd_workspace_bytes(B, n, m, n_iters, tol, want_cost));
    return c.size();
}

int dot_sinkhorn_points_fwd(const float* x, const float* y, int64_t B, int64_t n, int64_t m, int d,
                            float cost_scale, const float* log_a, const float* log_b, float tau, int n_iters,
                            float tol, float* plan, float* cost, float* pot_u, float* pot_v, int32_t* status,
                            void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    if (B < 0 || n < 0 || m < 0) return fail(DOT_ERR_INVALID, "negative dimension");
    if (d < 1) return fail(DOT_ERR_INVALID, "point dimension must be >= 1");
    if (!(tau > 0.0f) || bad_float(tau)) return fail(DOT_ERR_INVALID, "tau must be > 0");
    if (n_iters < 0) return fail(DOT_ERR_INVALID, "n_iters must be >= 0");
    if (bad_float(tol) || tol < 0.0f) return fail(DOT_ERR_INVALID, "tol must be finite and >= 0");
    if (bad_float(cost_scale)) return fail(DOT_ERR_INVALID, "cost_scale must be finite");
    if (B == 0 || n == 0 || m == 0) return DOT_OK;
    if (!x || !y || !pot_u || !pot_v || !status) return fail(DOT_ERR_INVALID, "null tensor pointer");
    const size_t need =
        dot_sinkhorn_points_fwd_workspace_bytes(B, n, m, d, n_iters, tol, plan != nullptr, cost != nullptr);
    if (workspace == nullptr || workspace_bytes < need)
        return fail(DOT_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes");
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    if (!points_fused(d, tol)) {
        Carve c(workspace);
        float* C = c.take<float>(size_t(B * n * m));
        float* P = plan != nullptr ? plan : c.take<float>(size_t(B * n * m));
        const size_t fws = dot_sinkhorn_fwd_workspace_bytes(B, n, m, n_iters, tol, cost != nullptr);
        void* rest = c.take<char>(fws);
        int rc = dot_sq_dist(x, y, B, n, m, d, cost_scale, C, stream);
        if (rc != DOT_OK) return rc;
        return dot_sinkhorn_fwd(C, -1.0f, log_a, log_b, B, n, m, tau, n_iters, tol, 0, P, cost, pot_u, pot_v,
                                status, rest, fws, stream);
    }

    Carve c(workspace);
    const PointsWs w = carve_points(c, B, n, m, d, cost != nullptr);
    const float kinv = -(1.0f / tau);
    const float kfold = cost_scale * kinv;
    const float la_def = -logf(float(n)), lb_def = -logf(float(m));   // uniform marginals, as dot_sinkhorn_fwd
    const int64_t rows = B * n;
    cudaMemsetAsync(pot_u, 0, sizeof(float) * size_t(rows), st);
    cudaMemsetAsync(pot_v, 0, sizeof(float) * size_t(B * m), st);
    cudaMemsetAsync(status, 0, sizeof(int32_t) * 4, st);
    {
        ProfScope ps(DOT_K_SK_FWD_EPI, st);
        skp_pack_kernel<<<unsigned(ceil_div(B * padded_points(n) / 2, 256)), 256, 0, st>>>(x, B, n, d, w.recx);
        skp_pack_kernel<<<unsigned(ceil_div(B * padded_points(m) / 2, 256)), 256, 0, st>>>(y, B, m, d, w.recy);
    }
    if (n_iters > 0) {
        // two half-steps per iteration, each a launch per batch slice and a merge
        const int per_iter = 2 * int(ceil_div(B, kMaxGridZ) + 1);
        ProfScope ps(DOT_K_SK_FWD_ITER, st, per_iter * n_iters);
        for (int it = 0; it < n_iters; ++it) {
            half_step(x, w.recx, w.recy, B, n, m, d, kfold, w.part, log_a, la_def, pot_u, st);   // u
            half_step(y, w.recy, w.recx, B, m, n, d, kfold, w.part, log_b, lb_def, pot_v, st);   // v
        }
    }
    {
        ProfScope ps(DOT_K_SK_FWD_EPI, st);
        skp_status_kernel<<<1, 32, 0, st>>>(status, n_iters);
    }
    if (plan != nullptr || cost != nullptr) {
        ProfScope ps(DOT_K_SK_FWD_EPI, st);
        switch (d) {
            case 1: launch_plan<1>(x, y, cost_scale, kinv, pot_u, pot_v, plan, w.cost_row, rows, n, m, st); break;
            case 2: launch_plan<2>(x, y, cost_scale, kinv, pot_u, pot_v, plan, w.cost_row, rows, n, m, st); break;
            case 3: launch_plan<3>(x, y, cost_scale, kinv, pot_u, pot_v, plan, w.cost_row, rows, n, m, st); break;
            default: launch_plan<4>(x, y, cost_scale, kinv, pot_u, pot_v, plan, w.cost_row, rows, n, m, st); break;
        }
    }
    if (cost != nullptr) {
        ProfScope ps(DOT_K_SK_FWD_EPI, st);
        skp_cost_sum_kernel<<<unsigned(ceil_div(B, 8)), 256, 0, st>>>(w.cost_row, cost, B, n);
    }
    return check_launch("sinkhorn forward (point clouds)");
}

}  // extern "C"

// Unrolled Sinkhorn backward: differentiation through the stored iterations
// (backward_mode='unrolled').
//
// The forward records the dual potentials after every half-step
// (dot_sinkhorn_fwd_hist: u_hist[t] after the row update of iteration t,
// v_hist[t] after its column update).  With K = X * (sign/tau) and
// G = dLoss/dP, the backward runs
//     Gamma = G * P
//     for t = T-1 .. 0:
//         column step  Gamma_Y_ik = Gamma_ik - exp(K_ik + u_t,i + v_t,k) * sum_i Gamma_ik
//         row step     Gamma_ik   = Gamma_Y_ik - exp(K_ik + u_t,i + v_{t-1},k) * sum_k Gamma_Y_ik
//                      (v_{-1} = 0)
//     grad_log_alpha = Gamma / tau,  grad_tau = -sum(Gamma * log_alpha) / tau^2
// which is the reference's dual unrolled backward
// (src/sinkhorn/kernels.cu:844-961,1622-1680; CPU form kernels_cpu.cpp:169-245)
// with its operation order for the exponent ((K + u) + v) and its clamped
// exp.  Per reverse step: one column-sum pass (CTA per 128 columns x row
// chunk, fixed-order merge: deterministic) and one warp-per-row pass that
// applies the column step, reduces the row, and applies the row step.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "sinkhorn.h"

namespace dotb {

namespace {

constexpr int kUT = 256;            // threads per CTA
constexpr int kUW = kUT / 32;
constexpr int kUColTile = 128;      // columns per column-sum CTA
constexpr int64_t kURowsPerChunk = 512;

// Gamma = G * P with G = grad_P + g_cost[b] * X (the cost term exists for
// score_sign = -1, where X is the cost).
__global__ void sku_init_kernel(const float* __restrict__ X, const float* __restrict__ P,
                                const float* __restrict__ gP, const float* __restrict__ gcost, bool cost_term,
                                float* __restrict__ Gm, int64_t nm, int64_t total) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    float g = gP ? gP[idx] : 0.0f;
    if (cost_term && gcost) g += gcost[idx / nm] * X[idx];
    Gm[idx] = g * P[idx];
}

// Column sums of Gamma over a row chunk: grid (ceil(m/128), chunks, B).
__global__ void __launch_bounds__(kUT)
sku_colsum_kernel(const float* __restrict__ Gm, int64_t n, int64_t m, int64_t rows_per_chunk, int chunks,
                  float* __restrict__ part, float* __restrict__ s_out, int64_t b0) {
    __shared__ float sm[kUW][kUColTile];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t b = b0 + blockIdx.z, chunk = blockIdx.y;
    const int64_t cbase = int64_t(blockIdx.x) * kUColTile;
    const int64_t r0 = chunk * rows_per_chunk, r1 = min(n, r0 + rows_per_chunk);
    const float* gb = Gm + b * n * m;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int64_t r = r0 + wid; r < r1; r += kUW) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int64_t c = cbase + lane + 32 * k;
            if (c < m) acc[k] += gb[r * m + c];
        }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) sm[wid][lane + 32 * k] = acc[k];
    __syncthreads();
    if (threadIdx.x < kUColTile) {
        const int64_t c = cbase + threadIdx.x;
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < kUW; ++w) s += sm[w][threadIdx.x];
        if (c < m) {
            if (chunks > 1) part[(b * chunks + chunk) * m + c] = s;
            else s_out[b * m + c] = s;
        }
    }
}

__global__ void sku_colsum_merge_kernel(const float* __restrict__ part, int chunks, int64_t B, int64_t m,
                                        float* __restrict__ s_out) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= B * m) return;
    const int64_t b = idx / m, c = idx - b * m;
    float s = 0.0f;
    for (int k = 0; k < chunks; ++k) s += part[(b * chunks + k) * m + c];
    s_out[idx] = s;
}

// One reverse step for one row per warp (column step, row reduction, row step).
__global__ void __launch_bounds__(kUT)
sku_step_kernel(const float* __restrict__ X, float kinv, const float* __restrict__ u_t,
                const float* __restrict__ v_t, const float* __restrict__ v_prev, const float* __restrict__ colsum,
                float* __restrict__ Gm, int64_t rows, int64_t n, int64_t m) {
    const int lane = threadIdx.x & 31;
    const int64_t row = int64_t(blockIdx.x) * kUW + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int64_t b = row / n;
    const float* xr = X + row * m;
    float* gr = Gm + row * m;
    const float* vt = v_t + b * m;
    const float* vp = v_prev ? v_prev + b * m : nullptr;
    const float* sb = colsum + b * m;
    const float ut = u_t[row];
    float ti = 0.0f;
    for (int64_t j = lane; j < m; j += 32) {
        const float ku = __fadd_rn(__fmul_rn(xr[j], kinv), ut);
        const float gy = gr[j] - safe_expf(__fadd_rn(ku, vt[j])) * sb[j];
        gr[j] = gy;
        ti += gy;
    }
    ti = warp_sum<32>(ti);
    for (int64_t j = lane; j < m; j += 32) {
        const float ku = __fadd_rn(__fmul_rn(xr[j], kinv), ut);
        const float p = safe_expf(__fadd_rn(ku, vp ? vp[j] : 0.0f));
        gr[j] = gr[j] - p * ti;
    }
}

// grad_X = sign * Gamma / tau (+ g_cost[b] * P for the cost term); per-row
// sums of Gamma * log_alpha (log_alpha = sign * X) for the tau gradient.
__global__ void __launch_bounds__(kUT)
sku_final_kernel(const float* __restrict__ X, float sign, const float* __restrict__ P,
                 const float* __restrict__ gcost, bool cost_term, const float* __restrict__ Gm, float inv_tau,
                 float* __restrict__ gX, float* __restrict__ tau_row, int64_t rows, int64_t n, int64_t m) {
    const int lane = threadIdx.x & 31;
    const int64_t row = int64_t(blockIdx.x) * kUW + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float gc = (cost_term && gcost) ? gcost[row / n] : 0.0f;
    float acc = 0.0f;
    for (int64_t j = lane; j < m; j += 32) {
        const int64_t idx = row * m + j;
        const float g = Gm[idx];
        float d = sign * (g * inv_tau);
        if (cost_term && gcost) d += gc * P[idx];
        gX[idx] = d;
        acc += g * (sign * X[idx]);
    }
    if (tau_row != nullptr) {
        acc = warp_sum<32>(acc);
        if (lane == 0) tau_row[row] = acc;
    }
}

__global__ void sku_batch_sum_kernel(const float* __restrict__ row_part, float* __restrict__ outv, int64_t B,
                                     int64_t n, float scale) {
    const int lane = threadIdx.x & 31;
    const int64_t b = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= B) return;
    float acc = 0.0f;
    for (int64_t i = lane; i < n; i += 32) acc += row_part[b * n + i];
    acc = warp_sum<32>(acc);
    if (lane == 0) outv[b] = acc * scale;
}

struct UnrolledWs {
    float* gamma;     // [B, n, m]
    float* colsum;    // [B, m]
    float* part;      // [B, chunks, m] or nullptr
    float* tau_row;   // [B, n]
};

UnrolledWs carve_unrolled(Carve& c, int64_t B, int64_t n, int64_t m) {
    UnrolledWs w{};
    const int64_t chunks = ceil_div(n, kURowsPerChunk);
    w.gamma = c.take<float>(size_t(B * n * m));
    w.colsum = c.take<float>(size_t(B * m));
    w.part = chunks > 1 ? c.take<float>(size_t(B * chunks * m)) : nullptr;
    w.tau_row = c.take<float>(size_t(B * n));
    return w;
}

}  // namespace

size_t sk_unrolled_bwd_ws(int64_t B, int64_t n, int64_t m) {
    Carve c(nullptr);
    carve_unrolled(c, B, n, m);
    return c.size();
}

int sk_unrolled_bwd(const SkBwdArgs& a, const float* u_hist, const float* v_hist, void* ws, cudaStream_t st) {
    Carve c(ws);
    UnrolledWs w = carve_unrolled(c, a.B, a.n, a.m);
    const int64_t rows = a.B * a.n, total = rows * a.m;
    const int chunks = int(ceil_div(a.n, kURowsPerChunk));
    const int64_t rpc = chunks > 1 ? kURowsPerChunk : a.n;
    const bool cost_term = a.sign < 0.0f && a.gcost != nullptr;
    const float kinv = a.sign * (1.0f / a.tau);
    const dim3 col_grid(unsigned(ceil_div(a.m, kUColTile)), unsigned(chunks), unsigned(a.B));
    const unsigned row_grid = unsigned(ceil_div(rows, kUW));
    {
        ProfScope ps(DOT_K_SK_BWD_EPI, st);
        sku_init_kernel<<<unsigned(ceil_div(total, 256)), 256, 0, st>>>(a.X, a.P, a.gP, a.gcost, cost_term, w.gamma,
                                                                         a.n * a.m, total);
    }
    if (a.bwd_iters > 0) {
        ProfScope ps(DOT_K_SK_BWD_ITER, st, a.bwd_iters * (chunks > 1 ? 3 : 2));
        for (int t = a.bwd_iters - 1; t >= 0; --t) {
            for (int64_t b0 = 0; b0 < a.B; b0 += kMaxGridZ) {
                const dim3 gz(col_grid.x, col_grid.y, unsigned(std::min<int64_t>(kMaxGridZ, a.B - b0)));
                sku_colsum_kernel<<<gz, kUT, 0, st>>>(w.gamma, a.n, a.m, rpc, chunks, w.part, w.colsum, b0);
            }
            if (chunks > 1)
                sku_colsum_merge_kernel<<<unsigned(ceil_div(a.B * a.m, 256)), 256, 0, st>>>(w.part, chunks, a.B,
                                                                                          a.m, w.colsum);
            sku_step_kernel<<<row_grid, kUT, 0, st>>>(a.X, kinv, u_hist + int64_t(t) * rows,
                                                      v_hist + int64_t(t) * a.B * a.m,
                                                      t > 0 ? v_hist + int64_t(t - 1) * a.B * a.m : nullptr,
                                                      w.colsum, w.gamma, rows, a.n, a.m);
        }
    }
    {
        ProfScope ps(DOT_K_SK_BWD_EPI, st);
        sku_final_kernel<<<row_grid, kUT, 0, st>>>(a.X, a.sign, a.P, a.gcost, cost_term, w.gamma, 1.0f / a.tau, a.gX,
                                                   a.gtau ? w.tau_row : nullptr, rows, a.n, a.m);
    }
    if (a.gtau != nullptr) {
        ProfScope ps(DOT_K_SK_BWD_EPI, st);
        sku_batch_sum_kernel<<<unsigned(ceil_div(a.B, 8)), 256, 0, st>>>(w.tau_row, a.gtau, a.B, a.n,
                                                                         -1.0f / (a.tau * a.tau));
    }
    return check_launch("sinkhorn unrolled backward");
}

}  // namespace dotb

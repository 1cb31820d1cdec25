// Streaming Sinkhorn kernels (any B, n, m): the cost stays in HBM and every
// iteration sweeps it.  These are the general path; the on-chip resident
// solvers in sinkhorn_resident.cu take over for shapes that fit.
//
// Forward iteration (reference: src/sinkhorn/torch_cuda.cpp:188-239, kernels
// src/sinkhorn/kernels.cu:503-753):
//   row pass   u_i = la_i - LSE_j(K_ij + v_j)     warp per row, coalesced float4
//   col pass   v_j = lb_j - LSE_i(K_ij + u_i)     CTA = 128 columns x row chunk,
//                                                 each warp walks rows (coalesced
//                                                 512-byte row segments) and keeps
//                                                 per-column online (max, sum)
//   col merge  chunk partials -> v (only when n spans several chunks)
// K = X * (sign/tau) is formed on the fly with the reference's rounding (no
// materialised log_K, unlike the reference's sinkhorn_init_kernel,
// kernels.cu:128-139).  Reductions run in
// a fixed order (no atomics on results), so results are deterministic.
//
// Implicit backward (reference: kernels.cu:965-1098, 1682-1726): the
// iteration-invariant sums sum_k P G, sum_k P (rows) and sum_i P G, sum_i P
// (columns) are computed once; each sweep is then a row mat-vec P mu and a
// column mat-vec P^T lambda.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "sinkhorn.h"
#include "tma.cuh"

namespace dotb {

namespace {

constexpr int kRowThreads = 256;          // 8 warps, one row each
constexpr int kRowsPerCta = kRowThreads / 32;
constexpr int kColWarps = 8;
constexpr int kColTile = 128;             // columns per column-pass CTA
constexpr int kColUnroll = 4;             // rows per warp per step

// Iteration control for tol > 0 (device-side early stop, no host sync).
// status = {n_iters_used, converged, done, unused}; delta[t] = max |du| of
// iteration t over the whole batch (the reference's criterion,
// src/sinkhorn/torch_cuda.cpp:225-238, which checks only u).
struct SkCtl {
    float* delta;
    int32_t* status;
    float tol;
    int iter;
};

__device__ __forceinline__ bool ctl_done(const SkCtl& c) {
    return c.delta != nullptr && *reinterpret_cast<volatile int32_t*>(c.status + 2) != 0;
}

// ---------------------------------------------------------------------------
// forward row pass
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kRowThreads)
sk_row_kernel(const float* __restrict__ X, float kinv, const float* __restrict__ v2,
              const float* __restrict__ la, float la_def, float* __restrict__ u2,
              int64_t rows, int64_t n, int64_t m, SkCtl ctl) {
    __shared__ float s_delta[kRowsPerCta];
    if (ctl.delta != nullptr) {
        if (ctl_done(ctl)) return;
        if (ctl.iter > 0 && ctl.delta[ctl.iter - 1] < ctl.tol) {
            if (blockIdx.x == 0 && threadIdx.x == 0) {
                ctl.status[0] = ctl.iter;
                ctl.status[1] = 1;
                ctl.status[2] = 1;
            }
            return;
        }
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t row = int64_t(blockIdx.x) * kRowsPerCta + wid;
    float dmax = 0.0f;
    if (row < rows) {
        const float* xr = X + row * m;
        const float* vb = v2 + (row / n) * m;
        float M = kNegBig, S = 0.0f;
        if (((m & 3) == 0) && aligned16(X) && aligned16(v2)) {
            const float4* x4 = reinterpret_cast<const float4*>(xr);
            const float4* v4 = reinterpret_cast<const float4*>(vb);
            const int64_t m4 = m >> 2;
            for (int64_t q0 = 0; q0 < m4; q0 += 128) {
                float t[16];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int64_t q = q0 + u * 32 + lane;
                    if (q < m4) {
                        const float4 x = __ldg(x4 + q);
                        const float4 v = __ldg(v4 + q);
                        t[4 * u + 0] = kplus(x.x, kinv, v.x);
                        t[4 * u + 1] = kplus(x.y, kinv, v.y);
                        t[4 * u + 2] = kplus(x.z, kinv, v.z);
                        t[4 * u + 3] = kplus(x.w, kinv, v.w);
                    } else {
                        t[4 * u + 0] = t[4 * u + 1] = t[4 * u + 2] = t[4 * u + 3] = -INFINITY;
                    }
                }
                lse_push<16>(M, S, t);
            }
        } else {
            for (int64_t j0 = 0; j0 < m; j0 += 128) {
                float t[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int64_t j = j0 + u * 32 + lane;
                    t[u] = j < m ? kplus(__ldg(xr + j), kinv, __ldg(vb + j)) : -INFINITY;
                }
                lse_push<4>(M, S, t);
            }
        }
        warp_lse<32>(M, S);
        if (lane == 0) {
            const float unew = (la ? la[row] : la_def) - lse_finish(M, S);
            dmax = fabsf(unew - u2[row]);
            u2[row] = unew;
        }
    }
    if (ctl.delta != nullptr) {
        if (lane == 0) s_delta[wid] = dmax;
        __syncthreads();
        if (threadIdx.x == 0) {
            float mx = 0.0f;
#pragma unroll
            for (int w = 0; w < kRowsPerCta; ++w) mx = fmaxf(mx, s_delta[w]);
            atomic_max_nonneg(ctl.delta + ctl.iter, mx);
        }
    }
}

// ---------------------------------------------------------------------------
// forward column pass: CTA = 128 columns x one row chunk of one problem
// grid (ceil(m/128), chunks, B)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kColWarps * 32)
sk_col_kernel(const float* __restrict__ X, float kinv, const float* __restrict__ u2,
              const float* __restrict__ lb, float lb_def, float* __restrict__ v2,
              float2* __restrict__ part, int64_t n, int64_t m, int64_t rows_per_chunk,
              int chunks, SkCtl ctl, float2* __restrict__ pair_out, int64_t b0) {
    __shared__ float sm_M[kColWarps][kColTile];
    __shared__ float sm_S[kColWarps][kColTile];
    if (ctl_done(ctl)) return;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t b = b0 + blockIdx.z, chunk = blockIdx.y;
    const int64_t cbase = int64_t(blockIdx.x) * kColTile;
    const int64_t r0 = chunk * rows_per_chunk;
    const int64_t r1 = min(n, r0 + rows_per_chunk);
    const float* Xb = X + b * n * m;
    const float* ub = u2 + b * n;
    float M[4], S[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) { M[k] = kNegBig; S[k] = 0.0f; }
    const bool vec = ((m & 3) == 0) && aligned16(X);
    for (int64_t r = r0 + wid; r < r1; r += kColWarps * kColUnroll) {
        float t[4][kColUnroll];
#pragma unroll
        for (int u = 0; u < kColUnroll; ++u) {
            const int64_t rr = r + int64_t(u) * kColWarps;
            const bool rok = rr < r1;
            const float uu = rok ? __ldg(ub + rr) : 0.0f;
            if (vec) {
                const int64_t c0 = cbase + 4 * lane;
                if (rok && c0 < m) {
                    const float4 x = __ldg(reinterpret_cast<const float4*>(Xb + rr * m + c0));
                    t[0][u] = kplus(x.x, kinv, uu);
                    t[1][u] = kplus(x.y, kinv, uu);
                    t[2][u] = kplus(x.z, kinv, uu);
                    t[3][u] = kplus(x.w, kinv, uu);
                } else {
                    t[0][u] = t[1][u] = t[2][u] = t[3][u] = -INFINITY;
                }
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int64_t c = cbase + lane + 32 * k;
                    t[k][u] = (rok && c < m) ? kplus(__ldg(Xb + rr * m + c), kinv, uu) : -INFINITY;
                }
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) lse_push<kColUnroll>(M[k], S[k], t[k]);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int slot = vec ? 4 * lane + k : lane + 32 * k;
        sm_M[wid][slot] = M[k];
        sm_S[wid][slot] = S[k];
    }
    __syncthreads();
    if (threadIdx.x < kColTile) {
        const int ci = threadIdx.x;
        const int64_t col = cbase + ci;
        float mm = sm_M[0][ci], ss = sm_S[0][ci];
#pragma unroll
        for (int w = 1; w < kColWarps; ++w) lse_merge(mm, ss, sm_M[w][ci], sm_S[w][ci]);
        if (col < m) {
            if (chunks > 1) part[(b * chunks + chunk) * m + col] = make_float2(mm, ss);
            else if (pair_out != nullptr) pair_out[b * m + col] = make_float2(mm, ss);
            else v2[b * m + col] = (lb ? lb[b * m + col] : lb_def) - lse_finish(mm, ss);
        }
    }
}

__global__ void sk_col_merge_kernel(const float2* __restrict__ part, const float* __restrict__ lb,
                                    float lb_def, float* __restrict__ v2, int64_t B, int64_t m,
                                    int chunks, SkCtl ctl, float2* __restrict__ pair_out) {
    if (ctl_done(ctl)) return;
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= B * m) return;
    const int64_t b = idx / m, col = idx - b * m;
    float mm = kNegBig, ss = 0.0f;
    for (int c = 0; c < chunks; ++c) {
        const float2 p = part[(b * chunks + c) * m + col];
        lse_merge(mm, ss, p.x, p.y);
    }
    if (pair_out != nullptr) pair_out[idx] = make_float2(mm, ss);
    else v2[idx] = (lb ? lb[idx] : lb_def) - lse_finish(mm, ss);
}

// Shard combine in one step: pairs [parts][count] (each shard's column
// (max, sum) over its rows, gathered from every rank) merged in shard order.
__global__ void sk_shard_merge_kernel(const float2* __restrict__ pairs, int parts, const float* __restrict__ lb,
                                      float lb_def, float* __restrict__ v2, int64_t count) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= count) return;
    float mm = kNegBig, ss = 0.0f;
    for (int p = 0; p < parts; ++p) {
        const float2 q = pairs[int64_t(p) * count + i];
        lse_merge(mm, ss, q.x, q.y);
    }
    v2[i] = (lb ? lb[i] : lb_def) - lse_finish(mm, ss);
}

// ---------------------------------------------------------------------------
// forward epilogue: plan (or log-plan) + per-row cost, warp per row
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kRowThreads)
sk_plan_kernel(const float* __restrict__ X, float kinv, const float* __restrict__ u2,
               const float* __restrict__ v2, float* __restrict__ out, int out_mode,
               float* __restrict__ cost_row, int64_t rows, int64_t n, int64_t m) {
    // log P = (K + u_i) + v_j, P = safe_exp(log P): src/sinkhorn/kernels.cu:755-775
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t row = int64_t(blockIdx.x) * kRowsPerCta + wid;
    if (row >= rows) return;
    const float* xr = X + row * m;
    const float* vb = v2 + (row / n) * m;
    float* orow = out + row * m;
    const float uu = u2[row];
    float acc = 0.0f;
    if (((m & 3) == 0) && aligned16(X) && aligned16(out) && aligned16(v2)) {
        const int64_t m4 = m >> 2;
        for (int64_t q = lane; q < m4; q += 32) {
            const float4 x = __ldg(reinterpret_cast<const float4*>(xr) + q);
            const float4 v = __ldg(reinterpret_cast<const float4*>(vb) + q);
            float4 o;
            const float t0 = __fadd_rn(kplus(x.x, kinv, uu), v.x);
            const float t1 = __fadd_rn(kplus(x.y, kinv, uu), v.y);
            const float t2 = __fadd_rn(kplus(x.z, kinv, uu), v.z);
            const float t3 = __fadd_rn(kplus(x.w, kinv, uu), v.w);
            if (out_mode == 0) {
                o = make_float4(safe_expf(t0), safe_expf(t1), safe_expf(t2), safe_expf(t3));
                acc += o.x * x.x + o.y * x.y + o.z * x.z + o.w * x.w;
            } else {
                o = make_float4(t0, t1, t2, t3);
            }
            reinterpret_cast<float4*>(orow)[q] = o;
        }
    } else {
        for (int64_t j = lane; j < m; j += 32) {
            const float x = __ldg(xr + j);
            const float t = __fadd_rn(kplus(x, kinv, uu), __ldg(vb + j));
            if (out_mode == 0) {
                const float p = safe_expf(t);
                orow[j] = p;
                acc += p * x;
            } else {
                orow[j] = t;
            }
        }
    }
    if (cost_row != nullptr) {
        acc = warp_sum<32>(acc);
        if (lane == 0) cost_row[row] = acc;
    }
}

// Sum per-row partials of each batch in a fixed order: one warp per batch.
// out_b = scale * sum_i row_part[b, i].
__global__ void sk_batch_sum_kernel(const float* __restrict__ row_part, float* __restrict__ outv,
                                    int64_t B, int64_t n, float scale) {
    const int lane = threadIdx.x & 31;
    const int64_t b = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= B) return;
    float acc = 0.0f;
    for (int64_t i = lane; i < n; i += 32) acc += row_part[b * n + i];
    acc = warp_sum<32>(acc);
    if (lane == 0) outv[b] = acc * scale;
}

// Final n_iters_used / converged for the whole batch (single thread).
__global__ void sk_status_kernel(const float* __restrict__ delta, int32_t* __restrict__ status,
                                 int n_iters, float tol) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    if (delta == nullptr) {
        status[0] = n_iters;
        status[1] = 0;
        return;
    }
    if (status[2] != 0) return;  // stopped early; fields already written
    status[0] = n_iters;
    status[1] = (n_iters > 0 && delta[n_iters - 1] < tol) ? 1 : 0;
    status[2] = 1;
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------

__device__ __forceinline__ float grad_total(float x, float gc, const float* gP, int64_t idx) {
    // G = grad_cost_b * X + grad_P, rounded as autograd forms it (product, then sum).
    float g = __fmul_rn(gc, x);
    if (gP != nullptr) g = __fadd_rn(g, __ldg(gP + idx));
    return g;
}

// Row invariants: rinv[row] = (sum_k P G, sum_k P).  Warp per row.
__global__ void __launch_bounds__(kRowThreads)
skb_row_prep_kernel(const float* __restrict__ X, const float* __restrict__ P,
                    const float* __restrict__ gP, const float* __restrict__ gcost,
                    float2* __restrict__ rinv, int64_t rows, int64_t n, int64_t m) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t row = int64_t(blockIdx.x) * kRowsPerCta + wid;
    if (row >= rows) return;
    const float gc = gcost ? gcost[row / n] : 0.0f;
    float spg = 0.0f, sp = 0.0f;
    for (int64_t j = lane; j < m; j += 32) {
        const int64_t idx = row * m + j;
        const float p = __ldg(P + idx);
        spg += p * grad_total(__ldg(X + idx), gc, gP, idx);
        sp += p;
    }
    spg = warp_sum<32>(spg);
    sp = warp_sum<32>(sp);
    if (lane == 0) rinv[row] = make_float2(spg, sp);
}

// Column invariants over a row chunk: (sum_i P G, sum_i P); grid (ceil(m/128), chunks, B).
__global__ void __launch_bounds__(kColWarps * 32)
skb_col_prep_kernel(const float* __restrict__ X, const float* __restrict__ P,
                    const float* __restrict__ gP, const float* __restrict__ gcost,
                    float2* __restrict__ cinv, float2* __restrict__ part, int64_t n, int64_t m,
                    int64_t rows_per_chunk, int chunks, int64_t b0) {
    __shared__ float2 sm[kColWarps][kColTile];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t b = b0 + blockIdx.z, chunk = blockIdx.y;
    const int64_t cbase = int64_t(blockIdx.x) * kColTile;
    const int64_t r0 = chunk * rows_per_chunk, r1 = min(n, r0 + rows_per_chunk);
    const float gc = gcost ? gcost[b] : 0.0f;
    float spg[4] = {0, 0, 0, 0}, sp[4] = {0, 0, 0, 0};
    for (int64_t r = r0 + wid; r < r1; r += kColWarps) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int64_t c = cbase + lane + 32 * k;
            if (c < m) {
                const int64_t idx = (b * n + r) * m + c;
                const float p = __ldg(P + idx);
                spg[k] += p * grad_total(__ldg(X + idx), gc, gP, idx);
                sp[k] += p;
            }
        }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) sm[wid][lane + 32 * k] = make_float2(spg[k], sp[k]);
    __syncthreads();
    if (threadIdx.x < kColTile) {
        const int ci = threadIdx.x;
        const int64_t col = cbase + ci;
        float2 acc = sm[0][ci];
#pragma unroll
        for (int w = 1; w < kColWarps; ++w) {
            acc.x += sm[w][ci].x;
            acc.y += sm[w][ci].y;
        }
        if (col < m) {
            if (chunks == 1) cinv[b * m + col] = acc;
            else part[(b * chunks + chunk) * m + col] = acc;
        }
    }
}

__global__ void skb_col_prep_merge_kernel(const float2* __restrict__ part, float2* __restrict__ cinv,
                                          int64_t B, int64_t m, int chunks) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= B * m) return;
    const int64_t b = idx / m, col = idx - b * m;
    float2 acc = make_float2(0.0f, 0.0f);
    for (int c = 0; c < chunks; ++c) {
        const float2 p = part[(b * chunks + c) * m + col];
        acc.x += p.x;
        acc.y += p.y;
    }
    cinv[idx] = acc;
}

// lambda_i = (sum_k P G - sum_k P mu_k) / max(sum_k P, 1e-12).  Warp per row.
__global__ void __launch_bounds__(kRowThreads)
skb_row_iter_kernel(const float* __restrict__ P, const float2* __restrict__ rinv,
                    const float* __restrict__ mu, float* __restrict__ lam, int64_t rows,
                    int64_t n, int64_t m) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t row = int64_t(blockIdx.x) * kRowsPerCta + wid;
    if (row >= rows) return;
    const float* pr = P + row * m;
    const float* mb = mu + (row / n) * m;
    float acc = 0.0f;
    if (((m & 3) == 0) && aligned16(P) && aligned16(mu)) {
        const int64_t m4 = m >> 2;
        for (int64_t q = lane; q < m4; q += 32) {
            const float4 p = __ldg(reinterpret_cast<const float4*>(pr) + q);
            const float4 u = __ldg(reinterpret_cast<const float4*>(mb) + q);
            acc += p.x * u.x + p.y * u.y + p.z * u.z + p.w * u.w;
        }
    } else {
        for (int64_t j = lane; j < m; j += 32) acc += __ldg(pr + j) * __ldg(mb + j);
    }
    acc = warp_sum<32>(acc);
    if (lane == 0) {
        const float2 ri = rinv[row];
        lam[row] = (ri.x - acc) / fmaxf(ri.y, kSumFloor);
    }
}

// Column mat-vec over a row chunk: sum_i P_ik lambda_i; grid (ceil(m/128), chunks, B).
__global__ void __launch_bounds__(kColWarps * 32)
skb_col_iter_kernel(const float* __restrict__ P, const float* __restrict__ lam,
                    const float2* __restrict__ cinv, float* __restrict__ mu,
                    float* __restrict__ part, int64_t n, int64_t m, int64_t rows_per_chunk,
                    int chunks, int64_t b0) {
    __shared__ float sm[kColWarps][kColTile];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t b = b0 + blockIdx.z, chunk = blockIdx.y;
    const int64_t cbase = int64_t(blockIdx.x) * kColTile;
    const int64_t r0 = chunk * rows_per_chunk, r1 = min(n, r0 + rows_per_chunk);
    const float* Pb = P + b * n * m;
    const float* lb = lam + b * n;
    float acc[4] = {0, 0, 0, 0};
    const bool vec = ((m & 3) == 0) && aligned16(P);
    for (int64_t r = r0 + wid; r < r1; r += kColWarps * kColUnroll) {
#pragma unroll
        for (int u = 0; u < kColUnroll; ++u) {
            const int64_t rr = r + int64_t(u) * kColWarps;
            if (rr < r1) {
                const float l = __ldg(lb + rr);
                if (vec) {
                    const int64_t c0 = cbase + 4 * lane;
                    if (c0 < m) {
                        const float4 p = __ldg(reinterpret_cast<const float4*>(Pb + rr * m + c0));
                        acc[0] += p.x * l;
                        acc[1] += p.y * l;
                        acc[2] += p.z * l;
                        acc[3] += p.w * l;
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int64_t c = cbase + lane + 32 * k;
                        if (c < m) acc[k] += __ldg(Pb + rr * m + c) * l;
                    }
                }
            }
        }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) sm[wid][vec ? 4 * lane + k : lane + 32 * k] = acc[k];
    __syncthreads();
    if (threadIdx.x < kColTile) {
        const int ci = threadIdx.x;
        const int64_t col = cbase + ci;
        float s = sm[0][ci];
#pragma unroll
        for (int w = 1; w < kColWarps; ++w) s += sm[w][ci];
        if (col < m) {
            if (chunks == 1) {
                const float2 ci2 = cinv[b * m + col];
                mu[b * m + col] = (ci2.x - s) / fmaxf(ci2.y, kSumFloor);
            } else {
                part[(b * chunks + chunk) * m + col] = s;
            }
        }
    }
}

__global__ void skb_col_iter_merge_kernel(const float* __restrict__ part, const float2* __restrict__ cinv,
                                          float* __restrict__ mu, int64_t B, int64_t m, int chunks) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= B * m) return;
    const int64_t b = idx / m, col = idx - b * m;
    float s = 0.0f;
    for (int c = 0; c < chunks; ++c) s += part[(b * chunks + c) * m + col];
    const float2 ci2 = cinv[idx];
    mu[idx] = (ci2.x - s) / fmaxf(ci2.y, kSumFloor);
}

// Gradient epilogue, warp per row:
//   g = P (G - lambda_i - mu_k) / tau ;  grad_X = sign * g + grad_cost_b * P ;
//   tau_row[row] = sum_k g * log_alpha   (log_alpha = sign * X)
__global__ void __launch_bounds__(kRowThreads)
skb_final_kernel(const float* __restrict__ X, float sign, const float* __restrict__ P,
                 const float* __restrict__ gP, const float* __restrict__ gcost,
                 const float* __restrict__ lam, const float* __restrict__ mu, float tau,
                 float* __restrict__ gX, float* __restrict__ tau_row, int64_t rows, int64_t n,
                 int64_t m) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t row = int64_t(blockIdx.x) * kRowsPerCta + wid;
    if (row >= rows) return;
    const int64_t b = row / n;
    const float gc = gcost ? gcost[b] : 0.0f;
    const float l = lam[row];
    const float* mb = mu + b * m;
    float acc = 0.0f;
    const bool vec = (m & 3) == 0 && aligned16(X) && aligned16(P) && aligned16(gX) && aligned16(mu) &&
                     (gP == nullptr || aligned16(gP));
    if (vec) {   // four columns per lane per step, 16-byte accesses
        for (int64_t j = 4 * lane; j < m; j += 128) {
            const int64_t idx = row * m + j;
            const float4 x4 = __ldg(reinterpret_cast<const float4*>(X + idx));
            const float4 p4 = __ldg(reinterpret_cast<const float4*>(P + idx));
            const float4 m4 = __ldg(reinterpret_cast<const float4*>(mb + j));
            float4 g4 = make_float4(0, 0, 0, 0);
            if (gP != nullptr) g4 = __ldg(reinterpret_cast<const float4*>(gP + idx));
            const float xs[4] = {x4.x, x4.y, x4.z, x4.w}, ps[4] = {p4.x, p4.y, p4.z, p4.w};
            const float ms[4] = {m4.x, m4.y, m4.z, m4.w}, gs[4] = {g4.x, g4.y, g4.z, g4.w};
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float gt = __fmul_rn(gc, xs[e]);
                if (gP != nullptr) gt = __fadd_rn(gt, gs[e]);
                const float g = ps[e] * (gt - l - ms[e]) / tau;
                o[e] = __fadd_rn(sign * g, __fmul_rn(gc, ps[e]));
                acc += g * (sign * xs[e]);
            }
            *reinterpret_cast<float4*>(gX + idx) = make_float4(o[0], o[1], o[2], o[3]);
        }
    }
    for (int64_t j = vec ? m : lane; j < m; j += 32) {
        const int64_t idx = row * m + j;
        const float x = __ldg(X + idx);
        const float p = __ldg(P + idx);
        const float centred = grad_total(x, gc, gP, idx) - l - __ldg(mb + j);
        const float g = p * centred / tau;
        gX[idx] = __fadd_rn(sign * g, __fmul_rn(gc, p));
        acc += g * (sign * x);
    }
    if (tau_row != nullptr) {
        acc = warp_sum<32>(acc);
        if (lane == 0) tau_row[row] = acc;
    }
}

int64_t col_rows_per_chunk(int64_t n) {
    // ~512 rows per column chunk: long columns split across CTAs, short ones
    // finish in one CTA (and skip the merge kernel).
    return n <= 1024 ? n : 512;
}

}  // namespace

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

struct SkFwdWs {
    float2* part;
    float* delta;
    float* cost_row;
    int32_t* cnt;
    char* wide;       // wide-row cluster kernels' scratch
};

// Fused kernels are used when the shape allows it; the workspace covers
// either path (column partials sized for the larger of the two).
static SkFwdWs carve_fwd(Carve& c, int64_t B, int64_t n, int64_t m, int n_iters, float tol,
                         bool want_cost) {
    SkFwdWs w{};
    const int64_t chunks = ceil_div(n, col_rows_per_chunk(n));
    const int64_t fseg = sk_fused_shape_ok(B, n, m) ? sk_fused_plan(B, n, m, true).nseg
                         : sk_mid_shape_ok(B, n, m) ? sk_mid_plan(B, n, m, true).nseg : 1;
    const int64_t parts = std::max(chunks > 1 ? chunks : int64_t(0), fseg > 1 ? fseg : int64_t(0));
    w.part = parts > 0 ? c.take<float2>(size_t(B * parts * m)) : nullptr;
    w.delta = tol > 0.0f ? c.take<float>(size_t(n_iters > 0 ? n_iters : 1)) : nullptr;
    w.cost_row = want_cost ? c.take<float>(size_t(B * n)) : nullptr;
    w.cnt = c.take<int32_t>(size_t(B));
    const bool wide_shape = m >= 8192 && m <= 65536 && (m % 32) == 0 && tol == 0.0f;
    w.wide = wide_shape ? c.take<char>(sk_wide_ws(B, n, m)) : nullptr;
    return w;
}

size_t sk_stream_fwd_ws(int64_t B, int64_t n, int64_t m, int n_iters, float tol, bool want_cost) {
    Carve c(nullptr);
    carve_fwd(c, B, n, m, n_iters, tol, want_cost);
    return c.size();
}

int sk_stream_fwd(const SkFwdArgs& a, void* ws, cudaStream_t st) {
    Carve c(ws);
    SkFwdWs w = carve_fwd(c, a.B, a.n, a.m, a.n_iters, a.tol, a.cost != nullptr);
    const int64_t rows = a.B * a.n;
    const int64_t rpc = col_rows_per_chunk(a.n);
    const int chunks = int(ceil_div(a.n, rpc));
    const dim3 row_grid(unsigned(ceil_div(rows, kRowsPerCta)));
    const dim3 col_grid(unsigned(ceil_div(a.m, kColTile)), unsigned(chunks), unsigned(a.B));
    const unsigned merge_grid = unsigned(ceil_div(a.B * a.m, 256));

    cudaMemsetAsync(a.u2, 0, sizeof(float) * size_t(rows), st);
    cudaMemsetAsync(a.v2, 0, sizeof(float) * size_t(a.B * a.m), st);
    cudaMemsetAsync(a.status, 0, sizeof(int32_t) * 4, st);
    if (w.delta) cudaMemsetAsync(w.delta, 0, sizeof(float) * size_t(a.n_iters > 0 ? a.n_iters : 1), st);

    SkCtl ctl{w.delta, a.status, a.tol, 0};
    // the single-pass kernels read v (and write u) in 16-byte vectors
    const bool pots16 = ((reinterpret_cast<uintptr_t>(a.v2) | reinterpret_cast<uintptr_t>(a.u2)) & 15u) == 0;
    const bool fused = pots16 && sk_fused_supported(a.B, a.n, a.m, a.X);
    const bool mid = pots16 && !fused && sk_mid_supported(a.B, a.n, a.m, a.X);
    FusedPlan plan;
    if (fused || mid) {
        plan = fused ? sk_fused_plan(a.B, a.n, a.m, true) : sk_mid_plan(a.B, a.n, a.m, true);
        cudaMemsetAsync(w.cnt, 0, sizeof(int32_t) * size_t(a.B), st);
    }
    const bool wide =
        pots16 && !fused && !mid && a.tol == 0.0f && w.wide != nullptr && sk_wide_supported(a.B, a.n, a.m, a.X);
    if (wide) {
        int rc = sk_wide_fwd(a, w.wide, st);
        if (rc != DOT_OK) return rc;
    }
    const bool hist = a.u_hist != nullptr && a.v_hist != nullptr;
    auto record = [&](int it) {   // potentials after iteration it (unrolled backward)
        if (!hist) return;
        cudaMemcpyAsync(a.u_hist + int64_t(it) * rows, a.u2, sizeof(float) * size_t(rows), cudaMemcpyDeviceToDevice,
                        st);
        cudaMemcpyAsync(a.v_hist + int64_t(it) * a.B * a.m, a.v2, sizeof(float) * size_t(a.B * a.m),
                        cudaMemcpyDeviceToDevice, st);
    };
    if ((fused || mid) && a.n_iters > 0) {
        ProfScope ps(DOT_K_SK_FWD_ITER, st, a.n_iters);
        for (int it = 0; it < a.n_iters; ++it) {
            // a copy between two iterations ends the programmatic dependency chain
            if (fused) sk_fused_fwd_iter(a, plan, w.part, w.cnt, w.delta, it, it == 0 || hist, it == a.n_iters - 1, st);
            else sk_mid_fwd_iter(a, plan, w.part, w.cnt, w.delta, it, it == 0 || hist, it == a.n_iters - 1, st);
            record(it);
        }
    }
    for (int it = 0; it < (fused || mid || wide ? 0 : a.n_iters); ++it) {
        if (it > 0) record(it - 1);
        ctl.iter = it;
        {
            ProfScope ps(DOT_K_SK_FWD_ITER, st);
            sk_row_kernel<<<row_grid, kRowThreads, 0, st>>>(a.X, a.kinv, a.v2, a.la, a.la_def, a.u2,
                                                            rows, a.n, a.m, ctl);
        }
        {
            ProfScope ps(DOT_K_SK_FWD_ITER, st);
            for (int64_t b0 = 0; b0 < a.B; b0 += kMaxGridZ) {
                const dim3 gz(col_grid.x, col_grid.y, unsigned(std::min<int64_t>(kMaxGridZ, a.B - b0)));
                sk_col_kernel<<<gz, kColWarps * 32, 0, st>>>(a.X, a.kinv, a.u2, a.lb, a.lb_def, a.v2,
                                                                   w.part, a.n, a.m, rpc, chunks, ctl, nullptr, b0);
            }
        }
        if (chunks > 1) {
            ProfScope ps(DOT_K_SK_FWD_ITER, st);
            sk_col_merge_kernel<<<merge_grid, 256, 0, st>>>(w.part, a.lb, a.lb_def, a.v2, a.B, a.m,
                                                            chunks, ctl, nullptr);
        }
    }
    if (!fused && !mid && !wide && a.n_iters > 0) record(a.n_iters - 1);
    {
        ProfScope ps(DOT_K_SK_FWD_EPI, st);
        sk_status_kernel<<<1, 32, 0, st>>>(w.delta, a.status, a.n_iters, a.tol);
    }
    {
        ProfScope ps(DOT_K_SK_FWD_EPI, st);
        sk_plan_kernel<<<row_grid, kRowThreads, 0, st>>>(a.X, a.kinv, a.u2, a.v2, a.out, a.out_mode,
                                                          w.cost_row, rows, a.n, a.m);
    }
    if (a.cost != nullptr) {
        ProfScope ps(DOT_K_SK_FWD_EPI, st);
        sk_batch_sum_kernel<<<unsigned(ceil_div(a.B, 8)), 256, 0, st>>>(w.cost_row, a.cost, a.B, a.n, 1.0f);
    }
    return check_launch("sinkhorn forward (streaming)");
}

struct SkBwdWs {
    float2* rinv;
    float2* cinv;
    float* lam;
    float* mu;
    float2* part2;
    float* part1;
    float* tau_row;
    int32_t* cnt;     // [B] arrival counters, then one error word
};

static SkBwdWs carve_bwd(Carve& c, int64_t B, int64_t n, int64_t m) {
    SkBwdWs w{};
    const int64_t chunks = ceil_div(n, col_rows_per_chunk(n));
    const int64_t fseg = sk_fused_shape_ok(B, n, m) ? sk_fused_plan(B, n, m).nseg
                         : sk_mid_shape_ok(B, n, m) ? sk_mid_plan(B, n, m, false).nseg : 1;
    w.rinv = c.take<float2>(size_t(B * n));
    w.cinv = c.take<float2>(size_t(B * m));
    w.lam = c.take<float>(size_t(B * n));
    w.mu = c.take<float>(size_t(B * m));
    const int64_t p2 = std::max(chunks > 1 ? chunks : int64_t(0), fseg > 1 ? fseg : int64_t(0));
    w.part2 = p2 > 0 ? c.take<float2>(size_t(B * p2 * m)) : nullptr;
    const int64_t p1 = std::max(chunks > 1 ? chunks : int64_t(0), fseg > 1 ? fseg : int64_t(0));
    w.part1 = p1 > 0 ? c.take<float>(size_t(B * p1 * m)) : nullptr;
    w.tau_row = c.take<float>(size_t(B * n));
    w.cnt = c.take<int32_t>(size_t(B + 1));
    return w;
}

static bool aligned16_host(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

size_t sk_stream_bwd_ws(int64_t B, int64_t n, int64_t m) {
    Carve c(nullptr);
    carve_bwd(c, B, n, m);
    return c.size();
}

int sk_stream_bwd(const SkBwdArgs& a, void* ws, cudaStream_t st) {
    Carve c(ws);
    SkBwdWs w = carve_bwd(c, a.B, a.n, a.m);
    const int64_t rows = a.B * a.n;
    const int64_t rpc = col_rows_per_chunk(a.n);
    const int chunks = int(ceil_div(a.n, rpc));
    const dim3 row_grid(unsigned(ceil_div(rows, kRowsPerCta)));
    const dim3 col_grid(unsigned(ceil_div(a.m, kColTile)), unsigned(chunks), unsigned(a.B));
    const unsigned merge_grid = unsigned(ceil_div(a.B * a.m, 256));

    cudaMemsetAsync(w.mu, 0, sizeof(float) * size_t(a.B * a.m), st);
    cudaMemsetAsync(w.lam, 0, sizeof(float) * size_t(rows), st);
    const bool vec16 = aligned16_host(a.X) && (a.gP == nullptr || aligned16_host(a.gP));
    const bool fused = sk_fused_supported(a.B, a.n, a.m, a.P) && vec16;
    // mid-width rows: single-pass adjoint sweeps; the invariants below come
    // from the two-sweep set-up (once per call)
    const bool mid = !fused && vec16 && sk_mid_supported(a.B, a.n, a.m, a.P);
    FusedPlan plan;
    if (mid) {
        plan = sk_mid_plan(a.B, a.n, a.m, false);
        cudaMemsetAsync(w.cnt, 0, sizeof(int32_t) * size_t(a.B + 1), st);
    }
    if (fused) {
        plan = sk_fused_plan(a.B, a.n, a.m);
        cudaMemsetAsync(w.cnt, 0, sizeof(int32_t) * size_t(a.B + 1), st);
        // invariants in one sweep over P and X on the iterations' schedule
        ProfScope ps(DOT_K_SK_BWD_EPI, st);
        sk_fused_bwd_prep(a, plan, w.rinv, w.cinv, w.part2, w.cnt, st);
    } else {
        {
            ProfScope ps(DOT_K_SK_BWD_EPI, st);
            skb_row_prep_kernel<<<row_grid, kRowThreads, 0, st>>>(a.X, a.P, a.gP, a.gcost, w.rinv, rows, a.n, a.m);
        }
        {
            ProfScope ps(DOT_K_SK_BWD_EPI, st);
            for (int64_t b0 = 0; b0 < a.B; b0 += kMaxGridZ) {
                const dim3 gz(col_grid.x, col_grid.y, unsigned(std::min<int64_t>(kMaxGridZ, a.B - b0)));
                skb_col_prep_kernel<<<gz, kColWarps * 32, 0, st>>>(a.X, a.P, a.gP, a.gcost, w.cinv, w.part2,
                                                                         a.n, a.m, rpc, chunks, b0);
            }
        }
        if (chunks > 1) {
            ProfScope ps(DOT_K_SK_BWD_EPI, st);
            skb_col_prep_merge_kernel<<<merge_grid, 256, 0, st>>>(w.part2, w.cinv, a.B, a.m, chunks);
        }
    }
    if ((fused || mid) && a.bwd_iters > 0) {
        ProfScope ps(DOT_K_SK_BWD_ITER, st, a.bwd_iters);
        for (int it = 0; it < a.bwd_iters; ++it) {
            if (fused)
                sk_fused_bwd_iter(a, plan, w.rinv, w.cinv, w.lam, w.mu, w.part1, w.cnt, w.cnt + a.B, it == 0,
                                  it == a.bwd_iters - 1, st);
            else
                sk_mid_bwd_iter(a, plan, w.rinv, w.cinv, w.lam, w.mu, w.part1, w.cnt, w.cnt + a.B, it == 0,
                                it == a.bwd_iters - 1, st);
        }
    }
    for (int it = 0; it < (fused || mid ? 0 : a.bwd_iters); ++it) {
        {
            ProfScope ps(DOT_K_SK_BWD_ITER, st);
            skb_row_iter_kernel<<<row_grid, kRowThreads, 0, st>>>(a.P, w.rinv, w.mu, w.lam, rows, a.n, a.m);
        }
        {
            ProfScope ps(DOT_K_SK_BWD_ITER, st);
            for (int64_t b0 = 0; b0 < a.B; b0 += kMaxGridZ) {
                const dim3 gz(col_grid.x, col_grid.y, unsigned(std::min<int64_t>(kMaxGridZ, a.B - b0)));
                skb_col_iter_kernel<<<gz, kColWarps * 32, 0, st>>>(a.P, w.lam, w.cinv, w.mu, w.part1,
                                                                         a.n, a.m, rpc, chunks, b0);
            }
        }
        if (chunks > 1) {
            ProfScope ps(DOT_K_SK_BWD_ITER, st);
            skb_col_iter_merge_kernel<<<merge_grid, 256, 0, st>>>(w.part1, w.cinv, w.mu, a.B, a.m, chunks);
        }
    }
    {
        ProfScope ps(DOT_K_SK_BWD_EPI, st);
        skb_final_kernel<<<row_grid, kRowThreads, 0, st>>>(a.X, a.sign, a.P, a.gP, a.gcost, w.lam, w.mu,
                                                            a.tau, a.gX, a.gtau ? w.tau_row : nullptr,
                                                            rows, a.n, a.m);
    }
    if (a.gtau != nullptr) {
        ProfScope ps(DOT_K_SK_BWD_EPI, st);
        sk_batch_sum_kernel<<<unsigned(ceil_div(a.B, 8)), 256, 0, st>>>(w.tau_row, a.gtau, a.B, a.n,
                                                                        -1.0f / a.tau);
    }
    return check_launch("sinkhorn backward (streaming)");
}


// ---------------------------------------------------------------------------
// split half-steps for row-sharded problems (host combines column partials
// across shards between them)
// ---------------------------------------------------------------------------

int sk_split_rows(const float* X, float kinv, const float* la, float la_def, int64_t B, int64_t n, int64_t m,
                  const float* v2, float* u2, cudaStream_t st) {
    const int64_t rows = B * n;
    SkCtl ctl{nullptr, nullptr, 0.0f, 0};
    ProfScope ps(DOT_K_SK_FWD_ITER, st);
    sk_row_kernel<<<unsigned(ceil_div(rows, kRowsPerCta)), kRowThreads, 0, st>>>(X, kinv, v2, la, la_def, u2, rows,
                                                                                 n, m, ctl);
    return check_launch("sinkhorn row half-step");
}

size_t sk_split_colpairs_ws(int64_t B, int64_t n, int64_t m) {
    Carve c(nullptr);
    const int64_t chunks = ceil_div(n, col_rows_per_chunk(n));
    if (chunks > 1) c.take<float2>(size_t(B * chunks * m));
    return c.size();
}

int sk_split_colpairs(const float* X, float kinv, const float* u2, int64_t B, int64_t n, int64_t m, float2* pairs,
                      void* ws, cudaStream_t st) {
    Carve c(ws);
    const int64_t rpc = col_rows_per_chunk(n);
    const int chunks = int(ceil_div(n, rpc));
    float2* part = chunks > 1 ? c.take<float2>(size_t(B * chunks * m)) : nullptr;
    SkCtl ctl{nullptr, nullptr, 0.0f, 0};
    const dim3 col_grid(unsigned(ceil_div(m, kColTile)), unsigned(chunks), unsigned(B));
    {
        ProfScope ps(DOT_K_SK_FWD_ITER, st);
        for (int64_t b0 = 0; b0 < B; b0 += kMaxGridZ) {
            const dim3 gz(col_grid.x, col_grid.y, unsigned(std::min<int64_t>(kMaxGridZ, B - b0)));
            sk_col_kernel<<<gz, kColWarps * 32, 0, st>>>(X, kinv, u2, nullptr, 0.0f, nullptr, part, n, m, rpc,
                                                               chunks, ctl, pairs, b0);
        }
    }
    if (chunks > 1) {
        ProfScope ps(DOT_K_SK_FWD_ITER, st);
        sk_col_merge_kernel<<<unsigned(ceil_div(B * m, 256)), 256, 0, st>>>(part, nullptr, 0.0f, nullptr, B, m,
                                                                            chunks, ctl, pairs);
    }
    return check_launch("sinkhorn column pairs");
}

int sk_split_pair_merge(const float2* pairs, int parts, const float* lb, float lb_def, int64_t B, int64_t m,
                        float* v2, cudaStream_t st) {
    // the shards' pairs laid out [parts][B*m] are the chunk partials of one
    // problem: merge them in shard order exactly as the chunk merge does
    ProfScope ps(DOT_K_SK_EXCHANGE, st);
    sk_shard_merge_kernel<<<unsigned(ceil_div(B * m, 256)), 256, 0, st>>>(pairs, parts, lb, lb_def, v2, B * m);
    return check_launch("sinkhorn shard merge");
}

size_t sk_split_plan_ws(int64_t B, int64_t n) {
    Carve c(nullptr);
    c.take<float>(size_t(B * n));
    return c.size();
}

int sk_split_plan(const float* X, float kinv, const float* u2, const float* v2, int64_t B, int64_t n, int64_t m,
                  int out_mode, float* out, float* cost, void* ws, cudaStream_t st) {
    Carve c(ws);
    float* cost_row = cost ? c.take<float>(size_t(B * n)) : nullptr;
    const int64_t rows = B * n;
    {
        ProfScope ps(DOT_K_SK_FWD_EPI, st);
        sk_plan_kernel<<<unsigned(ceil_div(rows, kRowsPerCta)), kRowThreads, 0, st>>>(X, kinv, u2, v2, out, out_mode,
                                                                                      cost_row, rows, n, m);
    }
    if (cost != nullptr) {
        ProfScope ps(DOT_K_SK_FWD_EPI, st);
        sk_batch_sum_kernel<<<unsigned(ceil_div(B, 8)), 256, 0, st>>>(cost_row, cost, B, n, 1.0f);
    }
    return check_launch("sinkhorn plan");
}

}  // namespace dotb

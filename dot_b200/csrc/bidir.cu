// Bidirectional softmax, forward and backward (any B, L1, L2; fp32 or bf16
// input read natively, fp32 arithmetic).
//
// out_ij = sqrt(1e-9 + row_ij * col_ij) inside each batch's length window,
// row = softmax over j of sim/T, col = softmax over i of sim/T
// (reference: src/bidirectional_softmax/kernels_cpu.cpp:41-143, CUDA
// kernels.cu:90-242).  Instead of the reference's two full-size softmax
// buffers (and its three full-size backward workspaces, torch_cuda.cpp:107-110)
// only per-row and per-column (max, 1/sum) statistics are stored; every pass
// recomputes row/col/out from sim and the statistics with the same
// expressions, so the backward sees bit-identical values.  The backward writes
// each gradient element once (no atomics, deterministic), where the reference
// accumulates row and column terms with atomicAdd (kernels.cu:277-361).
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace dotb {

namespace {

constexpr int kThreads = 256;
constexpr int kRowsPerCta = kThreads / 32;
constexpr int kColWarps = 8;
constexpr int kColTile = 128;

template <typename T>
__device__ __forceinline__ float ld(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld<float>(const float* p, int64_t i) { return __ldg(p + i); }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
    return __bfloat162float(p[i]);
}

// exp with the reference's clamp (kernels_cpu.cpp:31-35), natural base.
__device__ __forceinline__ float exp88(float x) {
    if (x < -88.0f) return 0.0f;
    return expf(fminf(x, 88.0f));
}

__device__ __forceinline__ void window(const int32_t* lengths, int64_t b, int64_t L1, int64_t L2,
                                       int64_t& l1, int64_t& l2) {
    l1 = min(max(int64_t(lengths[2 * b]), int64_t(0)), L1);
    l2 = min(max(int64_t(lengths[2 * b + 1]), int64_t(0)), L2);
}

struct Probs {
    float row, col, out;
};

// row/col softmax values and the output at one element (same expressions in
// every pass).  sim/T is rounded before the max is subtracted, as the
// reference computes it (kernels_cpu.cpp:72-77), so the row/column maximum
// gives exactly exp(0) = 1 (an FMA-contracted s*invT - max would not).
__device__ __forceinline__ Probs probs(float s, float invT, float2 rs, float2 cs) {
    const float val = __fmul_rn(s, invT);
    Probs p;
    p.row = exp88(val - rs.x) * rs.y;
    p.col = exp88(val - cs.x) * cs.y;
    p.out = sqrtf(__fadd_rn(1e-9f, __fmul_rn(p.row, p.col)));
    return p;
}

// ---- forward: row statistics, warp per row, max pass then sum pass ---------
template <typename T>
__global__ void __launch_bounds__(kThreads)
bs_row_stats_kernel(const T* __restrict__ sim, const int32_t* __restrict__ lengths, int64_t B,
                    int64_t L1, int64_t L2, float invT, float2* __restrict__ rstat) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t row = int64_t(blockIdx.x) * kRowsPerCta + wid;
    if (row >= B * L1) return;
    const int64_t b = row / L1, i = row - b * L1;
    int64_t l1, l2;
    window(lengths, b, L1, L2, l1, l2);
    if (i >= l1) {
        if (lane == 0) rstat[row] = make_float2(0.0f, 0.0f);
        return;
    }
    const T* sr = sim + row * L2;
    float mx = kNegBig;
    for (int64_t j = lane; j < l2; j += 32) mx = fmaxf(mx, __fmul_rn(ld(sr, j), invT));
    mx = warp_max<32>(mx);
    float s = 0.0f;
    for (int64_t j = lane; j < l2; j += 32) s += exp88(__fmul_rn(ld(sr, j), invT) - mx);
    s = warp_sum<32>(s);
    if (lane == 0) rstat[row] = make_float2(mx, s > 0.0f ? 1.0f / s : 0.0f);
}

// ---- forward: column statistics over a row chunk (online max/sum) ---------
// grid (ceil(L2/128), chunks, B)
template <typename T>
__global__ void __launch_bounds__(kColWarps * 32)
bs_col_stats_kernel(const T* __restrict__ sim, const int32_t* __restrict__ lengths, int64_t L1,
                    int64_t L2, float invT, int64_t rows_per_chunk, int chunks,
                    float2* __restrict__ cstat, float2* __restrict__ part, int64_t b0) {
    __shared__ float sm_M[kColWarps][kColTile];
    __shared__ float sm_S[kColWarps][kColTile];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t b = b0 + blockIdx.z, chunk = blockIdx.y;
    const int64_t cbase = int64_t(blockIdx.x) * kColTile;
    int64_t l1, l2;
    window(lengths, b, L1, L2, l1, l2);
    const int64_t r0 = chunk * rows_per_chunk, r1 = min(l1, r0 + rows_per_chunk);
    const T* sb = sim + b * L1 * L2;
    float M[4], S[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) { M[k] = kNegBig; S[k] = 0.0f; }
    for (int64_t r = r0 + wid; r < r1; r += kColWarps) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int64_t c = cbase + lane + 32 * k;
            if (c < l2) {
                const float val = __fmul_rn(ld(sb, r * L2 + c), invT);
                if (val > M[k]) {
                    S[k] *= exp88(M[k] - val);
                    M[k] = val;
                }
                S[k] += exp88(val - M[k]);
            }
        }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        sm_M[wid][lane + 32 * k] = M[k];
        sm_S[wid][lane + 32 * k] = S[k];
    }
    __syncthreads();
    if (threadIdx.x < kColTile) {
        const int ci = threadIdx.x;
        const int64_t col = cbase + ci;
        float mm = kNegBig;
#pragma unroll
        for (int w = 0; w < kColWarps; ++w) mm = fmaxf(mm, sm_M[w][ci]);
        float ss = 0.0f;
#pragma unroll
        for (int w = 0; w < kColWarps; ++w) ss += sm_S[w][ci] * exp88(sm_M[w][ci] - mm);
        if (col < L2) {
            if (chunks == 1) cstat[b * L2 + col] = make_float2(mm, ss > 0.0f ? 1.0f / ss : 0.0f);
            else part[(b * chunks + chunk) * L2 + col] = make_float2(mm, ss);
        }
    }
}

__global__ void bs_col_merge_kernel(const float2* __restrict__ part, float2* __restrict__ cstat,
                                    int64_t B, int64_t L2, int chunks) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= B * L2) return;
    const int64_t b = idx / L2, col = idx - b * L2;
    float mm = kNegBig;
    for (int c = 0; c < chunks; ++c) mm = fmaxf(mm, part[(b * chunks + c) * L2 + col].x);
    float ss = 0.0f;
    for (int c = 0; c < chunks; ++c) {
        const float2 p = part[(b * chunks + c) * L2 + col];
        ss += p.y * exp88(p.x - mm);
    }
    cstat[idx] = make_float2(mm, ss > 0.0f ? 1.0f / ss : 0.0f);
}

// ---- forward: output, warp per row ----------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads)
bs_out_kernel(const T* __restrict__ sim, const int32_t* __restrict__ lengths, int64_t B, int64_t L1,
              int64_t L2, float invT, const float2* __restrict__ rstat,
              const float2* __restrict__ cstat, float* __restrict__ out) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t row = int64_t(blockIdx.x) * kRowsPerCta + wid;
    if (row >= B * L1) return;
    const int64_t b = row / L1, i = row - b * L1;
    int64_t l1, l2;
    window(lengths, b, L1, L2, l1, l2);
    const T* sr = sim + row * L2;
    float* orow = out + row * L2;
    const float2 rs = rstat[row];
    const float2* cb = cstat + b * L2;
    for (int64_t j = lane; j < L2; j += 32) {
        float o = 0.0f;
        if (i < l1 && j < l2) o = probs(ld(sr, j), invT, rs, cb[j]).out;
        orow[j] = o;
    }
}

// ---- backward ---------------------------------------------------------------
struct BwdTerms {
    float row, col, d_row, d_col;
};

__device__ __forceinline__ BwdTerms bwd_terms(float s, float g, float invT, float2 rs, float2 cs) {
    const Probs p = probs(s, invT, rs, cs);
    const float dp = p.out > 1e-9f ? g * 0.5f / p.out : 0.0f;
    return BwdTerms{p.row, p.col, dp * p.col, dp * p.row};
}

// row dots: sum_j d_row * row.  Warp per row.
template <typename T>
__global__ void __launch_bounds__(kThreads)
bs_bwd_rowdot_kernel(const T* __restrict__ sim, const float* __restrict__ gout,
                     const int32_t* __restrict__ lengths, int64_t B, int64_t L1, int64_t L2,
                     float invT, const float2* __restrict__ rstat, const float2* __restrict__ cstat,
                     float* __restrict__ rdot) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t row = int64_t(blockIdx.x) * kRowsPerCta + wid;
    if (row >= B * L1) return;
    const int64_t b = row / L1, i = row - b * L1;
    int64_t l1, l2;
    window(lengths, b, L1, L2, l1, l2);
    float acc = 0.0f;
    if (i < l1) {
        const float2 rs = rstat[row];
        const float2* cb = cstat + b * L2;
        for (int64_t j = lane; j < l2; j += 32) {
            const BwdTerms t = bwd_terms(ld(sim, row * L2 + j), __ldg(gout + row * L2 + j), invT, rs, cb[j]);
            acc += t.d_row * t.row;
        }
    }
    acc = warp_sum<32>(acc);
    if (lane == 0) rdot[row] = acc;
}

// column dots: sum_i d_col * col over a row chunk; grid (ceil(L2/128), chunks, B)
template <typename T>
__global__ void __launch_bounds__(kColWarps * 32)
bs_bwd_coldot_kernel(const T* __restrict__ sim, const float* __restrict__ gout,
                     const int32_t* __restrict__ lengths, int64_t L1, int64_t L2, float invT,
                     const float2* __restrict__ rstat, const float2* __restrict__ cstat,
                     int64_t rows_per_chunk, int chunks, float* __restrict__ cdot,
                     float* __restrict__ part, int64_t b0) {
    __shared__ float sm[kColWarps][kColTile];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t b = b0 + blockIdx.z, chunk = blockIdx.y;
    const int64_t cbase = int64_t(blockIdx.x) * kColTile;
    int64_t l1, l2;
    window(lengths, b, L1, L2, l1, l2);
    const int64_t r0 = chunk * rows_per_chunk, r1 = min(l1, r0 + rows_per_chunk);
    float acc[4] = {0, 0, 0, 0};
    float2 cs[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int64_t c = cbase + lane + 32 * k;
        cs[k] = c < L2 ? cstat[b * L2 + c] : make_float2(0.0f, 0.0f);
    }
    for (int64_t r = r0 + wid; r < r1; r += kColWarps) {
        const float2 rs = rstat[b * L1 + r];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int64_t c = cbase + lane + 32 * k;
            if (c < l2) {
                const int64_t idx = (b * L1 + r) * L2 + c;
                const BwdTerms t = bwd_terms(ld(sim, idx), __ldg(gout + idx), invT, rs, cs[k]);
                acc[k] += t.d_col * t.col;
            }
        }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) sm[wid][lane + 32 * k] = acc[k];
    __syncthreads();
    if (threadIdx.x < kColTile) {
        const int ci = threadIdx.x;
        const int64_t col = cbase + ci;
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < kColWarps; ++w) s += sm[w][ci];
        if (col < L2) {
            if (chunks == 1) cdot[b * L2 + col] = s;
            else part[(b * chunks + chunk) * L2 + col] = s;
        }
    }
}

__global__ void bs_sum_merge_kernel(const float* __restrict__ part, float* __restrict__ dst,
                                    int64_t B, int64_t L2, int chunks) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= B * L2) return;
    const int64_t b = idx / L2, col = idx - b * L2;
    float s = 0.0f;
    for (int c = 0; c < chunks; ++c) s += part[(b * chunks + c) * L2 + col];
    dst[idx] = s;
}

template <typename T>
__device__ __forceinline__ void st_grad(T* p, int64_t i, float v);
template <>
__device__ __forceinline__ void st_grad<float>(float* p, int64_t i, float v) { p[i] = v; }
template <>
__device__ __forceinline__ void st_grad<__nv_bfloat16>(__nv_bfloat16* p, int64_t i, float v) {
    p[i] = __float2bfloat16_rn(v);
}

// gradient, warp per row; also per-row partial of sum grad * sim * invT.
template <typename T, typename G>
__global__ void __launch_bounds__(kThreads)
bs_bwd_grad_kernel(const T* __restrict__ sim, const float* __restrict__ gout,
                   const int32_t* __restrict__ lengths, int64_t B, int64_t L1, int64_t L2,
                   float invT, const float2* __restrict__ rstat, const float2* __restrict__ cstat,
                   const float* __restrict__ rdot, const float* __restrict__ cdot,
                   G* __restrict__ gsim, float* __restrict__ tau_row) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t row = int64_t(blockIdx.x) * kRowsPerCta + wid;
    if (row >= B * L1) return;
    const int64_t b = row / L1, i = row - b * L1;
    int64_t l1, l2;
    window(lengths, b, L1, L2, l1, l2);
    const float2 rs = rstat[row];
    const float rd = rdot[row];
    float acc = 0.0f;
    for (int64_t j = lane; j < L2; j += 32) {
        const int64_t idx = row * L2 + j;
        float g = 0.0f;
        if (i < l1 && j < l2) {
            const float s = ld(sim, idx);
            const BwdTerms t = bwd_terms(s, __ldg(gout + idx), invT, rs, cstat[b * L2 + j]);
            const float a = __fmul_rn(__fmul_rn(t.d_row - rd, t.row), invT);
            const float c = __fmul_rn(__fmul_rn(t.d_col - cdot[b * L2 + j], t.col), invT);
            g = __fadd_rn(a, c);
            acc += g * s * invT;
        }
        st_grad<G>(gsim, idx, g);
    }
    if (tau_row != nullptr) {
        acc = warp_sum<32>(acc);
        if (lane == 0) tau_row[row] = acc;
    }
}

__global__ void bs_batch_sum_kernel(const float* __restrict__ row_part, float* __restrict__ outv,
                                    int64_t B, int64_t n, float scale) {
    const int lane = threadIdx.x & 31;
    const int64_t b = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= B) return;
    float acc = 0.0f;
    for (int64_t i = lane; i < n; i += 32) acc += row_part[b * n + i];
    acc = warp_sum<32>(acc);
    if (lane == 0) outv[b] = acc * scale;
}

int64_t bs_rows_per_chunk(int64_t L1) { return L1 <= 1024 ? L1 : 512; }

struct BsFwdWs {
    float2* part;
};
struct BsBwdWs {
    float* rdot;
    float* cdot;
    float* part;
    float* tau_row;
};

BsFwdWs carve_bs_fwd(Carve& c, int64_t B, int64_t L1, int64_t L2) {
    const int64_t chunks = ceil_div(L1, bs_rows_per_chunk(L1));
    BsFwdWs w{};
    w.part = chunks > 1 ? c.take<float2>(size_t(B * chunks * L2)) : nullptr;
    return w;
}
BsBwdWs carve_bs_bwd(Carve& c, int64_t B, int64_t L1, int64_t L2) {
    const int64_t chunks = ceil_div(L1, bs_rows_per_chunk(L1));
    BsBwdWs w{};
    w.rdot = c.take<float>(size_t(B * L1));
    w.cdot = c.take<float>(size_t(B * L2));
    w.part = chunks > 1 ? c.take<float>(size_t(B * chunks * L2)) : nullptr;
    w.tau_row = c.take<float>(size_t(B * L1));
    return w;
}

template <typename T>
int bs_fwd_impl(const T* sim, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau,
                float* out, float2* rstat, float2* cstat, void* ws, cudaStream_t st) {
    Carve c(ws);
    BsFwdWs w = carve_bs_fwd(c, B, L1, L2);
    const float invT = 1.0f / tau;
    const int64_t rpc = bs_rows_per_chunk(L1);
    const int chunks = int(ceil_div(L1, rpc));
    const unsigned row_grid = unsigned(ceil_div(B * L1, kRowsPerCta));
    {
        ProfScope ps(DOT_K_BS_FWD, st);
        bs_row_stats_kernel<T><<<row_grid, kThreads, 0, st>>>(sim, lengths, B, L1, L2, invT, rstat);
    }
    {
        ProfScope ps(DOT_K_BS_FWD, st);
        for (int64_t b0 = 0; b0 < B; b0 += kMaxGridZ) {
            const dim3 g(unsigned(ceil_div(L2, kColTile)), unsigned(chunks), unsigned(std::min<int64_t>(kMaxGridZ, B - b0)));
            bs_col_stats_kernel<T><<<g, kColWarps * 32, 0, st>>>(sim, lengths, L1, L2, invT, rpc, chunks, cstat,
                                                                 w.part, b0);
        }
    }
    if (chunks > 1) {
        ProfScope ps(DOT_K_BS_FWD, st);
        bs_col_merge_kernel<<<unsigned(ceil_div(B * L2, 256)), 256, 0, st>>>(w.part, cstat, B, L2, chunks);
    }
    {
        ProfScope ps(DOT_K_BS_FWD, st);
        bs_out_kernel<T><<<row_grid, kThreads, 0, st>>>(sim, lengths, B, L1, L2, invT, rstat, cstat, out);
    }
    return check_launch("bidirectional softmax forward");
}

template <typename T, typename G>
int bs_bwd_impl(const T* sim, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau,
                const float2* rstat, const float2* cstat, const float* gout, G* gsim, float* gtau,
                void* ws, cudaStream_t st) {
    Carve c(ws);
    BsBwdWs w = carve_bs_bwd(c, B, L1, L2);
    const float invT = 1.0f / tau;
    const int64_t rpc = bs_rows_per_chunk(L1);
    const int chunks = int(ceil_div(L1, rpc));
    const unsigned row_grid = unsigned(ceil_div(B * L1, kRowsPerCta));
    {
        ProfScope ps(DOT_K_BS_BWD, st);
        bs_bwd_rowdot_kernel<T><<<row_grid, kThreads, 0, st>>>(sim, gout, lengths, B, L1, L2, invT, rstat,
                                                               cstat, w.rdot);
    }
    {
        ProfScope ps(DOT_K_BS_BWD, st);
        for (int64_t b0 = 0; b0 < B; b0 += kMaxGridZ) {
            const dim3 g(unsigned(ceil_div(L2, kColTile)), unsigned(chunks), unsigned(std::min<int64_t>(kMaxGridZ, B - b0)));
            bs_bwd_coldot_kernel<T><<<g, kColWarps * 32, 0, st>>>(sim, gout, lengths, L1, L2, invT, rstat, cstat,
                                                                  rpc, chunks, w.cdot, w.part, b0);
        }
    }
    if (chunks > 1) {
        ProfScope ps(DOT_K_BS_BWD, st);
        bs_sum_merge_kernel<<<unsigned(ceil_div(B * L2, 256)), 256, 0, st>>>(w.part, w.cdot, B, L2, chunks);
    }
    {
        ProfScope ps(DOT_K_BS_BWD, st);
        bs_bwd_grad_kernel<T, G><<<row_grid, kThreads, 0, st>>>(sim, gout, lengths, B, L1, L2, invT, rstat,
                                                                cstat, w.rdot, w.cdot, gsim,
                                                                gtau ? w.tau_row : nullptr);
    }
    if (gtau != nullptr) {
        ProfScope ps(DOT_K_BS_BWD, st);
        bs_batch_sum_kernel<<<unsigned(ceil_div(B, 8)), 256, 0, st>>>(w.tau_row, gtau, B, L1, -1.0f);
    }
    return check_launch("bidirectional softmax backward");
}

}  // namespace

// streaming sweeps (bidir_stream.cu) for L2 <= 1024, L2 % 4 == 0
bool bsf_supported(int64_t B, int64_t L1, int64_t L2, int dtype, const void* sim, const void* gout, const void* dst,
                   int dst_dtype);
size_t bsf_fwd_ws(int64_t B, int64_t L1, int64_t L2);
inline bool aligned16_host(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
size_t bsf_bwd_ws(int64_t B, int64_t L1, int64_t L2);
int bsf_fwd(const void* sim, int dtype, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau,
            float* out, float* row_stats, float* col_stats, void* ws, cudaStream_t st);
int bsf_bwd(const void* sim, int dtype, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau,
            const float* row_stats, const float* col_stats, const float* gout, void* gsim, int gdtype, float* gtau,
            void* ws, cudaStream_t st);

size_t bs_fwd_ws(int64_t B, int64_t L1, int64_t L2) {
    Carve c(nullptr);
    carve_bs_fwd(c, B, L1, L2);
    return std::max(c.size(), bsf_fwd_ws(B, L1, L2));
}

size_t bs_bwd_ws(int64_t B, int64_t L1, int64_t L2) {
    Carve c(nullptr);
    carve_bs_bwd(c, B, L1, L2);
    return std::max(c.size(), bsf_bwd_ws(B, L1, L2));
}

int bs_fwd(const void* sim, int dtype, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2,
           float tau, float* out, float* row_stats, float* col_stats, void* ws, cudaStream_t st) {
    // the fused kernels read the statistics as float4
    const bool stats16 = aligned16_host(row_stats) && aligned16_host(col_stats);
    if (stats16 && bsf_supported(B, L1, L2, dtype, sim, nullptr, out, DOT_F32))
        return bsf_fwd(sim, dtype, lengths, B, L1, L2, tau, out, row_stats, col_stats, ws, st);
    float2* rs = reinterpret_cast<float2*>(row_stats);
    float2* cs = reinterpret_cast<float2*>(col_stats);
    if (dtype == DOT_F32)
        return bs_fwd_impl(static_cast<const float*>(sim), lengths, B, L1, L2, tau, out, rs, cs, ws, st);
    return bs_fwd_impl(static_cast<const __nv_bfloat16*>(sim), lengths, B, L1, L2, tau, out, rs, cs, ws, st);
}

int bs_bwd(const void* sim, int dtype, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau,
           const float* row_stats, const float* col_stats, const float* gout, void* gsim, int gdtype,
           float* gtau, void* ws, cudaStream_t st) {
    const bool stats16 = aligned16_host(row_stats) && aligned16_host(col_stats);
    if (stats16 && bsf_supported(B, L1, L2, dtype, sim, gout, gsim, gdtype))
        return bsf_bwd(sim, dtype, lengths, B, L1, L2, tau, row_stats, col_stats, gout, gsim, gdtype, gtau, ws, st);
    const float2* rs = reinterpret_cast<const float2*>(row_stats);
    const float2* cs = reinterpret_cast<const float2*>(col_stats);
    if (dtype == DOT_F32) {
        const float* s = static_cast<const float*>(sim);
        if (gdtype == DOT_F32)
            return bs_bwd_impl(s, lengths, B, L1, L2, tau, rs, cs, gout, static_cast<float*>(gsim), gtau, ws, st);
        return bs_bwd_impl(s, lengths, B, L1, L2, tau, rs, cs, gout, static_cast<__nv_bfloat16*>(gsim), gtau,
                           ws, st);
    }
    const __nv_bfloat16* s = static_cast<const __nv_bfloat16*>(sim);
    if (gdtype == DOT_F32)
        return bs_bwd_impl(s, lengths, B, L1, L2, tau, rs, cs, gout, static_cast<float*>(gsim), gtau, ws, st);
    return bs_bwd_impl(s, lengths, B, L1, L2, tau, rs, cs, gout, static_cast<__nv_bfloat16*>(gsim), gtau, ws,
                       st);
}

}  // namespace dotb

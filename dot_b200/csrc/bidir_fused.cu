// Bidirectional softmax, fused passes for rows that fit a warp's registers
// (L2 <= 1024, L2 % 4 == 0; fp32 or bf16 input).
//
//   forward  stats  one read of sim: row (max, 1/sum) exactly (max pass then
//                   sum pass over the row in registers) and column sums
//                   reusing the row exponentials -- exp(v_ij - A) =
//                   E_ij * exp(max_i - A) for a warp-wide reference A >= every
//                   row max -- merged over warps and row segments (last CTA
//                   of a batch, no waiting); a column whose merged sum is too
//                   small to trust is recomputed exactly from sim.
//            out    out_ij = sqrt(1e-9 + row_ij * col_ij), vectorised.
//   backward dots   one read of sim and grad_out: per-row dots
//                   sum_j d_row*row and per-column dots sum_i d_col*col.
//            grad   vectorised: grad = (d_row - rdot_i)*row/T + (d_col - cdot_j)*col/T.
// Formulas: src/bidirectional_softmax/kernels_cpu.cpp:41-232.  Column
// statistics use the reference A instead of the column maximum; any reference
// gives the same softmax (exp(v - A)/sum_i exp(v - A)); exponentials go
// through the SFU (ex2), about 1e-6 relative on the outputs.
#include <cuda_bf16.h>

#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace dotb {

namespace {

constexpr int kBT = 256;
constexpr int kBW = kBT / 32;
constexpr float kRaiseB = 60.0f;
constexpr float kTinyB = 8.077935669463161e-28f;   // 2^-90

// 4 consecutive values of sim as fp32.
__device__ __forceinline__ void ld4(const float* p, float (&v)[4]) {
    const float4 x = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = x.x;
    v[1] = x.y;
    v[2] = x.z;
    v[3] = x.w;
}
__device__ __forceinline__ void ld4(const __nv_bfloat16* p, float (&v)[4]) {
    const uint2 x = __ldg(reinterpret_cast<const uint2*>(p));
    v[0] = __uint_as_float(x.x << 16);
    v[1] = __uint_as_float(x.x & 0xffff0000u);
    v[2] = __uint_as_float(x.y << 16);
    v[3] = __uint_as_float(x.y & 0xffff0000u);
}
__device__ __forceinline__ void st4(float* p, const float (&v)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void st4(__nv_bfloat16* p, const float (&v)[4]) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
    const __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 x;
    x.x = *reinterpret_cast<const uint32_t*>(&a);
    x.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = x;
}

__device__ __forceinline__ void window(const int32_t* lengths, int64_t b, int64_t L1, int64_t L2, int64_t& l1,
                                       int64_t& l2) {
    l1 = min(max(int64_t(lengths[2 * b]), int64_t(0)), L1);
    l2 = min(max(int64_t(lengths[2 * b + 1]), int64_t(0)), L2);
}

struct BsfCommon {
    const int32_t* lengths;
    int64_t L1, L2;
    float invT;
    int64_t seg_rows;
    int nseg;
    int32_t* cnt;   // [B] arrival counters
};

__device__ __forceinline__ bool arrive_last_b(int32_t* cnt, int nseg, int* s_flag) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *s_flag = (atomicAdd(cnt + blockIdx.y, 1) == nseg - 1) ? 1 : 0;
    __syncthreads();
    const bool last = *s_flag != 0;
    if (last) __threadfence();
    return last;
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
// forward statistics
// ---------------------------------------------------------------------------
template <typename T, int VPL>
__global__ void __launch_bounds__(kBT, 2)
bsf_stats_kernel(const T* __restrict__ sim, BsfCommon c, float2* __restrict__ rstat, float2* __restrict__ cpart,
                 float2* __restrict__ cstat) {
    constexpr int NC = 4 * VPL;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int s_flag, s_nfix;
    __shared__ int s_fix[1024];
    float2* mrg = reinterpret_cast<float2*>(smem);   // [kBW][L2]
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int64_t b = blockIdx.y, L1 = c.L1, L2 = c.L2;
    int64_t l1, l2;
    window(c.lengths, b, L1, L2, l1, l2);
    const int64_t r0 = int64_t(blockIdx.x) * c.seg_rows, r1 = min(L1, r0 + c.seg_rows);
    const T* sb = sim + b * L1 * L2;
    if (tid == 0) s_nfix = 0;

    float S[NC];
#pragma unroll
    for (int e = 0; e < NC; ++e) S[e] = 0.0f;
    float A = kNegBig;
    for (int64_t i = r0 + wid; i < r1; i += kBW) {
        if (i >= l1 || l2 == 0) {
            if (lane == 0) rstat[b * L1 + i] = make_float2(0.0f, 0.0f);
            continue;
        }
        float t[NC];
#pragma unroll
        for (int p = 0; p < VPL; ++p) {
            const int64_t col = 4 * lane + 128 * p;
            float v[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            if (col < L2) {
                ld4(sb + i * L2 + col, v);
#pragma unroll
                for (int e = 0; e < 4; ++e) v[e] = (col + e < l2) ? __fmul_rn(v[e], c.invT) : -INFINITY;
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) t[4 * p + e] = v[e];
        }
        float mx = t[0];
#pragma unroll
        for (int e = 1; e < NC; ++e) mx = fmaxf(mx, t[e]);
        mx = warp_max<32>(mx);
#pragma unroll
        for (int e = 0; e < NC; ++e) t[e] = exp_shift(t[e] - mx);
        const float s = warp_sum<32>(tree_sum(t));
        if (lane == 0) rstat[b * L1 + i] = make_float2(mx, s > 0.0f ? 1.0f / s : 0.0f);
        if (mx > A + kRaiseB) {   // warp-uniform
            const float sc = exp_shift(A - mx);
#pragma unroll
            for (int e = 0; e < NC; ++e) S[e] *= sc;
            A = mx;
        }
        const float w = exp_shift(mx - A);
#pragma unroll
        for (int e = 0; e < NC; ++e) S[e] = fmaf(t[e], w, S[e]);
    }
#pragma unroll
    for (int p = 0; p < VPL; ++p) {
        const int64_t col = 4 * lane + 128 * p;
        if (col < L2) {
#pragma unroll
            for (int e = 0; e < 4; ++e) mrg[int64_t(wid) * L2 + col + e] = make_float2(A, S[4 * p + e]);
        }
    }
    __syncthreads();
    auto finish = [&](int64_t col, float mm, float ss) {
        if (col >= l2) {
            cstat[b * L2 + col] = make_float2(0.0f, 0.0f);
        } else if (ss < kTinyB) {
            s_fix[atomicAdd(&s_nfix, 1)] = int(col);
        } else {
            cstat[b * L2 + col] = make_float2(mm, 1.0f / ss);
        }
    };
    float2* mypart = cpart + (b * c.nseg + blockIdx.x) * L2;
    for (int64_t col = tid; col < L2; col += kBT) {
        float mm = kNegBig, ss = 0.0f;
#pragma unroll
        for (int w = 0; w < kBW; ++w) {
            const float2 q = mrg[int64_t(w) * L2 + col];
            lse_merge(mm, ss, q.x, q.y);
        }
        if (c.nseg == 1) finish(col, mm, ss);
        else mypart[col] = make_float2(mm, ss);
    }
    if (c.nseg > 1) {
        if (!arrive_last_b(c.cnt, c.nseg, &s_flag)) return;
        for (int64_t col = tid; col < L2; col += kBT) {
            float mm = kNegBig, ss = 0.0f;
            for (int sg = 0; sg < c.nseg; ++sg) {
                const float2 q = __ldcg(cpart + (b * c.nseg + sg) * L2 + col);
                lse_merge(mm, ss, q.x, q.y);
            }
            finish(col, mm, ss);
        }
        if (tid == 0) c.cnt[b] = 0;
    }
    __syncthreads();
    const int nfix = s_nfix;
    for (int k = wid; k < nfix; k += kBW) {
        const int64_t col = s_fix[k];
        const float2 st = exact_col_stats(sb, L2, l1, col, c.invT);
        if (lane == 0) cstat[b * L2 + col] = st;
    }
}

// Per-element softmax values from the statistics (the same expressions in
// every pass, so forward and backward see identical values).
struct BsVals {
    float row, col, out;
};
// The column value's numerator exp(v - A) and its share of the column sum
// (accumulated as E*w) can differ by an ulp, so row*col may exceed 1 by
// rounding where one element dominates its row and column; out is capped at 1,
// its exact-arithmetic bound.
__device__ __forceinline__ BsVals bs_vals(float val, float2 rs, float2 cs) {
    BsVals v;
    v.row = exp_shift(val - rs.x) * rs.y;
    v.col = exp_shift(val - cs.x) * cs.y;
    v.out = fminf(sqrtf(__fadd_rn(1e-9f, __fmul_rn(v.row, v.col))), 1.0f);
    return v;
}

// ---------------------------------------------------------------------------
// forward output, warp per row
// ---------------------------------------------------------------------------
template <typename T, int VPL>
__global__ void __launch_bounds__(kBT)
bsf_out_kernel(const T* __restrict__ sim, BsfCommon c, int64_t B, const float2* __restrict__ rstat,
               const float2* __restrict__ cstat, float* __restrict__ out) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t L1 = c.L1, L2 = c.L2;
    const int64_t row = int64_t(blockIdx.x) * kBW + wid;
    if (row >= B * L1) return;
    const int64_t b = row / L1, i = row - b * L1;
    int64_t l1, l2;
    window(c.lengths, b, L1, L2, l1, l2);
    const float2 rs = rstat[row];
    const float2* cb = cstat + b * L2;
#pragma unroll
    for (int p = 0; p < VPL; ++p) {
        const int64_t col = 4 * lane + 128 * p;
        if (col >= L2) continue;
        float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (i < l1 && col < l2) {
            float v[4];
            ld4(sim + row * L2 + col, v);
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (col + e < l2) o[e] = bs_vals(__fmul_rn(v[e], c.invT), rs, cb[col + e]).out;
        }
        st4(out + row * L2 + col, o);
    }
}

// ---------------------------------------------------------------------------
// backward dots: row dots sum_j d_row*row, column dots sum_i d_col*col
// ---------------------------------------------------------------------------
template <typename T, int VPL>
__global__ void __launch_bounds__(kBT, 2)
bsf_dots_kernel(const T* __restrict__ sim, const float* __restrict__ gout, BsfCommon c,
                const float2* __restrict__ rstat, const float2* __restrict__ cstat, float* __restrict__ rdot,
                float* __restrict__ cpart, float* __restrict__ cdot) {
    constexpr int NC = 4 * VPL;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int s_flag;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int64_t b = blockIdx.y, L1 = c.L1, L2 = c.L2;
    float2* cs = reinterpret_cast<float2*>(smem);               // [L2] column statistics
    float* mrg = reinterpret_cast<float*>(smem) + 2 * L2;       // [kBW][L2]
    int64_t l1, l2;
    window(c.lengths, b, L1, L2, l1, l2);
    const int64_t r0 = int64_t(blockIdx.x) * c.seg_rows, r1 = min(L1, r0 + c.seg_rows);
    const T* sb = sim + b * L1 * L2;
    const float* gb = gout + b * L1 * L2;
    for (int64_t col = tid; col < L2; col += kBT) cs[col] = cstat[b * L2 + col];
    __syncthreads();
    float C[NC];
#pragma unroll
    for (int e = 0; e < NC; ++e) C[e] = 0.0f;
    for (int64_t i = r0 + wid; i < r1; i += kBW) {
        float rd = 0.0f;
        if (i < l1) {
            const float2 rs = rstat[b * L1 + i];
#pragma unroll
            for (int p = 0; p < VPL; ++p) {
                const int64_t col = 4 * lane + 128 * p;
                if (col < l2) {
                    float v[4], g[4];
                    ld4(sb + i * L2 + col, v);
                    ld4(gb + i * L2 + col, g);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        if (col + e < l2) {
                            const BsVals q = bs_vals(__fmul_rn(v[e], c.invT), rs, cs[col + e]);
                            const float dp = q.out > 1e-9f ? g[e] * 0.5f / q.out : 0.0f;
                            rd += __fmul_rn(__fmul_rn(dp, q.col), q.row);
                            C[4 * p + e] += __fmul_rn(__fmul_rn(dp, q.row), q.col);
                        }
                    }
                }
            }
        }
        rd = warp_sum<32>(rd);
        if (lane == 0) rdot[b * L1 + i] = rd;
    }
#pragma unroll
    for (int p = 0; p < VPL; ++p) {
        const int64_t col = 4 * lane + 128 * p;
        if (col < L2) {
#pragma unroll
            for (int e = 0; e < 4; ++e) mrg[int64_t(wid) * L2 + col + e] = C[4 * p + e];
        }
    }
    __syncthreads();
    float* mypart = cpart + (b * c.nseg + blockIdx.x) * L2;
    for (int64_t col = tid; col < L2; col += kBT) {
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < kBW; ++w) s += mrg[int64_t(w) * L2 + col];
        if (c.nseg == 1) cdot[b * L2 + col] = s;
        else mypart[col] = s;
    }
    if (c.nseg == 1) return;
    if (!arrive_last_b(c.cnt, c.nseg, &s_flag)) return;
    for (int64_t col = tid; col < L2; col += kBT) {
        float s = 0.0f;
        for (int sg = 0; sg < c.nseg; ++sg) s += __ldcg(cpart + (b * c.nseg + sg) * L2 + col);
        cdot[b * L2 + col] = s;
    }
    if (tid == 0) c.cnt[b] = 0;
}

// ---------------------------------------------------------------------------
// backward gradient, warp per row
// ---------------------------------------------------------------------------
template <typename T, typename G, int VPL>
__global__ void __launch_bounds__(kBT)
bsf_grad_kernel(const T* __restrict__ sim, const float* __restrict__ gout, BsfCommon c, int64_t B,
                const float2* __restrict__ rstat, const float2* __restrict__ cstat, const float* __restrict__ rdot,
                const float* __restrict__ cdot, G* __restrict__ gsim, float* __restrict__ tau_row) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t L1 = c.L1, L2 = c.L2;
    const int64_t row = int64_t(blockIdx.x) * kBW + wid;
    if (row >= B * L1) return;
    const int64_t b = row / L1, i = row - b * L1;
    int64_t l1, l2;
    window(c.lengths, b, L1, L2, l1, l2);
    const float2 rs = rstat[row];
    const float rd = rdot[row];
    const float2* cb = cstat + b * L2;
    const float* cd = cdot + b * L2;
    float acc = 0.0f;
#pragma unroll
    for (int p = 0; p < VPL; ++p) {
        const int64_t col = 4 * lane + 128 * p;
        if (col >= L2) continue;
        float gr[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (i < l1 && col < l2) {
            float v[4], g[4];
            ld4(sim + row * L2 + col, v);
            ld4(gout + row * L2 + col, g);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (col + e < l2) {
                    const BsVals q = bs_vals(__fmul_rn(v[e], c.invT), rs, cb[col + e]);
                    const float dp = q.out > 1e-9f ? g[e] * 0.5f / q.out : 0.0f;
                    const float a = __fmul_rn(__fmul_rn(__fsub_rn(__fmul_rn(dp, q.col), rd), q.row), c.invT);
                    const float cc =
                        __fmul_rn(__fmul_rn(__fsub_rn(__fmul_rn(dp, q.row), cd[col + e]), q.col), c.invT);
                    gr[e] = __fadd_rn(a, cc);
                    acc += gr[e] * v[e] * c.invT;
                }
            }
        }
        st4(gsim + row * L2 + col, gr);
    }
    if (tau_row != nullptr) {
        acc = warp_sum<32>(acc);
        if (lane == 0) tau_row[row] = acc;
    }
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

int vpl_of(int64_t L2) { return L2 <= 128 ? 1 : L2 <= 256 ? 2 : L2 <= 512 ? 4 : 8; }

int bsf_sm_count() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

// Rows per segment: about 4 CTA waves over the batch, at least 8 rows per warp.
int64_t bsf_seg_rows(int64_t B, int64_t L1) {
    const int64_t slots = int64_t(bsf_sm_count()) * 2;
    int64_t nseg = (4 * slots + B - 1) / B;
    nseg = std::max<int64_t>(1, std::min<int64_t>(nseg, (L1 + 63) / 64));
    int64_t seg = (L1 + nseg - 1) / nseg;
    return ((seg + kBW - 1) / kBW) * kBW;
}

struct BsfWs {
    float2* cpart2;
    float* cpart1;
    float* rdot;
    float* cdot;
    float* tau_row;
    int32_t* cnt;
};

BsfWs carve_bsf(Carve& c, int64_t B, int64_t L1, int64_t L2, bool bwd) {
    const int64_t seg = bsf_seg_rows(B, L1);
    const int64_t nseg = (L1 + seg - 1) / seg;
    BsfWs w{};
    if (!bwd) {
        w.cpart2 = c.take<float2>(size_t(B * nseg * L2));
    } else {
        w.cpart1 = c.take<float>(size_t(B * nseg * L2));
        w.rdot = c.take<float>(size_t(B * L1));
        w.cdot = c.take<float>(size_t(B * L2));
        w.tau_row = c.take<float>(size_t(B * L1));
    }
    w.cnt = c.take<int32_t>(size_t(B));
    return w;
}

template <typename T, int VPL>
int fwd_impl(const T* sim, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau, float* out,
             float2* rstat, float2* cstat, void* ws, cudaStream_t st) {
    Carve cv(ws);
    BsfWs w = carve_bsf(cv, B, L1, L2, false);
    BsfCommon c{lengths, L1, L2, 1.0f / tau, bsf_seg_rows(B, L1), 0, w.cnt};
    c.nseg = int((L1 + c.seg_rows - 1) / c.seg_rows);
    const size_t sm = size_t(kBW) * L2 * sizeof(float2);
    cudaFuncSetAttribute(bsf_stats_kernel<T, VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
    cudaMemsetAsync(w.cnt, 0, sizeof(int32_t) * size_t(B), st);
    {
        ProfScope ps(DOT_K_BS_FWD, st);
        bsf_stats_kernel<T, VPL><<<dim3(unsigned(c.nseg), unsigned(B)), kBT, sm, st>>>(sim, c, rstat, w.cpart2, cstat);
    }
    {
        ProfScope ps(DOT_K_BS_FWD, st);
        bsf_out_kernel<T, VPL><<<unsigned(ceil_div(B * L1, kBW)), kBT, 0, st>>>(sim, c, B, rstat, cstat, out);
    }
    return check_launch("bidirectional softmax forward (fused)");
}

template <typename T, typename G, int VPL>
int bwd_impl(const T* sim, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau, const float2* rstat,
             const float2* cstat, const float* gout, G* gsim, float* gtau, void* ws, cudaStream_t st) {
    Carve cv(ws);
    BsfWs w = carve_bsf(cv, B, L1, L2, true);
    BsfCommon c{lengths, L1, L2, 1.0f / tau, bsf_seg_rows(B, L1), 0, w.cnt};
    c.nseg = int((L1 + c.seg_rows - 1) / c.seg_rows);
    const size_t sm = size_t(kBW) * L2 * sizeof(float) + size_t(L2) * sizeof(float2);
    cudaFuncSetAttribute(bsf_dots_kernel<T, VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
    cudaMemsetAsync(w.cnt, 0, sizeof(int32_t) * size_t(B), st);
    {
        ProfScope ps(DOT_K_BS_BWD, st);
        bsf_dots_kernel<T, VPL><<<dim3(unsigned(c.nseg), unsigned(B)), kBT, sm, st>>>(sim, gout, c, rstat, cstat,
                                                                                      w.rdot, w.cpart1, w.cdot);
    }
    {
        ProfScope ps(DOT_K_BS_BWD, st);
        bsf_grad_kernel<T, G, VPL><<<unsigned(ceil_div(B * L1, kBW)), kBT, 0, st>>>(
            sim, gout, c, B, rstat, cstat, w.rdot, w.cdot, gsim, gtau ? w.tau_row : nullptr);
    }
    if (gtau != nullptr) {
        ProfScope ps(DOT_K_BS_BWD, st);
        bsf_batch_sum_kernel<<<unsigned(ceil_div(B, 8)), 256, 0, st>>>(w.tau_row, gtau, B, L1, -1.0f);
    }
    return check_launch("bidirectional softmax backward (fused)");
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

bool bsf_supported(int64_t L2, const void* sim, int dtype, const void* gout, const void* gsim) {
    const uintptr_t al = dtype == DOT_F32 ? 15u : 7u;
    auto ok = [&](const void* p, uintptr_t mask) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & mask) == 0; };
    return L2 >= 4 && L2 <= 1024 && (L2 % 4) == 0 && ok(sim, al) && ok(gout, 15u) && ok(gsim, 7u);
}

size_t bsf_fwd_ws(int64_t B, int64_t L1, int64_t L2) {
    Carve c(nullptr);
    carve_bsf(c, B, L1, L2, false);
    return c.size();
}

size_t bsf_bwd_ws(int64_t B, int64_t L1, int64_t L2) {
    Carve c(nullptr);
    carve_bsf(c, B, L1, L2, true);
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

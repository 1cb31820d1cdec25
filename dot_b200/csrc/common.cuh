// Shared device helpers for the dot_b200 kernels (sm_100a).
//
// Arithmetic conventions shared with the reference (caseysm/dot):
//  * Sinkhorn works in the log domain, in natural-log units, with the
//    reference's operation order: K = X * (sign/tau) rounded to fp32 (the
//    reference materialises log_K = log_alpha * inv_tau, src/sinkhorn/
//    kernels.cu:128-139,1338-1353), then t = K + v rounded, max over the
//    reduced axis, sum of exp(t - max).  Only the exponential of the
//    (non-positive) shifted difference goes through base 2: exp(d) =
//    2^(d*log2 e) on the SFU (ex2.approx); its argument error is |d|*2^-24,
//    so the terms that dominate a sum (small |d|) are accurate to a few ulp.
//  * exp clamp: the reference's safe_exp returns 0 below -88 and caps the
//    argument at +88 (src/sinkhorn/kernels.cu:21-25).
//  * log floor: log(max(sum, 1e-12)) on every log-sum-exp
//    (src/sinkhorn/kernels.cu:538,620).
//  * empty max: -FLT_MAX, as the reference's reductions start from it.
#pragma once

#include <cfloat>
#include <cstdint>
#include <cuda_runtime.h>

namespace dotb {

constexpr float kLog2e = 1.4426950408889634f;   // log2(e)
constexpr float kLn2 = 0.6931471805599453f;     // ln(2)
constexpr float kSumFloor = 1.0e-12f;
constexpr float kNegBig = -FLT_MAX;

// 2^x on the SFU (ex2.approx, subnormal results flushed to zero).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ln(x) from the SFU's base-2 log (lg2.approx, absolute error about 2^-22 in
// log2 over the normal range), for a row sum in [1, m]: the sum of a row's
// exp(t - max), whose largest term is 1.  Accurate log-sum-exps elsewhere use
// lse_finish.
__device__ __forceinline__ float fast_log(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y * 0.6931471805599453f;
}

// exp(d) for a shifted difference d <= 0 inside a log-sum-exp.
__device__ __forceinline__ float exp_shift(float d) { return ex2(d * kLog2e); }

// The reference's safe_exp (accurate expf, 0 below -88, argument capped at 88),
// used where a value is written out (the plan).
__device__ __forceinline__ float safe_expf(float x) {
    if (x < -88.0f) return 0.0f;
    return expf(fminf(x, 88.0f));
}

// log of a log-sum-exp partial (max m, sum s of exp(x - m)) with the 1e-12 floor.
__device__ __forceinline__ float lse_finish(float m, float s) {
    return m + logf(fmaxf(s, kSumFloor));
}

// Merge two (max, sum) log-sum-exp partials.
__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
    float mn = fmaxf(m, m2);
    s = s * exp_shift(m - mn) + s2 * exp_shift(m2 - mn);
    m = mn;
}

template <int W>
__device__ __forceinline__ void warp_lse(float& m, float& s) {
#pragma unroll
    for (int off = W / 2; off > 0; off >>= 1) {
        float m2 = __shfl_xor_sync(0xffffffffu, m, off);
        float s2 = __shfl_xor_sync(0xffffffffu, s, off);
        lse_merge(m, s, m2, s2);
    }
}

template <int W>
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = W / 2; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

template <int W>
__device__ __forceinline__ float warp_max(float v) {
    if constexpr (W == 32) {
        // one instruction on sm_100a (redux.sync with .f32, PTX ISA 8.6); max is
        // exact, so this equals the shuffle tree bit for bit
        float r;
        asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
        return r;
    } else {
#pragma unroll
        for (int off = W / 2; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
        return v;
    }
}

// Sum of N registers as a balanced tree (short dependency chain).
template <int N>
__device__ __forceinline__ float tree_sum(const float (&x)[N]) {
    if constexpr (N == 1) {
        return x[0];
    } else {
        float h[(N + 1) / 2];
#pragma unroll
        for (int k = 0; k < N / 2; ++k) h[k] = x[2 * k] + x[2 * k + 1];
        if constexpr (N % 2 == 1) h[N / 2] = x[N - 1];
        return tree_sum<(N + 1) / 2>(h);
    }
}

// Max of N registers as a balanced tree (max is exact: any order gives the
// same value).
template <int N>
__device__ __forceinline__ float tree_max(const float (&x)[N]) {
    if constexpr (N == 1) {
        return x[0];
    } else {
        float h[(N + 1) / 2];
#pragma unroll
        for (int k = 0; k < N / 2; ++k) h[k] = fmaxf(x[2 * k], x[2 * k + 1]);
        if constexpr (N % 2 == 1) h[N / 2] = x[N - 1];
        return tree_max<(N + 1) / 2>(h);
    }
}

// Online update of a (max, sum) partial with a group of K new values
// (-INFINITY marks an empty slot).
template <int K>
__device__ __forceinline__ void lse_push(float& m, float& s, const float (&t)[K]) {
    float gm = t[0];
#pragma unroll
    for (int k = 1; k < K; ++k) gm = fmaxf(gm, t[k]);
    if (gm > m) {
        s *= exp_shift(m - gm);
        m = gm;
    }
#pragma unroll
    for (int k = 0; k < K; ++k) s += exp_shift(t[k] - m);
}

// K_ij + w: the scaled kernel entry (rounded, as the reference stores log_K)
// plus a potential, without FMA contraction.
__device__ __forceinline__ float kplus(float x, float kinv, float w) {
    return __fadd_rn(__fmul_rn(x, kinv), w);
}

// Scaled squared Euclidean distance of two points of dimension d:
//   s = (x_0 - y_0)^2, then s = fma(x_k - y_k, x_k - y_k, s) for k = 1..d-1
//   (every difference rounded to fp32), cost = s * scale rounded.
// The point-cloud solvers build every cost entry with exactly these
// operations (the packed f32x2 forms perform the same IEEE operations per
// half), so a cost matrix materialised by dot_sq_dist equals, bit for bit,
// the one the fused sweeps see.
template <int PD>
__device__ __forceinline__ float sq_dist(const float (&x)[PD], const float (&y)[PD], float scale) {
    float d = __fsub_rn(x[0], y[0]);
    float s = __fmul_rn(d, d);
#pragma unroll
    for (int k = 1; k < PD; ++k) {
        d = __fsub_rn(x[k], y[k]);
        s = __fmaf_rn(d, d, s);
    }
    return __fmul_rn(s, scale);
}
__device__ __forceinline__ float sq_dist_n(const float* x, const float* y, int dim, float scale) {
    float d = __fsub_rn(x[0], y[0]);
    float s = __fmul_rn(d, d);
    for (int k = 1; k < dim; ++k) {
        d = __fsub_rn(x[k], y[k]);
        s = __fmaf_rn(d, d, s);
    }
    return __fmul_rn(s, scale);
}

// Column kernels put the batch index in gridDim.z, at most kMaxGridZ per
// launch; larger batches are launched in slices, each kernel adding the
// slice's first batch index b0 to blockIdx.z.
constexpr int64_t kMaxGridZ = 65535;

__device__ __forceinline__ bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// float <-> order-preserving uint for atomicMax on non-negative floats.
__device__ __forceinline__ void atomic_max_nonneg(float* addr, float v) {
    atomicMax(reinterpret_cast<unsigned int*>(addr), __float_as_uint(v));
}

}  // namespace dotb

// Packed two-lane fp32 arithmetic for sm_100a (PTX add/sub/mul/fma .rn.f32x2):
// one instruction performs the same IEEE round-to-nearest operation on both
// halves of a 64-bit register pair -- each instruction on its own is
// bit-identical per half to the scalar __fadd_rn / __fmul_rn / fmaf (measured
// on 1M operand pairs) -- while the issue slots halve.  One difference from
// the scalar intrinsics: ptxas contracts a mul.rn.f32x2 whose result feeds an
// add.rn.f32x2 into a fused multiply-add (measured: add2(mul2(a, b), c)
// equals fmaf(a, b, c) in both lanes), where __fadd_rn(__fmul_rn(a, b), c)
// always rounds the product first.  Code that needs the product rounded
// first does the add in scalar form.  Also the three-input max.f32 (sm_100a).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace dotb {

__device__ __forceinline__ unsigned long long f2_bits(float2 a) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a.x), "f"(a.y));
    return r;
}
__device__ __forceinline__ float2 f2_of(unsigned long long r) {
    float2 a;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a.x), "=f"(a.y) : "l"(r));
    return a;
}

// a + b
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    unsigned long long r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_of(r);
}
// a - b
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
    unsigned long long r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_of(r);
}
// a * b
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
    unsigned long long r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_of(r);
}
// a * b + c, one rounding per half
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
    return f2_of(r);
}
__device__ __forceinline__ float2 splat2(float x) { return make_float2(x, x); }

// max(a, b, c) in one instruction
__device__ __forceinline__ float max3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// Max of N floats (N even, pairs) with three-input max: a chain over the
// halves, then one combine.
template <int N>
__device__ __forceinline__ float max_of(const float2 (&x)[N]) {
    float a = fmaxf(x[0].x, x[0].y);
    float b = N > 1 ? fmaxf(x[N > 1 ? 1 : 0].x, x[N > 1 ? 1 : 0].y) : a;
#pragma unroll
    for (int k = 2; k < N; k += 2) {
        a = max3(a, x[k].x, x[k].y);
        if (k + 1 < N) b = max3(b, x[k + 1 < N ? k + 1 : k].x, x[k + 1 < N ? k + 1 : k].y);
    }
    return fmaxf(a, b);
}

// Sum of N float2 as a balanced tree of packed adds, then the two halves.
template <int N>
__device__ __forceinline__ float2 tree_sum2(const float2 (&x)[N]) {
    if constexpr (N == 1) {
        return x[0];
    } else {
        float2 h[(N + 1) / 2];
#pragma unroll
        for (int k = 0; k < N / 2; ++k) h[k] = add2(x[2 * k], x[2 * k + 1]);
        if constexpr (N % 2 == 1) h[N / 2] = x[N - 1];
        return tree_sum2<(N + 1) / 2>(h);
    }
}

}  // namespace dotb

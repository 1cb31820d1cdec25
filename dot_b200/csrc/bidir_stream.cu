// Bidirectional softmax for rows of at most 1024 columns (fp32 input with
// L2 % 4 == 0 or bf16 input with L2 % 8 == 0; 16-byte aligned tensors): two
// streaming sweeps per direction.
//
//   out_ij  = sqrt(1e-9 + row_ij * col_ij),  row = softmax_j(sim/T),
//             col = softmax_i(sim/T), 0 outside the length window
//   grad_ij = (2 q_ij - rdot_i*row_ij - cdot_j*col_ij) / T,
//             q = (g * 0.5 / out) * row * col, rdot_i = sum_j q_ij,
//             cdot_j = sum_i q_ij
// (reference: src/bidirectional_softmax/kernels_cpu.cpp:41-232).
//
// forward   statistics sweep: persistent CTAs (one wave), each streaming an
//           equal contiguous range of row blocks (R rows, <= 32 KB) through a
//           2-stage ring of 1-D bulk copies.  A warp (two for rows over 512
//           columns) takes a row: its max and sum of exp(v - max) give the row
//           statistics; the same exponentials rescaled by exp(max - A), A a
//           warp-wide reference, accumulate the columns' sums (one FFMA per
//           element).  When a CTA's range leaves a problem it merges its
//           warps' column partials and publishes them; the CTA that arrives
//           last for the problem (atomic counter, no waiting) merges the
//           segments in order into the column statistics.  A column whose
//           merged sum is too small to trust is recomputed exactly from sim.
//           output sweep: the same ring again, elementwise from sim and the
//           statistics.
// backward  dot sweep: the same ring over sim and grad_out rows: q, its row
//           sums (rdot) and column partials (cdot, merged as above).
//           gradient sweep: the same ring again, elementwise; per-row partials
//           of sum grad * sim / T for the temperature gradient.
// The statistics are (max, 1/sum); every sweep recomputes its values from
// sim.  The output and dot sweeps need only row * col, which they take from
// one exponential, exp(2v - rmax - cmax), with the same expression; the
// gradient sweep needs row and col apart and forms row * col from them
// (within a few ulp of the other form).  Element pairs go through the packed
// f32x2 instructions (half the issue slots of scalar FP32 code); full-width
// rows (l2 == L2 == 128 * VPL) take a path without per-element masks.  Each
// sweep reads its inputs once (the second sweep of a direction re-reads sim,
// and grad_out: 1.5x / 1.67x the compulsory bytes of the two directions) and
// runs at streaming bandwidth instead of holding whole problems in flight.
// The second sweep of a direction is a programmatic dependent launch: it sets
// up and starts copying sim while the first finishes.
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "common.cuh"
#include "internal.h"
#include "pack.cuh"
#include "tma.cuh"

namespace dotb {

namespace {

constexpr int kT = 256;             // threads per CTA
constexpr int kW = kT / 32;         // warps per CTA
constexpr int kStage = 32768;       // bytes per ring stage
constexpr int kS = 2;               // ring stages
constexpr int kMaxL2 = 1024;
constexpr int kMaxR = 64;           // rows per block at most
constexpr float kRaiseB = 60.0f;
constexpr float kTinyB = 8.077935669463161e-28f;   // 2^-90

// Warps per row and the columns a lane holds: a row of L2 <= 128*VPL columns
// is split over WPR warps; lane l of part c holds columns
// c*128*VPLW + 4l + 128p + e (p < VPLW, e < 4).
template <int VPL>
struct WL {
    static constexpr int WPR = VPL >= 8 ? 2 : 1;
    static constexpr int VPLW = VPL / WPR;
    static constexpr int NC = 4 * VPLW;
    static constexpr int NP = NC / 2;   // value pairs per lane
    static constexpr int SLOTS = kW / WPR;
};

// ---------------------------------------------------------------------------
// element access
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ld4s(const float* p, float (&v)[4]) {   // shared memory
    const float4 x = *reinterpret_cast<const float4*>(p);
    v[0] = x.x;
    v[1] = x.y;
    v[2] = x.z;
    v[3] = x.w;
}
__device__ __forceinline__ void ld4s(const __nv_bfloat16* p, float (&v)[4]) {
    const uint2 x = *reinterpret_cast<const uint2*>(p);
    v[0] = __uint_as_float(x.x << 16);
    v[1] = __uint_as_float(x.x & 0xffff0000u);
    v[2] = __uint_as_float(x.y << 16);
    v[3] = __uint_as_float(x.y & 0xffff0000u);
}
__device__ __forceinline__ void st4g(float* p, const float (&v)[4]) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(v[0], v[1], v[2], v[3]));
}
__device__ __forceinline__ void st4g(__nv_bfloat16* p, const float (&v)[4]) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
    const __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 x;
    x.x = *reinterpret_cast<const uint32_t*>(&a);
    x.y = *reinterpret_cast<const uint32_t*>(&b);
    __stcs(reinterpret_cast<uint2*>(p), x);
}
// four consecutive columns' statistics (shared memory, 16-byte aligned) as
// pairs (c0, c1), (c2, c3): f from pf, g from pg
__device__ __forceinline__ void cs4_pairs(const float* pf, const float* pg, float2 (&f)[2], float2 (&g)[2]) {
    const float4 a = *reinterpret_cast<const float4*>(pf);
    const float4 b = *reinterpret_cast<const float4*>(pg);
    f[0] = make_float2(a.x, a.y);
    f[1] = make_float2(a.z, a.w);
    g[0] = make_float2(b.x, b.y);
    g[1] = make_float2(b.z, b.w);
}
__device__ __forceinline__ float rsqrt_approx(float x) {
    float y;
    asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void window(const int32_t* lengths, int64_t b, int64_t L1, int64_t L2, int64_t& l1,
                                       int64_t& l2) {
    l1 = min(max(int64_t(__ldg(lengths + 2 * b)), int64_t(0)), L1);
    l2 = min(max(int64_t(__ldg(lengths + 2 * b + 1)), int64_t(0)), L2);
}

// Per-element values (the output, dot and gradient sweeps) come from the
// statistics: row = exp(v - rmax) * rinv, col = exp(v - cmax) * cinv,
// out = min(sqrt(1e-9 + row * col), 1), 1/out = rsqrt(1e-9 + row * col).
// sqrt and rsqrt run on the SFU (~2^-22 relative).  The column value's
// numerator exp(v - A) and its share of the column sum (accumulated as E*w)
// can differ by an ulp, so row * col may exceed 1 by rounding where one
// element dominates its row and column; out is capped at 1, its
// exact-arithmetic bound (1/out then differs from 1 by those few ulp).
// out >= sqrt(1e-9) > 1e-9, so the reference's guard dp = 0 for out <= 1e-9
// never applies.  Pairs of elements go through the packed f32x2
// instructions.

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

__device__ __forceinline__ float sqrt_approx(float x) {
    float y;
    asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float2 ex2x2(float2 x) { return make_float2(ex2(x.x), ex2(x.y)); }

// This lane's values of a row, scaled by 1/T (rounded), as pairs; -inf
// outside [0, l2).  FULL: the row is l2 == L2 == 128 * VPLW * WPR columns.
template <typename T, int VPLW, bool FULL>
__device__ __forceinline__ void load_scaled(const T* xr, int cbase, int lane, int64_t L2, int64_t l2, float invT,
                                            float2 (&t)[2 * VPLW]) {
#pragma unroll
    for (int p = 0; p < VPLW; ++p) {
        const int col = cbase + 4 * lane + 128 * p;
        if (FULL || col < L2) {
            float v[4];
            ld4s(xr + col, v);
            t[2 * p] = mul2(make_float2(v[0], v[1]), splat2(invT));
            t[2 * p + 1] = mul2(make_float2(v[2], v[3]), splat2(invT));
            if (!FULL && col + 3 >= l2) {
                if (col + 0 >= l2) t[2 * p].x = -INFINITY;
                if (col + 1 >= l2) t[2 * p].y = -INFINITY;
                if (col + 2 >= l2) t[2 * p + 1].x = -INFINITY;
                t[2 * p + 1].y = -INFINITY;
            }
        } else {
            t[2 * p] = t[2 * p + 1] = make_float2(-INFINITY, -INFINITY);
        }
    }
}

// row * col for a pair of elements from one exponential:
// 2^((2v - rmax - cmax) log2 e) * rinv * cinv, the exponent formed as
// fma(v, 2 log2 e, -rmL) - cmL (rmL, cmL: the maxima times log2 e, rounded;
// nrmL = -rmL).  The output and dot sweeps use this same expression.
__device__ __forceinline__ float2 rowcol2(float2 val, float2 nrmL, float2 rinv, float2 cmL, float2 cinv) {
    const float2 d = sub2(fma2(val, splat2(2.0f * kLog2e), nrmL), cmL);
    return mul2(mul2(ex2x2(d), rinv), cinv);
}

// ---------------------------------------------------------------------------
// balanced persistent schedule over the B * nblk row blocks
// ---------------------------------------------------------------------------
struct Sched {
    int T;        // total blocks (< 2^31: bsf_supported)
    int nblk;     // blocks per problem
    int G;        // CTAs
    int maxseg;   // most CTAs touching one problem
};
__host__ __device__ __forceinline__ int sched_q(const Sched& s, int k) { return int(int64_t(k) * s.T / s.G); }
__host__ __device__ __forceinline__ int sched_owner(const Sched& s, int x) {
    return int((int64_t(x + 1) * s.G + s.T - 1) / s.T) - 1;
}

struct SweepArgs {
    const unsigned char* sim;
    const float* gout;         // backward: grad_out rows follow the sim rows in a stage
    const int32_t* lengths;
    int64_t L1, L2;
    int esz;                   // bytes per sim element
    int R;                     // rows per block
    uint32_t gout_off;         // byte offset of the grad_out rows in a stage
    Sched s;
    float invT;
    float2* rstat;             // forward: written; backward: read
    float2* cstat;
    float* rdot;               // backward
    float* cdot;
    float* out;                // forward output sweep
    float* tau_row;            // backward: per-row sum of grad * sim / T, or nullptr
    void* part;                // [B][maxseg][L2]: float2 (forward) or float (backward)
    int32_t* cnt;              // [B] arrival counters, zero between launches
    int32_t* err;              // bounded-wait expiry word
};

// Arrival at the end of a problem segment; true (to every thread) in the CTA
// that arrived last for problem b.
__device__ __forceinline__ bool arrive_last(int32_t* cnt, int64_t b, int nseg, int* s_flag) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *s_flag = (atomicAdd(cnt + b, 1) == nseg - 1) ? 1 : 0;
    __syncthreads();
    const bool last = *s_flag != 0;
    if (last) __threadfence();
    return last;
}

// The CTA's ring over its block range [g0, g1) (stage k at smem + k * kStage).
// Positions p run g0 .. g1-1; the block at position p is p, or, for a ring
// walked backwards (rev), g0 + g1 - 1 - p.  The second sweep of a direction
// walks its range backwards: the first sweep gave every CTA the same range
// and read it forwards, so its last blocks -- the first ones read again --
// are the ones still in L2.
struct Ring {
    const SweepArgs* a;
    unsigned char* smem;
    uint64_t* bar;
    int g0, g1;
    bool rev;

    __device__ int block(int p) const { return rev ? g0 + g1 - 1 - p : p; }
    __device__ unsigned char* stage(int p) const { return smem + size_t((p - g0) % kS) * kStage; }
    __device__ uint64_t* barrier(int p) const { return bar + (p - g0) % kS; }
    __device__ uint32_t parity(int p) const { return uint32_t(((p - g0) / kS) & 1); }
    __device__ void issue(int p) const {   // one thread
        const int g = block(p);
        const int b = g / a->s.nblk, jb = g - b * a->s.nblk;
        const int64_t r0 = int64_t(jb) * a->R;
        const uint32_t rows = uint32_t(min(int64_t(a->R), a->L1 - r0));
        const int64_t row0 = int64_t(b) * a->L1 + r0;
        const uint32_t b0 = rows * uint32_t(a->L2) * uint32_t(a->esz);
        const uint32_t b1 = a->gout ? rows * uint32_t(a->L2) * 4u : 0u;
        uint64_t* bb = barrier(p);
        mbar_arrive_expect_tx(bb, b0 + b1);
        bulk_g2s(stage(p), a->sim + row0 * a->L2 * a->esz, b0, bb);
        if (a->gout) bulk_g2s(stage(p) + a->gout_off, a->gout + row0 * a->L2, b1, bb);
    }
    __device__ bool wait(int p) const { return mbar_wait_sleep(barrier(p), parity(p), a->err); }
};

__device__ __forceinline__ Ring ring_start(const SweepArgs& a, uint64_t* bars, unsigned char* smem,
                                           bool rev = false) {
    Ring r;
    r.a = &a;
    r.smem = smem;
    r.bar = bars;
    r.rev = rev;
    r.g0 = sched_q(a.s, blockIdx.x);
    r.g1 = sched_q(a.s, int(blockIdx.x) + 1);
    if (threadIdx.x == 0) {
#pragma unroll
        for (int k = 0; k < kS; ++k) mbar_init(&bars[k], 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x == 0)
        for (int g = r.g0; g < r.g1 && g < r.g0 + kS; ++g) r.issue(g);
    return r;
}

// Wait (bounded) for the copies of positions [k0, k1) (clipped to the range),
// then the CTA may return.
__device__ __forceinline__ void ring_drain_span(const Ring& r, int k0, int k1) {
    if (threadIdx.x == 0)
        for (int k = k0; k < r.g1 && k < k1; ++k) r.wait(k);
    __syncthreads();
}

// After a failed wait at block g: wait (bounded) for the copies still in flight.
__device__ __forceinline__ void ring_drain(const Ring& r, int g) {
    if (threadIdx.x == 0)
        for (int k = g; k < r.g1 && k < g + kS; ++k) r.wait(k);
    __syncthreads();
}

// ---------------------------------------------------------------------------
// forward: statistics sweep
// ---------------------------------------------------------------------------
template <typename T, int VPL>
__global__ void __launch_bounds__(kT, 3) bs2_stats_kernel(SweepArgs a) {
    using W = WL<VPL>;
    constexpr int WPR = W::WPR, VPLW = W::VPLW, NP = W::NP, SLOTS = W::SLOTS;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[kS];
    __shared__ float2 s_rp[2][kMaxR][WPR];   // per-row (max, sum) of the row's warps, two blocks
    __shared__ int s_flag, s_nfix, s_abort;
    __shared__ int s_fix[kMaxL2];

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int slot = wid / WPR, cpart = wid % WPR;
    const int cbase = cpart * 128 * VPLW;
    const int64_t L1 = a.L1, L2 = a.L2;
    if (tid == 0) {
        s_nfix = 0;
        s_abort = 0;
    }
    pdl_launch_dependents();   // the second sweep may start its copies of the read-only input
    const Ring rg = ring_start(a, bars, smem);
    const T* simT = reinterpret_cast<const T*>(a.sim);
    // row statistics of a block from its warps' partials (threads < rows)
    auto write_rstat = [&](int buf, int bb, int jbb, int rws, int64_t ll1, int64_t ll2) {
        if (tid < rws) {
            const int64_t i = int64_t(jbb) * a.R + tid;
            float2 st = make_float2(0.0f, 0.0f);
            if (i < ll1 && ll2 > 0) {
                float mm = kNegBig, ss = 0.0f;
#pragma unroll
                for (int c = 0; c < WPR; ++c) lse_merge(mm, ss, s_rp[buf][tid][c].x, s_rp[buf][tid][c].y);
                st = make_float2(mm, ss > 0.0f ? 1.0f / ss : 0.0f);
            }
            a.rstat[int64_t(bb) * L1 + i] = st;
        }
    };
    // the previous block's row statistics are written after the next
    // barrier; such a block is never a problem's last, so it is the full
    // block jb - 1 of the current problem
    bool pend = false;

    float2 Sc[NP];   // column sums of exp(v - A), this lane's columns in pairs
    float A = kNegBig;
    const bool wide = L2 == 128 * VPL;
    int64_t l1 = 0, l2 = 0;
    int b = rg.g0 / a.s.nblk, jb = rg.g0 - b * a.s.nblk;   // advanced per block, no division
    int cur = -1;

    // column statistic of column col from its merged (max, sum)
    auto finish = [&](int bb, int64_t col, float mm, float ss) {
        if (col < l2) {
            if (ss < kTinyB) s_fix[atomicAdd(&s_nfix, 1)] = int(col);
            else a.cstat[int64_t(bb) * L2 + col] = make_float2(mm, 1.0f / ss);
        } else {
            a.cstat[int64_t(bb) * L2 + col] = make_float2(0.0f, 0.0f);
        }
    };

    for (int g = rg.g0; g < rg.g1; ++g) {
        if (b != cur) {
            cur = b;
            window(a.lengths, b, L1, L2, l1, l2);
#pragma unroll
            for (int k = 0; k < NP; ++k) Sc[k] = make_float2(0.0f, 0.0f);
            A = kNegBig;
        }
        const int rows = int(min(int64_t(a.R), L1 - int64_t(jb) * a.R));
        const int pb = (g - rg.g0) & 1;
        // One barrier per block: the previous block's rows are done, so its
        // stage is refilled and its row statistics written here; a failed
        // copy wait (recorded in s_abort, the rows below then read stale
        // but in-bounds shared memory) ends the CTA at the next barrier.
        __syncthreads();
        if (s_abort) {
            ring_drain_span(rg, g - 1, g - 1 + kS);
            return;
        }
        if (g > rg.g0) {
            if (tid == 0 && g - 1 + kS < rg.g1) rg.issue(g - 1 + kS);
            if (pend) write_rstat(pb ^ 1, b, jb - 1, a.R, l1, l2);
        }
        if (!rg.wait(g)) s_abort = 1;
        const T* xs = reinterpret_cast<const T*>(rg.stage(g));
        const bool fullw = wide && l2 == L2;
        // The row's exponentials, sums and column weights: a row whose warp
        // part is all masked (max -inf) contributes nothing.  Rows enter the
        // column sums in the order il, il + SLOTS, ...
        // exp(t - mx) as 2^(t*log2e - mL) in one FFMA, mL = mx*log2e rounded;
        // every term carries 2^cr, cr = mx*log2e - mL exactly (FMA remainder),
        // taken out of the row sum and the column weight.  A row whose warp
        // part is all masked (mx = -inf; warp-uniform) gets mL = 0: its terms
        // are exp(-inf) = 0.
        auto exps = [&](float2 (&t)[NP], float mx, float& cr) {
            const float mL = mx == -INFINITY ? 0.0f : mx * kLog2e;
            cr = mx == -INFINITY ? 0.0f : fmaf(mx, kLog2e, -mL);
#pragma unroll
            for (int k = 0; k < NP; ++k) t[k] = ex2x2(fma2(t[k], splat2(kLog2e), splat2(-mL)));
        };
        auto accumulate = [&](float2 (&t)[NP], float mx, float cr) {
            if (mx == -INFINITY) return;
            if (mx > A + kRaiseB) {
                const float sc = exp_shift(A - mx);
#pragma unroll
                for (int k = 0; k < NP; ++k) Sc[k] = mul2(Sc[k], splat2(sc));
                A = mx;
            }
            const float w = ex2(fmaf(mx - A, kLog2e, -cr));   // exp(mx - A) / 2^cr
#pragma unroll
            for (int k = 0; k < NP; ++k) Sc[k] = fma2(t[k], splat2(w), Sc[k]);
        };
        int il = slot;
        if (fullw) {
            // two live full-width rows per pass: their loads, maxima and sums
            // overlap (same results as one at a time)
            for (; il + SLOTS < rows && int64_t(jb) * a.R + il + SLOTS < l1; il += 2 * SLOTS) {
                float2 t0[NP], t1[NP];
                load_scaled<T, VPLW, true>(xs + il * L2, cbase, lane, L2, l2, a.invT, t0);
                load_scaled<T, VPLW, true>(xs + (il + SLOTS) * L2, cbase, lane, L2, l2, a.invT, t1);
                const float m0 = warp_max<32>(max_of(t0)), m1 = warp_max<32>(max_of(t1));
                float cr0, cr1;
                exps(t0, m0, cr0);
                exps(t1, m1, cr1);
                const float2 u0 = tree_sum2(t0), u1 = tree_sum2(t1);
                float s0 = u0.x + u0.y, s1 = u1.x + u1.y;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    s0 += __shfl_xor_sync(0xffffffffu, s0, off);
                    s1 += __shfl_xor_sync(0xffffffffu, s1, off);
                }
                s0 = m0 == -INFINITY ? 0.0f : s0 * ex2(-cr0);
                s1 = m1 == -INFINITY ? 0.0f : s1 * ex2(-cr1);
                accumulate(t0, m0, cr0);
                accumulate(t1, m1, cr1);
                if (lane == 0) {
                    s_rp[pb][il][cpart] = make_float2(m0 == -INFINITY ? kNegBig : m0, s0);
                    s_rp[pb][il + SLOTS][cpart] = make_float2(m1 == -INFINITY ? kNegBig : m1, s1);
                }
            }
        }
        for (; il < rows; il += SLOTS) {
            const int64_t i = int64_t(jb) * a.R + il;
            if (i >= l1 || l2 == 0) {
                if (lane == 0) s_rp[pb][il][cpart] = make_float2(kNegBig, 0.0f);
                continue;
            }
            float2 t[NP];
            if (fullw) load_scaled<T, VPLW, true>(xs + il * L2, cbase, lane, L2, l2, a.invT, t);
            else load_scaled<T, VPLW, false>(xs + il * L2, cbase, lane, L2, l2, a.invT, t);
            const float mx = warp_max<32>(max_of(t));
            float cr;
            exps(t, mx, cr);
            const float2 u = tree_sum2(t);
            const float s = mx == -INFINITY ? 0.0f : warp_sum<32>(u.x + u.y) * ex2(-cr);
            accumulate(t, mx, cr);
            if (lane == 0) s_rp[pb][il][cpart] = make_float2(mx == -INFINITY ? kNegBig : mx, s);
        }
        pend = !(g + 1 == rg.g1 || jb + 1 == a.s.nblk);
        if (!pend) {
            // ---- end of this CTA's part of problem b: publish its column partials
            // (the next block's barrier orders the merge buffer before the refill) ----
            __syncthreads();   // the stage is free; s_rp is complete
            write_rstat(pb, b, jb, rows, l1, l2);
            const int kfirst = sched_owner(a.s, b * a.s.nblk);
            const int nseg = sched_owner(a.s, (b + 1) * a.s.nblk - 1) - kfirst + 1;
            const int seg = int(blockIdx.x) - kfirst;
            float2* mb = reinterpret_cast<float2*>(rg.stage(g));   // [SLOTS][L2] <= 32 KB
#pragma unroll
            for (int p = 0; p < VPLW; ++p) {
                const int64_t col = cbase + 4 * lane + 128 * p;
                if (col < L2) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 pr = Sc[2 * p + (e >> 1)];
                        mb[slot * L2 + col + e] = make_float2(A, (e & 1) ? pr.y : pr.x);
                    }
                }
            }
            __syncthreads();
            float2* mypart = static_cast<float2*>(a.part) + (int64_t(b) * a.s.maxseg + seg) * L2;
            for (int64_t col = tid; col < L2; col += kT) {
                float mm = kNegBig, ss = 0.0f;
#pragma unroll
                for (int q = 0; q < SLOTS; ++q) {
                    const float2 v = mb[q * L2 + col];
                    lse_merge(mm, ss, v.x, v.y);
                }
                if (nseg == 1) finish(b, col, mm, ss);
                else mypart[col] = make_float2(mm, ss);
            }
            bool merged = nseg == 1;
            if (nseg > 1 && arrive_last(a.cnt, b, nseg, &s_flag)) {
                merged = true;
                const float2* pb = static_cast<const float2*>(a.part) + int64_t(b) * a.s.maxseg * L2;
                for (int64_t col = tid; col < L2; col += kT) {
                    float mm = kNegBig, ss = 0.0f;
                    for (int sg = 0; sg < nseg; ++sg) {
                        const float2 pp = __ldcg(pb + int64_t(sg) * L2 + col);
                        lse_merge(mm, ss, pp.x, pp.y);
                    }
                    finish(b, col, mm, ss);
                }
                if (tid == 0) a.cnt[b] = 0;
            }
            if (merged) {
                __syncthreads();
                const int nfix = s_nfix;
                for (int k = wid; k < nfix; k += kW) {
                    const int64_t col = s_fix[k];
                    const float2 st = exact_col_stats(simT + int64_t(b) * L1 * L2, L2, l1, col, a.invT);
                    if (lane == 0) a.cstat[int64_t(b) * L2 + col] = st;
                }
                __syncthreads();
                if (tid == 0) s_nfix = 0;
            }
            fence_proxy_async_smem();   // merge-buffer writes before the stage is refilled by a bulk copy
        }
        if (++jb == a.s.nblk) {
            jb = 0;
            ++b;
        }
    }
    // the range always ends with a problem end (nothing pending); a failed
    // wait in the last block leaves its copy to be drained
    __syncthreads();
    if (s_abort) ring_drain_span(rg, rg.g1 - 1, rg.g1);
}

// ---------------------------------------------------------------------------
// forward: output sweep over the same ring (the statistics sweep's warps per row)
// ---------------------------------------------------------------------------
template <typename T, int VPL>
__global__ void __launch_bounds__(kT, 3) bs2_out_kernel(SweepArgs a) {
    using W = WL<VPL>;
    constexpr int WPR = W::WPR, VPLW = W::VPLW, SLOTS = W::SLOTS;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[kS];
    __shared__ __align__(16) float s_cm[kMaxL2];   // the problem's columns: cmax * log2 e
    __shared__ __align__(16) float s_ci[kMaxL2];   // and 1/sum

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int slot = wid / WPR, cpart = wid % WPR;
    const int cbase = cpart * 128 * VPLW;
    const int64_t L1 = a.L1, L2 = a.L2;
    const bool wide = L2 == 128 * VPL;
    const Ring rg = ring_start(a, bars, smem, true);
    pdl_wait();   // the first sweep's statistics / dots are complete and visible
    int64_t l1 = 0, l2 = 0;
    int cur = -1;

    for (int pos = rg.g0; pos < rg.g1; ++pos) {
        const int g = rg.block(pos);
        const int b = g / a.s.nblk, jb = g - b * a.s.nblk;
        if (b != cur) {   // the barrier below orders these writes before their reads
            cur = b;
            window(a.lengths, b, L1, L2, l1, l2);
            for (int64_t col = tid; col < L2; col += kT) {
                const float2 c = __ldg(a.cstat + int64_t(b) * L2 + col);
                s_cm[col] = c.x * kLog2e;
                s_ci[col] = c.y;
            }
        }
        const int rows = int(min(int64_t(a.R), L1 - int64_t(jb) * a.R));
        const bool ok = rg.wait(pos);
        if (!__syncthreads_and(ok)) {
            ring_drain(rg, pos);
            return;
        }
        const T* xs = reinterpret_cast<const T*>(rg.stage(pos));
        for (int il = slot; il < rows; il += SLOTS) {
            const int64_t i = int64_t(jb) * a.R + il;
            const int64_t row = int64_t(b) * L1 + i;
            float* orow = a.out + row * L2;
            const bool live = i < l1;
            const float2 rs = live ? __ldg(a.rstat + row) : make_float2(0.0f, 0.0f);
            const float2 nrmL = splat2(-(rs.x * kLog2e)), rinv = splat2(rs.y);
            const bool full = wide && l2 == L2;
#pragma unroll
            for (int p = 0; p < VPLW; ++p) {
                const int col = cbase + 4 * lane + 128 * p;
                if (!full && col >= L2) continue;
                float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (live && (full || col < l2)) {
                    float v[4];
                    float2 cm[2], ci[2];
                    ld4s(xs + il * L2 + col, v);
                    cs4_pairs(s_cm + col, s_ci + col, cm, ci);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const float2 val = mul2(make_float2(v[2 * h], v[2 * h + 1]), splat2(a.invT));
                        const float2 x = add2(rowcol2(val, nrmL, rinv, cm[h], ci[h]), splat2(1e-9f));
                        o[2 * h] = fminf(sqrt_approx(x.x), 1.0f);
                        o[2 * h + 1] = fminf(sqrt_approx(x.y), 1.0f);
                    }
                    if (!full && col + 3 >= l2) {
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            if (col + e >= l2) o[e] = 0.0f;
                    }
                }
                st4g(orow + col, o);
            }
        }
        __syncthreads();   // the stage is free
        if (tid == 0 && pos + kS < rg.g1) rg.issue(pos + kS);
    }
}

// ---------------------------------------------------------------------------
// backward: dot sweep (rdot, cdot)
// ---------------------------------------------------------------------------
template <typename T, int VPL>
__global__ void __launch_bounds__(kT, 3) bs2_dots_kernel(SweepArgs a) {
    using W = WL<VPL>;
    constexpr int WPR = W::WPR, VPLW = W::VPLW, NP = W::NP, SLOTS = W::SLOTS;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[kS];
    __shared__ __align__(16) float s_cm[kMaxL2];   // the problem's columns: cmax * log2 e
    __shared__ __align__(16) float s_ci[kMaxL2];   // and 1/sum
    __shared__ float s_rd[2][kMaxR][WPR];            // per-row q sums of the row's warps, two blocks
    __shared__ int s_flag, s_abort;

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int slot = wid / WPR, cpart = wid % WPR;
    const int cbase = cpart * 128 * VPLW;
    const int64_t L1 = a.L1, L2 = a.L2;
    if (tid == 0) s_abort = 0;
    pdl_launch_dependents();   // the second sweep may start its copies of the read-only input
    const Ring rg = ring_start(a, bars, smem);
    // rdot of a block's rows from its warps' partials (threads < rows)
    auto write_rdot = [&](int buf, int bb, int jbb, int rws) {
        if (tid < rws) {
            float rd = 0.0f;
#pragma unroll
            for (int c = 0; c < WPR; ++c) rd += s_rd[buf][tid][c];
            a.rdot[int64_t(bb) * L1 + int64_t(jbb) * a.R + tid] = rd;
        }
    };
    bool pend = false;   // the previous (full, same-problem) block's rdot, written after the next barrier

    float2 Sd[NP];   // column sums of q, this lane's columns in pairs
    const bool wide = L2 == 128 * VPL;
    int64_t l1 = 0, l2 = 0;
    int b = rg.g0 / a.s.nblk, jb = rg.g0 - b * a.s.nblk;
    int cur = -1;

    for (int g = rg.g0; g < rg.g1; ++g) {
        const int rows = int(min(int64_t(a.R), L1 - int64_t(jb) * a.R));
        const int pb = (g - rg.g0) & 1;
        // One barrier per block, as in the statistics sweep.
        __syncthreads();
        if (s_abort) {
            ring_drain_span(rg, g - 1, g - 1 + kS);
            return;
        }
        if (g > rg.g0) {
            if (tid == 0 && g - 1 + kS < rg.g1) rg.issue(g - 1 + kS);
            if (pend) write_rdot(pb ^ 1, b, jb - 1, a.R);
        }
        if (b != cur) {   // no warp reads s_cm / s_ci between the barriers around these writes
            cur = b;
            window(a.lengths, b, L1, L2, l1, l2);
            for (int64_t col = tid; col < L2; col += kT) {
                const float2 c = __ldg(a.cstat + int64_t(b) * L2 + col);
                s_cm[col] = c.x * kLog2e;
                s_ci[col] = c.y;
            }
#pragma unroll
            for (int k = 0; k < NP; ++k) Sd[k] = make_float2(0.0f, 0.0f);
            __syncthreads();
        }
        if (!rg.wait(g)) s_abort = 1;
        const T* xs = reinterpret_cast<const T*>(rg.stage(g));
        const float* gs = reinterpret_cast<const float*>(rg.stage(g) + a.gout_off);
        for (int il = slot; il < rows; il += SLOTS) {
            const int64_t i = int64_t(jb) * a.R + il;
            float rd = 0.0f;
            if (i < l1) {   // warp-uniform
                const float2 rs = __ldg(a.rstat + int64_t(b) * L1 + i);
                const float2 nrmL = splat2(-(rs.x * kLog2e)), rinv = splat2(rs.y);
                const bool full = wide && l2 == L2;
                float2 rd2 = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int p = 0; p < VPLW; ++p) {
                    const int col = cbase + 4 * lane + 128 * p;
                    if (full || col < l2) {
                        float v[4], gv[4];
                        float2 cm[2], ci[2];
                        ld4s(xs + il * L2 + col, v);
                        ld4s(gs + il * L2 + col, gv);
                        cs4_pairs(s_cm + col, s_ci + col, cm, ci);
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            // q needs row * col only: the output sweep's expression
                            const float2 val = mul2(make_float2(v[2 * h], v[2 * h + 1]), splat2(a.invT));
                            const float2 rc = rowcol2(val, nrmL, rinv, cm[h], ci[h]);
                            const float2 x = add2(rc, splat2(1e-9f));
                            const float2 iout = make_float2(rsqrt_approx(x.x), rsqrt_approx(x.y));
                            float2 q = mul2(mul2(mul2(make_float2(gv[2 * h], gv[2 * h + 1]), splat2(0.5f)), iout), rc);
                            if (!full && col + 3 >= l2) {
                                if (col + 2 * h >= l2) q.x = 0.0f;
                                if (col + 2 * h + 1 >= l2) q.y = 0.0f;
                            }
                            rd2 = add2(rd2, q);
                            Sd[2 * p + h] = add2(Sd[2 * p + h], q);
                        }
                    }
                }
                rd = rd2.x + rd2.y;
                rd = warp_sum<32>(rd);
            }
            if (lane == 0) s_rd[pb][il][cpart] = rd;
        }
        pend = !(g + 1 == rg.g1 || jb + 1 == a.s.nblk);
        if (!pend) {
            __syncthreads();   // the stage is free; s_rd is complete
            write_rdot(pb, b, jb, rows);
            const int kfirst = sched_owner(a.s, b * a.s.nblk);
            const int nseg = sched_owner(a.s, (b + 1) * a.s.nblk - 1) - kfirst + 1;
            const int seg = int(blockIdx.x) - kfirst;
            float* mb = reinterpret_cast<float*>(rg.stage(g));   // [SLOTS][L2]
#pragma unroll
            for (int p = 0; p < VPLW; ++p) {
                const int64_t col = cbase + 4 * lane + 128 * p;
                if (col < L2) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 pr = Sd[2 * p + (e >> 1)];
                        mb[slot * L2 + col + e] = (e & 1) ? pr.y : pr.x;
                    }
                }
            }
            __syncthreads();
            float* mypart = static_cast<float*>(a.part) + (int64_t(b) * a.s.maxseg + seg) * L2;
            for (int64_t col = tid; col < L2; col += kT) {
                float ss = 0.0f;
#pragma unroll
                for (int q = 0; q < SLOTS; ++q) ss += mb[q * L2 + col];
                if (nseg == 1) a.cdot[int64_t(b) * L2 + col] = col < l2 ? ss : 0.0f;
                else mypart[col] = ss;
            }
            if (nseg > 1 && arrive_last(a.cnt, b, nseg, &s_flag)) {
                const float* pb = static_cast<const float*>(a.part) + int64_t(b) * a.s.maxseg * L2;
                for (int64_t col = tid; col < L2; col += kT) {
                    float ss = 0.0f;
                    for (int sg = 0; sg < nseg; ++sg) ss += __ldcg(pb + int64_t(sg) * L2 + col);
                    a.cdot[int64_t(b) * L2 + col] = col < l2 ? ss : 0.0f;
                }
                if (tid == 0) a.cnt[b] = 0;
            }
            fence_proxy_async_smem();   // merge-buffer writes before the next barrier and the refill
        }
        if (++jb == a.s.nblk) {
            jb = 0;
            ++b;
        }
    }
    __syncthreads();
    if (s_abort) ring_drain_span(rg, rg.g1 - 1, rg.g1);
}

// ---------------------------------------------------------------------------
// backward: gradient sweep over the dot sweep's ring
// ---------------------------------------------------------------------------
template <typename T, typename G, int VPL>
__global__ void __launch_bounds__(kT, 3) bs2_grad_kernel(SweepArgs a, G* __restrict__ gsim) {
    using W = WL<VPL>;
    constexpr int WPR = W::WPR, VPLW = W::VPLW, SLOTS = W::SLOTS;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[kS];
    __shared__ __align__(16) float s_cm[kMaxL2];   // the problem's columns: cmax
    __shared__ __align__(16) float s_ci[kMaxL2];   // and 1/sum
    __shared__ float s_tp[kMaxR][WPR];               // per-row tau partials of the row's warps

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int slot = wid / WPR, cpart = wid % WPR;
    const int cbase = cpart * 128 * VPLW;
    const int64_t L1 = a.L1, L2 = a.L2;
    const bool wide = L2 == 128 * VPL;
    const Ring rg = ring_start(a, bars, smem, true);
    pdl_wait();   // the first sweep's statistics / dots are complete and visible
    int64_t l1 = 0, l2 = 0;
    int cur = -1;

    for (int pos = rg.g0; pos < rg.g1; ++pos) {
        const int g = rg.block(pos);
        const int b = g / a.s.nblk, jb = g - b * a.s.nblk;
        if (b != cur) {   // the barrier below orders these writes before their reads
            cur = b;
            window(a.lengths, b, L1, L2, l1, l2);
            for (int64_t col = tid; col < L2; col += kT) {
                const float2 c = __ldg(a.cstat + int64_t(b) * L2 + col);
                s_cm[col] = c.x;
                s_ci[col] = c.y;
            }
        }
        const int rows = int(min(int64_t(a.R), L1 - int64_t(jb) * a.R));
        const bool ok = rg.wait(pos);
        if (!__syncthreads_and(ok)) {
            ring_drain(rg, pos);
            return;
        }
        const T* xs = reinterpret_cast<const T*>(rg.stage(pos));
        const float* gs = reinterpret_cast<const float*>(rg.stage(pos) + a.gout_off);
        const float* db = a.cdot + int64_t(b) * L2;
        for (int il = slot; il < rows; il += SLOTS) {
            const int64_t i = int64_t(jb) * a.R + il;
            const int64_t row = int64_t(b) * L1 + i;
            G* grow = gsim + row * L2;
            const bool live = i < l1;
            const float2 rs = live ? __ldg(a.rstat + row) : make_float2(0.0f, 0.0f);
            const float2 rmax = splat2(rs.x), rinv = splat2(rs.y);
            const float2 nrd = splat2(live ? -__ldg(a.rdot + row) : 0.0f);
            const float2 it = splat2(a.invT), lg = splat2(kLog2e);
            const bool full = wide && l2 == L2;
            float2 acc2 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int p = 0; p < VPLW; ++p) {
                const int col = cbase + 4 * lane + 128 * p;
                if (!full && col >= L2) continue;
                float gr[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (live && (full || col < l2)) {
                    float v[4], gv[4];
                    float2 cm[2], ci[2];
                    ld4s(xs + il * L2 + col, v);
                    ld4s(gs + il * L2 + col, gv);
                    cs4_pairs(s_cm + col, s_ci + col, cm, ci);
                    const float4 d4 = __ldg(reinterpret_cast<const float4*>(db + col));
                    const float2 cd[2] = {make_float2(d4.x, d4.y), make_float2(d4.z, d4.w)};
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        // row = exp(v - rmax) rinv, col = exp(v - cmax) cinv, out from
                        // one rsqrt of 1e-9 + row * col; 2q = g * (1/out) * row * col
                        const float2 val = mul2(make_float2(v[2 * h], v[2 * h + 1]), it);
                        const float2 rw = mul2(ex2x2(mul2(sub2(val, rmax), lg)), rinv);
                        const float2 cl = mul2(ex2x2(mul2(sub2(val, cm[h]), lg)), ci[h]);
                        const float2 rc = mul2(rw, cl);
                        const float2 x = add2(rc, splat2(1e-9f));
                        const float2 iout = make_float2(rsqrt_approx(x.x), rsqrt_approx(x.y));
                        const float2 q2 = mul2(mul2(make_float2(gv[2 * h], gv[2 * h + 1]), iout), rc);
                        float2 g2 = mul2(sub2(fma2(nrd, rw, q2), mul2(cd[h], cl)), it);
                        if (!full && col + 3 >= l2) {
                            if (col + 2 * h >= l2) g2.x = 0.0f;
                            if (col + 2 * h + 1 >= l2) g2.y = 0.0f;
                        }
                        acc2 = fma2(g2, val, acc2);
                        gr[2 * h] = g2.x;
                        gr[2 * h + 1] = g2.y;
                    }
                }
                st4g(grow + col, gr);
            }
            float acc = acc2.x + acc2.y;
            if (a.tau_row != nullptr) {
                acc = warp_sum<32>(acc);
                if (lane == 0) s_tp[il][cpart] = acc;
            }
        }
        __syncthreads();   // the stage is free; s_tp is complete
        if (a.tau_row != nullptr && tid < rows) {
            float acc = 0.0f;
#pragma unroll
            for (int c = 0; c < WPR; ++c) acc += s_tp[tid][c];
            a.tau_row[int64_t(b) * L1 + int64_t(jb) * a.R + tid] = acc;
        }
        __syncthreads();   // s_tp is read before the next block writes it
        if (tid == 0 && pos + kS < rg.g1) rg.issue(pos + kS);
    }
}

__global__ void bs2_batch_sum_kernel(const float* __restrict__ row_part, float* __restrict__ outv, int64_t B,
                                     int64_t n, float scale) {
    const int lane = threadIdx.x & 31;
    const int64_t b = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= B) return;
    float acc = 0.0f;
    for (int64_t i = lane; i < n; i += 32) acc += row_part[b * n + i];
    acc = warp_sum<32>(acc);
    if (lane == 0) outv[b] = acc * scale;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
size_t sweep_smem() { return size_t(kS) * kStage; }

int vpl_of(int64_t L2) { return L2 <= 128 ? 1 : L2 <= 256 ? 2 : L2 <= 512 ? 4 : 8; }

// Rows per block and the grad_out offset in a stage: as many rows as fit one
// stage (at most kMaxR), a multiple of the CTA's row slots where possible (no
// slot idles while another takes a second row), grad_out rows 128-byte
// aligned after the sim rows.
void block_shape(int64_t L2, int esz, bool with_grad, int& R, uint32_t& gout_off) {
    const int64_t per = L2 * esz + (with_grad ? L2 * 4 : 0);
    int64_t r = std::min<int64_t>(kStage / per, kMaxR);
    auto off = [&](int64_t rr) { return (rr * L2 * esz + 127) / 128 * 128; };
    while (r > 1 && with_grad && off(r) + r * L2 * 4 > kStage) --r;
    const int64_t slots = vpl_of(L2) >= 8 ? kW / 2 : kW;
    if (r > slots) r = r / slots * slots;
    R = int(std::max<int64_t>(r, 1));
    gout_off = with_grad ? uint32_t(off(R)) : 0u;
}

int sm_count_now() {
    static int cached[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n < 1) n = 1;
    if (dev >= 0 && dev < 64) cached[dev] = n;
    return n;
}

template <typename K>
int resident_ctas(K kernel) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sweep_smem()));
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kernel, kT, sweep_smem()) != cudaSuccess || nb < 1) {
        cudaGetLastError();
        nb = 1;
    }
    return nb * sm_count_now();
}

// CTAs per launch of the ring sweeps: the resident capacity of the
// (fp32, VPL = 8) variant, cached per device; every variant holds at least as
// many (same shared memory, no more registers).
int ring_slots(bool bwd) {
    static int cached[2][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const int k = bwd ? 1 : 0;
    if (dev >= 0 && dev < 64 && cached[k][dev] > 0) return cached[k][dev];
    const int v = bwd ? resident_ctas(bs2_dots_kernel<float, 8>) : resident_ctas(bs2_stats_kernel<float, 8>);
    if (dev >= 0 && dev < 64) cached[k][dev] = v;
    return v;
}

Sched make_sched(int64_t B, int64_t L1, int R, bool bwd) {
    Sched s;
    s.nblk = int((L1 + R - 1) / R);
    s.T = int(B * s.nblk);
    s.G = int(std::min<int64_t>(s.T, ring_slots(bwd)));
    s.maxseg = 1;
    for (int b = 0; b < int(B); ++b) {
        const int k0 = sched_owner(s, b * s.nblk), k1 = sched_owner(s, (b + 1) * s.nblk - 1);
        s.maxseg = std::max(s.maxseg, k1 - k0 + 1);
    }
    return s;
}

// Most segments over both element sizes (the workspace query has no dtype).
int maxseg_any(int64_t B, int64_t L1, int64_t L2, bool bwd) {
    int ms = 1;
    for (int esz : {2, 4}) {
        int R;
        uint32_t off;
        block_shape(L2, esz, bwd, R, off);
        ms = std::max(ms, make_sched(B, L1, R, bwd).maxseg);
    }
    return ms;
}

struct FwdWs {
    int32_t* err;
    int32_t* cnt;
    float2* part;
};
FwdWs carve_fwd(Carve& c, int64_t B, int64_t L1, int64_t L2) {
    FwdWs w;
    w.err = c.take<int32_t>(1);
    w.cnt = c.take<int32_t>(size_t(B));
    w.part = c.take<float2>(size_t(B * maxseg_any(B, L1, L2, false) * L2));
    return w;
}

struct BwdWs {
    int32_t* err;
    int32_t* cnt;
    float* part;
    float* rdot;
    float* cdot;
    float* tau_row;
};
BwdWs carve_bwd(Carve& c, int64_t B, int64_t L1, int64_t L2) {
    BwdWs w;
    w.err = c.take<int32_t>(1);
    w.cnt = c.take<int32_t>(size_t(B));
    w.part = c.take<float>(size_t(B * maxseg_any(B, L1, L2, true) * L2));
    w.rdot = c.take<float>(size_t(B * L1));
    w.cdot = c.take<float>(size_t(B * L2));
    w.tau_row = c.take<float>(size_t(B * L1));
    return w;
}

SweepArgs sweep_args(const void* sim, int esz, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau,
                     const float* gout) {
    SweepArgs a{};
    a.sim = static_cast<const unsigned char*>(sim);
    a.gout = gout;
    a.lengths = lengths;
    a.L1 = L1;
    a.L2 = L2;
    a.esz = esz;
    block_shape(L2, esz, gout != nullptr, a.R, a.gout_off);
    a.s = make_sched(B, L1, a.R, gout != nullptr);
    a.invT = 1.0f / tau;
    return a;
}

// Launch of a second sweep with programmatic dependent launch: its CTAs may
// start (barrier set-up, first copies of the read-only input) while the first
// sweep finishes; they wait for it before reading its results.
template <typename K, typename... Args>
void launch_dependent(K kernel, int grid, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(grid));
    cfg.blockDim = dim3(kT);
    cfg.dynamicSmemBytes = sweep_smem();
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <typename T, int VPL>
int fwd_impl(const T* sim, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau, float* out,
             float2* rstat, float2* cstat, void* ws, cudaStream_t st) {
    SweepArgs a = sweep_args(sim, sizeof(T), lengths, B, L1, L2, tau, nullptr);
    Carve cv(ws);
    FwdWs w = carve_fwd(cv, B, L1, L2);
    a.rstat = rstat;
    a.cstat = cstat;
    a.part = w.part;
    a.cnt = w.cnt;
    a.err = w.err;
    cudaMemsetAsync(w.err, 0, sizeof(int32_t), st);
    cudaMemsetAsync(w.cnt, 0, sizeof(int32_t) * size_t(B), st);
    cudaFuncSetAttribute(bs2_stats_kernel<T, VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sweep_smem()));
    a.out = out;
    cudaFuncSetAttribute(bs2_out_kernel<T, VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sweep_smem()));
    ProfScope ps(DOT_K_BS_FWD, st, 2);
    bs2_stats_kernel<T, VPL><<<unsigned(a.s.G), kT, sweep_smem(), st>>>(a);
    launch_dependent(bs2_out_kernel<T, VPL>, a.s.G, st, a);
    return check_launch("bidirectional softmax forward");
}

template <typename T, typename G, int VPL>
int bwd_impl(const T* sim, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau, const float2* rstat,
             const float2* cstat, const float* gout, G* gsim, float* gtau, void* ws, cudaStream_t st) {
    SweepArgs a = sweep_args(sim, sizeof(T), lengths, B, L1, L2, tau, gout);
    Carve cv(ws);
    BwdWs w = carve_bwd(cv, B, L1, L2);
    a.rstat = const_cast<float2*>(rstat);
    a.cstat = const_cast<float2*>(cstat);
    a.rdot = w.rdot;
    a.cdot = w.cdot;
    a.part = w.part;
    a.cnt = w.cnt;
    a.err = w.err;
    cudaMemsetAsync(w.err, 0, sizeof(int32_t), st);
    cudaMemsetAsync(w.cnt, 0, sizeof(int32_t) * size_t(B), st);
    a.tau_row = gtau ? w.tau_row : nullptr;
    cudaFuncSetAttribute(bs2_dots_kernel<T, VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sweep_smem()));
    cudaFuncSetAttribute(bs2_grad_kernel<T, G, VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(sweep_smem()));
    {
        ProfScope ps(DOT_K_BS_BWD, st, 2);
        bs2_dots_kernel<T, VPL><<<unsigned(a.s.G), kT, sweep_smem(), st>>>(a);
        launch_dependent(bs2_grad_kernel<T, G, VPL>, a.s.G, st, a, gsim);
    }
    if (gtau != nullptr) {
        ProfScope ps(DOT_K_BS_BWD, st);
        bs2_batch_sum_kernel<<<unsigned(ceil_div(B, 8)), 256, 0, st>>>(w.tau_row, gtau, B, L1, -1.0f);
    }
    return check_launch("bidirectional softmax backward");
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

bool bsf_supported(int64_t B, int64_t L1, int64_t L2, int dtype, const void* sim, const void* gout, const void* dst,
                   int dst_dtype) {
    auto aligned = [](const void* p, uintptr_t a) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) % a) == 0; };
    if (L2 < 4 || L2 > kMaxL2 || L1 < 1 || B < 1) return false;
    if (dtype == DOT_F32 ? (L2 % 4) != 0 : (L2 % 8) != 0) return false;
    const int esz = dtype == DOT_F32 ? 4 : 2;
    int R;
    uint32_t off;
    block_shape(L2, esz, gout != nullptr, R, off);
    if (B * ((L1 + R - 1) / R) >= (int64_t(1) << 31)) return false;   // block indices are 32-bit
    return aligned(sim, 16) && aligned(gout, 16) && aligned(dst, dst_dtype == DOT_F32 ? 16 : 8);
}

size_t bsf_fwd_ws(int64_t B, int64_t L1, int64_t L2) {
    if (L2 < 4 || L2 > kMaxL2 || L1 < 1 || B < 1) return 0;
    Carve c(nullptr);
    carve_fwd(c, B, L1, L2);
    return c.size();
}

size_t bsf_bwd_ws(int64_t B, int64_t L1, int64_t L2) {
    if (L2 < 4 || L2 > kMaxL2 || L1 < 1 || B < 1) return 0;
    Carve c(nullptr);
    carve_bwd(c, B, L1, L2);
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

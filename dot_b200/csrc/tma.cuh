// Bulk-copy (TMA engine) and mbarrier helpers for sm_100a, written as inline PTX.
//
// Every wait is bounded: a wait that does not complete within the spin limit
// records an error code in a caller-provided device word and returns false,
// so a kernel never hangs the GPU on a lost copy.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace dotb {

// Error codes written to the status word by bounded waits.
constexpr int kErrBarrierTimeout = 0x100;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}

// 1-D bulk copy global -> shared, completion signalled on `bar` (bytes and
// both addresses must be multiples of 16).
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` to complete.  Spins, then backs off with
// nanosleep; gives up after ~2^22 polls (well over 100 ms), records
// kErrBarrierTimeout in *err and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* err) {
    for (uint32_t i = 0; i < (1u << 22); ++i) {
        if (mbar_test(bar, parity)) return true;
        if (i > 64) __nanosleep(64);
    }
    if (err != nullptr) atomicOr(err, kErrBarrierTimeout);
    return false;
}

}  // namespace dotb

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

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
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

// L2 eviction-priority policies (createpolicy) for bulk copies: evict_last
// keeps a line resident across launches that stream the same matrix again;
// evict_first marks a line that will not be read again soon.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// bulk_g2s with an L2 cache-policy operand (no multicast).
__device__ __forceinline__ void bulk_g2s_hint(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) accesses to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Programmatic dependent launch (sm_90+).  launch_dependents lets the next
// kernel in the stream be scheduled once every CTA of this grid has issued it
// (or exited); wait blocks until the preceding grid has completed and its
// memory is visible.  Before wait a kernel may only read data that the
// preceding grid does not write.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// One bounded hardware wait: the thread may be suspended until the phase
// completes or about kSuspendNs elapse.
constexpr uint32_t kSuspendNs = 4000;
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` with suspending try_wait; gives up after
// 2^19 attempts (between ~10 ms and ~2 s), records kErrBarrierTimeout in *err
// and returns false.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, int32_t* err) {
    for (uint32_t i = 0; i < (1u << 19); ++i) {
        if (mbar_try(bar, parity)) return true;
    }
    if (err != nullptr) atomicOr(err, kErrBarrierTimeout);
    return false;
}

// mbar_try / mbar_wait_sleep with cluster-scope acquire: for phases completed
// by stores from other CTAs of the cluster (st.async below).
__device__ __forceinline__ bool mbar_try_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int32_t* err) {
    for (uint32_t i = 0; i < (1u << 19); ++i) {
        if (mbar_try_cluster(bar, parity)) return true;
    }
    if (err != nullptr) atomicOr(err, kErrBarrierTimeout);
    return false;
}

// Address of the same shared-memory object in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t cluster_map(const void* local, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(local)), "r"(rank));
    return a;
}

// Store a float2 into another CTA's shared memory (cluster addresses from
// cluster_map); its 8 bytes complete a transaction on that CTA's mbarrier.
__device__ __forceinline__ void st_async_f2(uint32_t remote_addr, uint32_t remote_bar, float2 v) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
                     remote_addr),
                 "f"(v.x), "f"(v.y), "r"(remote_bar)
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

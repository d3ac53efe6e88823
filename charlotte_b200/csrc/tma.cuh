// Bulk asynchronous copies (TMA, untiled cp.async.bulk) into shared memory,
// completed on mbarriers, and the bounded waits that guard them.
//
// Every wait here is bounded: after kSpinLimit polls it records a timeout in
// the launch's fault word (read back by the host as a step failure) and
// gives up, so no kernel of this library can spin forever on a copy that
// never lands.
#pragma once

#include <cstdint>

namespace cb {

constexpr uint32_t kSpinLimit = 1u << 24;   // polls (each can suspend ~hundreds of ns): seconds at most
constexpr uint32_t kFaultTimeout = 1u;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes mbarrier inits visible to the async proxy (the copy engine).
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) accesses of the same memory.
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// The same for global memory (a row this thread stored that a bulk copy
// will read).
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// Raises the current phase's expected transaction bytes without arriving
// (copies issued now; the arrival comes later with the rest of the phase).
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// The polls a kernel's first wait on a copy may take: the word after the
// device's fault word holds 1 + a shorter bound when a test set one
// (cb_debug_spin_limit, so a wait can be made to run out), else 0 for the
// full bound. Read at run time, so a captured graph follows it too.
__device__ __forceinline__ uint32_t spin_limit_of(const unsigned int* fault) {
    const uint32_t v = fault ? fault[1] : 0u;
    return v ? v - 1u : kSpinLimit;
}

// Waits for the phase of `parity` to complete; false (and the fault word
// set) if it did not within `limit` polls. The wait that drains a CTA's
// copies before it leaves always takes the full bound.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* fault,
                                          uint32_t limit = kSpinLimit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (fault) atomicOr(fault, kFaultTimeout);
    return false;
}

// Global -> shared bulk copy of `bytes` (a multiple of 16; both addresses
// 16-byte aligned), completing `bytes` transactions on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// 16 bytes global -> shared, asynchronous, through L2 only (coherent with
// writes of a grid this one waited on); completed by cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// An arrival on `bar` once every cp.async this thread issued so far has
// landed (the arrival counts toward the barrier's expected count).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Thread-block clusters: this CTA's rank and the cluster's size; a shared
// address of this CTA mapped to the same offset in CTA `rank`'s shared
// memory, and a 32-bit store there; a barrier over the whole cluster that
// also orders shared-memory writes before it with reads after it.
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t n;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
    return n;
}
__device__ __forceinline__ uint32_t cluster_map(const void* p, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_addr(p)), "r"(rank));
    return a;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

}  // namespace cb

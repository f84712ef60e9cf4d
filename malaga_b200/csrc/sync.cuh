// Asynchronous copies and bounded waits shared by the TMA-fed kernels (sm_100a).
//
// Every wait on an mbarrier is bounded by %globaltimer: after kWaitNs of device
// time the waiter gives up, the kernel records a flag in the engine's device
// error word and stops, and the host turns the flag into MGB_ERR_CUDA.
#pragma once
#include <stdint.h>

namespace mgb {

constexpr uint64_t kWaitNs = 500000000ull;  // give up a wait after 0.5 s of device time

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// 1-D bulk copy global -> shared (both 16-byte aligned, bytes a multiple of
// 16), completion counted on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// One arrival on an mbarrier (no transaction bytes).
__device__ __forceinline__ void mbar_arrive_cta(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// L2 prefetch of [p, p + bytes), rounded out to 16-byte bounds.
__device__ __forceinline__ void prefetch_l2(const void *p, size_t bytes) {
    uint64_t lo = (uint64_t)p & ~15ull, hi = ((uint64_t)p + bytes + 15) & ~15ull;
    while (lo < hi) {
        const uint64_t n = (hi - lo) > (1ull << 30) ? (1ull << 30) : (hi - lo);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lo), "r"((uint32_t)n) : "memory");
        lo += n;
    }
}

// One try_wait: a thread whose phase is not complete may sleep until it
// completes (or a time limit runs out: MGB_WAIT_HINT_NS when nonzero, else the
// hardware's own) instead of spinning, so waiting warps do not take issue
// slots from working ones.
#ifndef MGB_WAIT_HINT_NS
#define MGB_WAIT_HINT_NS 0
#endif
__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
    uint32_t done;
#if MGB_WAIT_HINT_NS > 0
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity), "r"((uint32_t)MGB_WAIT_HINT_NS)
        : "memory");
#else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
#endif
    return done != 0;
}

// Bounded wait for phase `parity` of the mbarrier; false once `limit_ns` passed.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t limit_ns = kWaitNs) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try(a, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (;;) {
        if (mbar_try(a, parity)) return true;
        if (globaltimer() - t0 > limit_ns) return false;
    }
}

// Thread-block clusters: this CTA's rank and the cluster size; a full cluster
// barrier (hardware; every thread of every CTA of the cluster arrives, release /
// acquire ordering of shared-memory writes across the cluster).
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Stores into the shared memory of CTA `rank` of the cluster at the offset of
// this CTA's shared address `a` (distributed shared memory).
__device__ __forceinline__ void st_cluster_u8(uint32_t a, uint32_t rank, uint32_t v) {
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
    asm volatile("st.shared::cluster.u8 [%0], %1;" ::"r"(ra), "r"(v) : "memory");
}

__device__ __forceinline__ void st_cluster_f32(uint32_t a, uint32_t rank, float v) {
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}

}  // namespace mgb

// cluster.cuh -- thread-block cluster helpers (sm_90+): the cluster barrier
// halves, mapping a shared-memory address into another CTA of the cluster,
// stores into distributed shared memory, and the proxy fence that orders
// generic accesses of shared memory before later bulk copies into it.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace styx {

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// cluster barrier halves; every thread of every CTA of the cluster takes part
__device__ __forceinline__ void cl_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cl_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cl_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// the shared-memory address `saddr` of this CTA, in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t cl_map(uint32_t saddr, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(saddr), "r"(rank));
    return a;
}
__device__ __forceinline__ void cl_st(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
// orders this thread's generic-proxy accesses of shared memory before later
// bulk copies into the same bytes
__device__ __forceinline__ void fence_proxy_async_cta() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

}  // namespace styx

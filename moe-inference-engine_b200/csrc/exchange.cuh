// Device-wide exchange words and thread-block-cluster primitives of the
// persistent decode steps (sm_100a).
//
// An exchange word is one 64-bit value {f32 payload, u32 tag} written with a
// single 64-bit store: a consumer that polls the word sees either the old tag
// or the new value together with its tag, so a word is complete the moment its
// tag is visible and needs no fence, counter or barrier.
//
// Inside a cluster, CTAs hand values to each other through distributed shared
// memory: a store to a peer's shared memory (st.shared::cluster at an address
// from mapa) followed by the cluster barrier (arrive.release / wait.acquire),
// after which every CTA reads what its peers wrote into its own shared memory.
#pragma once

#include <stdint.h>

namespace mie {

__device__ __forceinline__ void ll_put(uint64_t* p, float v, uint32_t tag) {
  const uint64_t w = ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ll_ld(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// The same words across GPUs (system scope): a store into a peer's memory
// through an IPC mapping, and the poll of this GPU's own copy.
__device__ __forceinline__ void ll_put_sys(uint64_t* p, float v, uint32_t tag) {
  const uint64_t w = ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ll_ld_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ll_tag(uint64_t w) { return (uint32_t)(w >> 32); }
__device__ __forceinline__ float ll_val(uint64_t w) { return __uint_as_float((uint32_t)w); }

// ---- clusters ----
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster: the release half orders this CTA's
// earlier shared-memory stores (local and remote) before the acquire half of
// every peer.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared-memory address (shared::cta window) -> the same offset in CTA `rank`
// of this cluster (shared::cluster window).
__device__ __forceinline__ uint32_t dsmem_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(r)
               : "r"((uint32_t)__cvta_generic_to_shared(local)), "r"(rank));
  return r;
}
__device__ __forceinline__ void dsmem_st(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void dsmem_st4(uint32_t addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

}  // namespace mie

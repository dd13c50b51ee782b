// Thread-block cluster helpers (sm_90+): the CTA's rank in its cluster,
// cluster barriers, and loads from another CTA's shared memory (distributed
// shared memory).  Used by the kernels that combine partial results across
// the CTAs of a cluster instead of through a global workspace.
#pragma once

#include <cstdint>

namespace tvr {

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA of the cluster arrives; shared-memory writes
// before it are visible to the cluster's CTAs after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ uint32_t smem_addr_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

__device__ __forceinline__ float ld_dsmem(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ int64_t ld_dsmem_s64(uint32_t addr) {
  int64_t v;
  asm volatile("ld.shared::cluster.s64 %0, [%1];" : "=l"(v) : "r"(addr));
  return v;
}

}  // namespace tvr

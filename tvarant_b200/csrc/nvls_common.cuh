// Device-side pieces shared by the kernels that sum over ranks through NVLink
// SHARP: the in-place all-reduce (nvls.cu) and the GEMM whose epilogue feeds
// that reduction tile by tile (gemm_tc.cu, NVLS instances).
//
//   * flags in every rank's memory, written with system-scope release stores
//     or reductions and read with system-scope acquire loads, every wait
//     bounded (TVR_DEV_TIMEOUT_PEER in the device status word on expiry);
//   * multimem.ld_reduce (the switch reads every rank's copy and adds) and
//     multimem.st (the switch writes every rank's copy) through a buffer's
//     multicast address.
//
// One rank's flag array (TVR_NVLS_FLAG_WORDS uint32, zero when first used):
// barrier words [3 phases][TVR_NVLS_MAX_BLOCKS slots][TVR_NVLS_MAX_RANKS
// source ranks] (phases 0 and 1: the all-reduce's two barriers; 2: the fused
// GEMM's closing barrier), then TVR_NVLS_MAX_TILES per-tile arrival counters.
// Barrier words hold the epoch of the last call that passed them, so they
// never need resetting; a tile counter is reset by the rank that reduced the
// tile, before that rank's closing barrier.
//
// No load here uses TMA or cluster multicast.
#pragma once

#include "internal.h"

namespace tvr {
namespace nvls {

constexpr unsigned long long kPeerTimeoutNs = 2000000000ull;  // 2 s per wait
constexpr int kBarrierWords = 3 * TVR_NVLS_MAX_BLOCKS * TVR_NVLS_MAX_RANKS;
constexpr int kTileCounters = kBarrierWords;  // first tile counter
static_assert(kBarrierWords + TVR_NVLS_MAX_TILES == TVR_NVLS_FLAG_WORDS, "flag layout");

struct PeerFlags {
  uint32_t* flags[TVR_NVLS_MAX_RANKS];  // each rank's flag array, by its address here
};

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void store_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void red_release_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ float4 multimem_ld_reduce_add(const float* mc) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

__device__ __forceinline__ void multimem_st(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

// Barrier word of (phase, slot, source rank) in a rank's flag array.
__device__ __forceinline__ size_t flag_index(int phase, int slot, int src) {
  return (static_cast<size_t>(phase) * TVR_NVLS_MAX_BLOCKS + slot) * TVR_NVLS_MAX_RANKS + src;
}

// Waits until *p >= target (acquire, system scope).  Returns false after
// kPeerTimeoutNs, having recorded TVR_DEV_TIMEOUT_PEER.
__device__ __forceinline__ bool wait_at_least(const uint32_t* p, uint32_t target, int* status) {
  if (load_acquire_sys(p) >= target) return true;
  const unsigned long long t0 = now_ns();
  unsigned polls = 0;
  while (load_acquire_sys(p) < target) {
    if ((++polls & 63u) == 0 && now_ns() - t0 > kPeerTimeoutNs) {
      atomicCAS(status, TVR_DEV_OK, TVR_DEV_TIMEOUT_PEER);
      return false;
    }
  }
  return true;
}

// The CTAs with the same `slot` on every rank meet: thread t < world
// publishes `epoch` into rank t's word (phase, slot, rank) and waits for this
// rank's word (phase, slot, t).  Everything the CTA wrote before is visible
// to every rank before its flag is.  Returns false for the whole CTA when a
// wait expired.
__device__ __forceinline__ bool rank_barrier(const PeerFlags& pf, int rank, int world, int phase,
                                             int slot, uint32_t epoch, int* status,
                                             int* expired) {
  __syncthreads();
  const int t = threadIdx.x;
  if (t < world) {
    fence_sys();
    store_release_sys(pf.flags[t] + flag_index(phase, slot, rank), epoch);
    if (!wait_at_least(pf.flags[rank] + flag_index(phase, slot, t), epoch, status)) *expired = 1;
  }
  __syncthreads();
  return *expired == 0;
}

}  // namespace nvls
}  // namespace tvr

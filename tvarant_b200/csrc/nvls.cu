// In-place sum all-reduce of fp32 through NVLink SHARP: the NVSwitch reads
// and adds every rank's copy (multimem.ld_reduce) and writes the sum back to
// every rank (multimem.st).
//
// The buffer is bound to a multicast object: the same offset in it names
// each rank's copy, and the multicast address names all of them at once.
// Rank r reduces the r-th of `world` equal slices, so each GPU sends its
// whole buffer to the switch once (answering the reads of all ranks) and
// receives the whole sum once.  That is half of what a ring all-reduce
// moves over a GPU's links.
//
// Ordering across ranks uses flags in every rank's memory (peer stores with
// release semantics, local loads with acquire semantics).  Block b of every
// rank meets block b of every other rank twice.  The first barrier ensures
// all ranks' inputs are written before any rank reads through the switch.
// The second ensures every rank's stores are done before any rank returns
// (and reads or rewrites its copy).  Every wait is bounded: past the limit
// the block records TVR_DEV_TIMEOUT_PEER in the device status word and
// returns, so a missing rank ends the kernel instead of hanging the GPU.
//
// The reference has one device and no collectives; this serves the
// tensor-parallel MLP stack (tvarant_b200/tp.py).  No load here uses TMA or
// cluster multicast; multimem accesses go through the NVSwitch.
#include "internal.h"

namespace tvr {
namespace {

constexpr int kThreads = 512;
constexpr int kUnroll = 4;
constexpr unsigned long long kPeerTimeoutNs = 2000000000ull;  // 2 s per barrier

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

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

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

// Flag word of (phase, block, source rank) in a rank's flag array.
__device__ __forceinline__ size_t flag_index(int phase, int block, int src) {
  return (static_cast<size_t>(phase) * TVR_NVLS_MAX_BLOCKS + block) * TVR_NVLS_MAX_RANKS + src;
}

// Block b meets block b of every rank: thread t < world publishes `epoch`
// into rank t's slot (phase, b, rank) and waits for this rank's slot
// (phase, b, t).  Returns false for the whole block when a wait expired.
__device__ bool rank_barrier(const PeerFlags& pf, int rank, int world, int phase, uint32_t epoch,
                             int* status, int* expired) {
  __syncthreads();
  const int t = threadIdx.x;
  if (t < world) {
    // everything this block (and, by the kernel boundary, this stream) wrote
    // before is visible to every rank before the flag is
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    store_release_sys(pf.flags[t] + flag_index(phase, blockIdx.x, rank), epoch);
    const uint32_t* mine = pf.flags[rank] + flag_index(phase, blockIdx.x, t);
    if (load_acquire_sys(mine) < epoch) {
      const unsigned long long t0 = now_ns();
      unsigned polls = 0;
      while (load_acquire_sys(mine) < epoch) {
        if ((++polls & 63u) == 0 && now_ns() - t0 > kPeerTimeoutNs) {
          atomicCAS(status, TVR_DEV_OK, TVR_DEV_TIMEOUT_PEER);
          *expired = 1;
          break;
        }
      }
    }
  }
  __syncthreads();
  return *expired == 0;
}

// Advances the call counter: one launch before each all-reduce, so that
// every replay of a captured graph uses a fresh epoch.
__global__ void nvls_next_epoch_kernel(uint32_t* counter) { *counter += 1; }

__global__ void __launch_bounds__(kThreads)
    nvls_all_reduce_kernel(float* mc, int64_t per_rank, const __grid_constant__ PeerFlags pf,
                           int rank, int world, const uint32_t* counter, int* status) {
  __shared__ int expired;
  if (threadIdx.x == 0) expired = 0;
  const uint32_t epoch = *counter;
  if (!rank_barrier(pf, rank, world, 0, epoch, status, &expired)) return;
  float* slice = mc + static_cast<int64_t>(rank) * per_rank;
  const int64_t n4 = per_rank / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = multimem_ld_reduce_add(slice + 4 * (i + u * stride));
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) multimem_st(slice + 4 * (i + u * stride), v[u]);
  }
  for (; i < n4; i += stride) multimem_st(slice + 4 * i, multimem_ld_reduce_add(slice + 4 * i));
  rank_barrier(pf, rank, world, 1, epoch, status, &expired);
}

}  // namespace
}  // namespace tvr

using namespace tvr;

extern "C" int tvr_nvls_all_reduce_f32(void* multicast, int64_t count, void* const* peer_flags,
                                       int rank, int world, uint32_t* epoch_counter, int blocks,
                                       void* stream) {
  TVR_CHECK(world >= 2 && world <= TVR_NVLS_MAX_RANKS, "nvls_all_reduce: world %d (2..%d)", world,
            TVR_NVLS_MAX_RANKS);
  TVR_CHECK(rank >= 0 && rank < world, "nvls_all_reduce: rank %d of %d", rank, world);
  TVR_CHECK(count >= 0 && count % (4 * world) == 0,
            "nvls_all_reduce: count %lld is not a multiple of 4 x %d ranks", (long long)count,
            world);
  TVR_CHECK(blocks >= 1 && blocks <= TVR_NVLS_MAX_BLOCKS, "nvls_all_reduce: %d blocks (1..%d)",
            blocks, TVR_NVLS_MAX_BLOCKS);
  TVR_CHECK(epoch_counter != nullptr && reinterpret_cast<uintptr_t>(epoch_counter) % 4 == 0,
            "nvls_all_reduce: null or unaligned epoch counter");
  TVR_CHECK(multicast != nullptr && reinterpret_cast<uintptr_t>(multicast) % 16 == 0,
            "nvls_all_reduce: multicast address must be non-null and 16-byte aligned");
  TVR_CHECK(peer_flags != nullptr, "nvls_all_reduce: null flag array");
  PeerFlags pf;
  memset(&pf, 0, sizeof(pf));
  for (int r = 0; r < world; ++r) {
    TVR_CHECK(peer_flags[r] != nullptr && reinterpret_cast<uintptr_t>(peer_flags[r]) % 4 == 0,
              "nvls_all_reduce: flag array of rank %d is null or unaligned", r);
    pf.flags[r] = static_cast<uint32_t*>(peer_flags[r]);
  }
  if (count == 0) return TVR_OK;  // (the epoch does not advance)
  const int dev = current_device();
  int* status = device_status_ptr(dev);
  TVR_CHECK(status != nullptr, "nvls_all_reduce: device status word unavailable");
  cudaStream_t s = as_stream(stream);
  nvls_next_epoch_kernel<<<1, 1, 0, s>>>(epoch_counter);
  TVR_LAUNCH_CHECK();
  nvls_all_reduce_kernel<<<blocks, kThreads, 0, s>>>(static_cast<float*>(multicast),
                                                      count / world, pf, rank, world,
                                                      epoch_counter, status);
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

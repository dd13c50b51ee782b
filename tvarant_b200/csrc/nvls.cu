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
#include "nvls_common.cuh"

#include "gemm_common.cuh"

namespace tvr {
namespace {

using namespace nvls;

constexpr int kThreads = 512;
constexpr int kUnroll = 4;

// Advances the call counter: one launch before each all-reduce, so that
// every replay of a captured graph uses a fresh epoch.
__global__ void nvls_next_epoch_kernel(uint32_t* counter) { *counter += 1; }

__global__ void __launch_bounds__(kThreads)
    nvls_all_reduce_kernel(float* mc, int64_t per_rank, const __grid_constant__ PeerFlags pf,
                           int rank, int world, const uint32_t* counter, int* status) {
  __shared__ int expired;
  if (threadIdx.x == 0) expired = 0;
  const uint32_t epoch = *counter;
  if (!rank_barrier(pf, rank, world, 0, blockIdx.x, epoch, status, &expired)) return;
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
  rank_barrier(pf, rank, world, 1, blockIdx.x, epoch, status, &expired);
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

extern "C" int tvr_gemm_nvls_all_reduce_f32(const float* a, const float* b, float* c,
                                            void* c_multicast, int64_t m, int64_t n, int64_t k,
                                            int64_t lda, int64_t ldb, int64_t ldc,
                                            void* const* peer_flags, int rank, int world,
                                            uint32_t* epoch_counter, int reduce_ctas,
                                            void* stream) {
  TVR_CHECK(world >= 2 && world <= TVR_NVLS_MAX_RANKS, "gemm_nvls_all_reduce: world %d (2..%d)",
            world, TVR_NVLS_MAX_RANKS);
  TVR_CHECK(rank >= 0 && rank < world, "gemm_nvls_all_reduce: rank %d of %d", rank, world);
  TVR_CHECK(m >= 0 && n >= 0 && k >= 0, "gemm_nvls_all_reduce: negative size");
  TVR_CHECK(a != nullptr && b != nullptr && c != nullptr && c_multicast != nullptr,
            "gemm_nvls_all_reduce: null operand");
  TVR_CHECK(epoch_counter != nullptr && reinterpret_cast<uintptr_t>(epoch_counter) % 4 == 0,
            "gemm_nvls_all_reduce: null or unaligned epoch counter");
  TVR_CHECK(peer_flags != nullptr, "gemm_nvls_all_reduce: null flag array");
  for (int r = 0; r < world; ++r) {
    TVR_CHECK(peer_flags[r] != nullptr && reinterpret_cast<uintptr_t>(peer_flags[r]) % 4 == 0,
              "gemm_nvls_all_reduce: flag array of rank %d is null or unaligned", r);
  }
  // (the shape checks, the epoch advance and the launch: gemm_tc.cu)
  return gemm_tcgen05_nvls(a, b, c, c_multicast, m, n, k, lda, ldb, ldc, peer_flags, rank, world,
                           epoch_counter, reduce_ctas, as_stream(stream));
}

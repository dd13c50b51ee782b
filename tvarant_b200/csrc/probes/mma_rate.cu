// Rate of tcgen05.mma kind::tf32 instructions by shape, the measurement behind
// the attention kernel's block schedule.  One thread per CTA issues `iters`
// MMAs (M=128, K=8, N in {64, 128, 256}) into one TMEM accumulator, with A
// from shared or tensor memory and B K-major or N-major, on 148 CTAs (one per
// SM) and on 296 (two per SM, sharing the tensor core); it prints the time per
// instruction and how long the issuing thread itself took (the MMA queue is
// shallow, so issue keeps pace with execution).  The last rows put a
// tcgen05.commit after every 8 MMAs, with and without a wait for it.  Operands are zeroed shared
// and tensor memory; every address stays inside the CTA's own buffers and the
// one completion wait is bounded.
//
//   nvcc -O3 -std=c++17 -gencode arch=compute_100a,code=sm_100a \
//        -I tvarant_b200/csrc -I include -o mma_rate tvarant_b200/csrc/probes/mma_rate.cu -lcuda
#include "tc_ptx.cuh"
#include <cstdio>
#include <vector>
#include <algorithm>
using namespace tvr::tc;

constexpr int SMEM = 1024 + 16384 + 32768 + 64;

// COMMIT: 0 = no commits, 1 = a tcgen05.commit after every 8 MMAs (to an
// mbarrier nobody waits on), 2 = the same commit and a wait for it
// (mbarrier.try_wait, which may suspend the thread), 3 = the commit and a
// spin on mbarrier.test_wait (bounded by a poll count), 4 = the commit and
// a wait in try_wait polls that suspend for at most 32 ns each.
template <int N, bool A_TMEM, bool B_NMAJOR, int COMMIT = 0>
__global__ void __launch_bounds__(128) mma_probe(unsigned long long* out, int iters) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t s_bar;
  __shared__ uint64_t s_step;
  __shared__ uint32_t s_tmem;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t sa = base, sb = base + 16384;
  const int warp = threadIdx.x >> 5;
  float* fz = reinterpret_cast<float*>(smem_raw + (base - raw));
  for (int i = threadIdx.x; i < (16384 + 32768) / 4; i += blockDim.x) fz[i] = 0.f;
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  const uint32_t bar = smem_u32(&s_bar);
  const uint32_t step = smem_u32(&s_step);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    mbar_init(step, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)), "r"(256u) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  if (A_TMEM) {  // zero A columns 128..159 of this warp's 32 lanes
    float z[32];
    for (int i = 0; i < 32; ++i) z[i] = 0.f;
    tmem_store_32(tmem + (static_cast<uint32_t>(32 * warp) << 16) + 128, z);
    tmem_wait_stores();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) {
    constexpr uint32_t idesc = idesc_tf32(128, N, B_NMAJOR);
    const unsigned long long t0 = global_ns();
    for (int it = 0; it < iters; ++it) {
      const uint32_t k32 = (it & 3) * 32;
      const uint64_t db = B_NMAJOR ? make_desc(sb + (it & 7) * 1024, 64 * 128, 512, 1) : desc_kmajor(sb + k32);
      if (A_TMEM) {
        mma_tf32_tmem_a(tmem, tmem + 128 + (it & 3) * 8, db, idesc, it > 0 ? 1u : 0u);
      } else {
        mma_tf32(tmem, desc_kmajor(sa + k32), db, idesc, it > 0 ? 1u : 0u);
      }
      if (COMMIT != 0 && (it & 7) == 7) {
        mma_commit(step);
        if (COMMIT == 2 && !mbar_wait(step, (it >> 3) & 1, nullptr)) break;
        if (COMMIT == 4 && !mbar_wait_poll(step, (it >> 3) & 1, nullptr)) break;
        if (COMMIT == 3) {
          unsigned polls = 0;
          while (!mbar_test(step, (it >> 3) & 1) && ++polls < (1u << 26)) {
          }
          if (polls >= (1u << 26)) break;
        }
      }
    }
    const unsigned long long t1 = global_ns();
    mma_commit(bar);
    const bool ok = mbar_wait(bar, 0, nullptr);
    const unsigned long long t2 = global_ns();
    out[3 * blockIdx.x] = t2 - t0;
    out[3 * blockIdx.x + 1] = t1 - t0;
    unsigned sm;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    out[3 * blockIdx.x + 2] = ok ? sm : 9999;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256u) : "memory");
}

template <int N, bool AT, bool BN_, int COMMIT = 0>
void run(const char* name, int ctas, int iters, unsigned long long* d) {
  auto k = mma_probe<N, AT, BN_, COMMIT>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  k<<<ctas, 128, SMEM>>>(d, iters);  // warm
  cudaDeviceSynchronize();
  k<<<ctas, 128, SMEM>>>(d, iters);
  cudaError_t e = cudaDeviceSynchronize();
  std::vector<unsigned long long> h(3 * ctas);
  cudaMemcpy(h.data(), d, h.size() * 8, cudaMemcpyDeviceToHost);
  std::vector<double> tot, iss;
  int bad = 0;
  std::vector<int> per_sm(200, 0);
  for (int i = 0; i < ctas; ++i) { tot.push_back(h[3*i] / double(iters)); iss.push_back(h[3*i+1] / double(iters)); if (h[3*i+2] == 9999) ++bad; else per_sm[h[3*i+2] % 200]++; }
  std::sort(tot.begin(), tot.end()); std::sort(iss.begin(), iss.end());
  const int maxper = *std::max_element(per_sm.begin(), per_sm.end());
  const double flop = 2.0 * 128 * N * 8;
  printf("%-28s ctas %3d (max %d/SM): ns/MMA median %.2f (issue %.2f) max %.2f -> %.0f FLOP/ns per CTA; err %s bad %d\n",
         name, ctas, maxper, tot[ctas/2], iss[ctas/2], tot[ctas-1], flop / tot[ctas/2], cudaGetErrorString(e), bad);
}

int main() {
  unsigned long long* d;
  cudaMalloc(&d, 3 * 512 * 8);
  const int iters = 4096;
  for (int ctas : {148, 296}) {
    run<64, false, false>("N=64  A smem  B K-major", ctas, iters, d);
    run<128, false, false>("N=128 A smem  B K-major", ctas, iters, d);
    run<256, false, false>("N=256 A smem  B K-major", ctas, iters, d);
    run<64, true, false>("N=64  A tmem  B K-major", ctas, iters, d);
    run<64, true, true>("N=64  A tmem  B N-major", ctas, iters, d);
    run<128, true, false>("N=128 A tmem  B K-major", ctas, iters, d);
    run<64, false, false, 1>("N=64 A smem, commit per 8", ctas, iters, d);
    run<64, false, false, 2>("N=64 A smem, commit+wait/8", ctas, iters, d);
    run<64, true, true, 1>("N=64 A tmem B N, commit/8", ctas, iters, d);
    run<64, true, true, 2>("N=64 A tmem B N, c+wait/8", ctas, iters, d);
    run<64, false, false, 3>("N=64 A smem, commit+spin/8", ctas, iters, d);
    run<64, true, true, 3>("N=64 A tmem B N, c+spin/8", ctas, iters, d);
    run<64, false, false, 4>("N=64 A smem, commit+poll/8", ctas, iters, d);
    run<64, true, true, 4>("N=64 A tmem B N, c+poll/8", ctas, iters, d);
  }
  cudaFree(d);
  return 0;
}

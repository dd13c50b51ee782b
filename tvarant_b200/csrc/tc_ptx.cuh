// PTX building blocks shared by the tcgen05 kernels: mbarriers with bounded
// waits, TMA tile loads, tensor-memory loads, tcgen05.mma kind::tf32 and its
// shared-memory matrix descriptors, and the host-side tensor-map encoder.
// No TMA load here uses cluster multicast.
#pragma once

#include "internal.h"

namespace tvr {
namespace tc {

constexpr unsigned long long WAIT_TIMEOUT_NS = 2000000000ull;  // 2 s per barrier phase
constexpr unsigned WAIT_MAX_POLLS = 1u << 30;

// ---- PTX wrappers ------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking: whether the phase of `bar` with parity `parity` has completed
// (for event loops that poll several barriers).
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that suspends the thread for at most `ns` nanoseconds before
// returning false.  Without the hint a thread suspended in try_wait on a
// barrier that tcgen05.commit completes woke ~0.37 us after the arrival (8
// MMAs, commit and wait: 1.14 us against 0.77 us for a test_wait spin).
__device__ __forceinline__ bool mbar_try_wait_ns(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

constexpr uint32_t WAIT_POLL_NS = 32;

// mbar_wait with short suspensions (WAIT_POLL_NS), for waits on the critical
// path of a pipeline whose barriers tcgen05.commit completes.
__device__ __forceinline__ bool mbar_wait_poll(uint32_t bar, uint32_t parity,
                                               const volatile int* abort) {
  if (mbar_try_wait_ns(bar, parity, WAIT_POLL_NS)) return true;
  const unsigned long long t0 = global_ns();
  for (unsigned polls = 1; polls < WAIT_MAX_POLLS; ++polls) {
    if (mbar_try_wait_ns(bar, parity, WAIT_POLL_NS)) return true;
    if ((polls & 31u) == 0) {
      if (abort != nullptr && *abort) return false;
      if (global_ns() - t0 > WAIT_TIMEOUT_NS) return false;
    }
  }
  return false;
}

// Waits for the phase of `bar` with parity `parity` to complete.  Gives up
// (returns false) when the CTA abort flag is raised (if `abort` is given) or
// after WAIT_TIMEOUT_NS / WAIT_MAX_POLLS.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          const volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (unsigned polls = 1; polls < WAIT_MAX_POLLS; ++polls) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((polls & 31u) == 0) {
      if (abort != nullptr && *abort) return false;
      if (global_ns() - t0 > WAIT_TIMEOUT_NS) return false;
    }
  }
  return false;
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// A hint: bring one tile of the tensor into L2 (no shared memory, no
// barrier).  L2 is where the GPU's writes become visible, so a prefetch that
// runs before the tile's writer has finished brings in nothing stale: later
// loads read the written values.
__device__ __forceinline__ void tma_prefetch_l2_3d(const CUtensorMap* map, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

__device__ __forceinline__ void tma_prefetch_l2_4d(const CUtensorMap* map, int c0, int c1, int c2,
                                                   int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// Tile store shared -> global through the tensor map (bulk-group completion).
// Elements outside the tensor's extent are not written.  The x coordinate
// (c0, fp32 elements) must be a multiple of 4 and no coordinate negative.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1,
                                             int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Waits until the committed bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Waits until the committed bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptors (tcgen05 "matrix descriptor" format):
// start address >> 4 in bits [0,14), leading byte offset >> 4 in [16,30),
// stride byte offset >> 4 in [32,46), version 1 in [46,48), layout type in
// [61,64): 2 = 128-byte swizzle of 16-byte chunks, 1 = 128-byte swizzle of
// 32-byte chunks (the only N-major layout kind::tf32 accepts).
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout) << 61;
  return d;
}

// K-major tile: rows of 128 bytes (32 fp32 along K) with 16-byte chunks
// swizzled over 8 rows; 8-row groups 1024 B apart.  The leading offset is
// unused for swizzled K-major layouts.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr) {
  return make_desc(saddr, 16, 1024, 2);
}

// Instruction descriptor for kind::tf32: D f32 (bits 4-5 = 1), A and B tf32
// (bits 7-9 and 10-12 = 2), A / B major-ness in bits 15 / 16, N >> 3 in bits
// 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n, bool b_nmajor) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((b_nmajor ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t da, uint64_t db,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same MMA with A read from tensor memory: M rows on TMEM lanes 0..M-1,
// K along columns (one tf32 per 32-bit column), starting at column
// a_tmem; A is K-major by construction (idesc bit 15 = 0).
__device__ __forceinline__ void mma_tf32_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t db,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 lanes x 32 columns of 32-bit accumulator -> 32 registers per thread
// (thread t holds TMEM lane base+t, columns col..col+31).  Completion is
// awaited separately with tmem_wait_loads(), so several loads overlap.
__device__ __forceinline__ void tmem_load_32_async(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_loads() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 registers per thread -> 32 columns of its TMEM lane (the inverse of
// tmem_load_32_async); tmem_wait_stores() waits until they are written.
__device__ __forceinline__ void tmem_store_32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_stores() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status != nullptr) atomicCAS(status, TVR_DEV_OK, code);
}

// ---- host side -----------------------------------------------------------------

inline int encode_3d(CUtensorMap* map, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2,
              uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1,
              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  const DriverApi* drv = driver();
  if (drv == nullptr) return TVR_ERR_CUDA;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {box0, box1, 1};
  const cuuint32_t elem_strides[3] = {1, 1, 1};
  CUresult r = drv->tensorMapEncodeTiled(
      map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(ptr), dims, strides, box,
      elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    const char* msg = "?";
    if (drv->getErrorString) drv->getErrorString(r, &msg);
    return fail(TVR_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d: %s) dims {%llu, %llu, %llu}",
                static_cast<int>(r), msg, (unsigned long long)d0, (unsigned long long)d1,
                (unsigned long long)d2);
  }
  return TVR_OK;
}

// 4-D fp32 tensor map: dims {d0 (contiguous), d1, d2, d3}, byte strides of
// d1..d3, box {box0, box1, 1, 1}.
inline int encode_4d(CUtensorMap* map, const void* ptr, const uint64_t dims[4],
                     const uint64_t strides_bytes[3], uint32_t box0, uint32_t box1,
                     CUtensorMapSwizzle swizzle) {
  const DriverApi* drv = driver();
  if (drv == nullptr) return TVR_ERR_CUDA;
  const cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  const cuuint64_t st[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  const cuuint32_t box[4] = {box0, box1, 1, 1};
  const cuuint32_t elem_strides[4] = {1, 1, 1, 1};
  CUresult r = drv->tensorMapEncodeTiled(
      map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(ptr), d, st, box, elem_strides,
      CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    const char* msg = "?";
    if (drv->getErrorString) drv->getErrorString(r, &msg);
    return fail(TVR_ERR_CUDA, "cuTensorMapEncodeTiled (4-D) failed (%d: %s)", static_cast<int>(r),
                msg);
  }
  return TVR_OK;
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace tc
}  // namespace tvr

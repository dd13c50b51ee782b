// Internal helpers shared by the translation units of libtvarant_cuda.so.
// Nothing here is part of the C ABI (include/tvarant.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "../../include/tvarant.h"

namespace tvr {

// Records a printf-style message as the calling thread's last error and
// returns `code`, so call sites read `return fail(TVR_ERR_INVALID, ...)`.
int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

// Number of SMs of `device` (cached after the first query).
int sm_count(int device);

// Device whose context is current on this thread.
int current_device();

// Per-device int in device memory that kernels with bounded waits write a
// TVR_DEV_* code into.
int* device_status_ptr(int device);
// The same word if the device has already been set up, else nullptr; never
// sets the device up (so never allocates).
int* device_status_ptr_if_ready(int device);

// Driver API entry points resolved through cudaGetDriverEntryPoint, so the
// library does not link libcuda directly.
struct DriverApi {
  CUresult (*tensorMapEncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill) = nullptr;
  CUresult (*moduleLoadData)(CUmodule*, const void*) = nullptr;
  CUresult (*moduleGetFunction)(CUfunction*, CUmodule, const char*) = nullptr;
  CUresult (*launchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned,
                           unsigned, unsigned, CUstream, void**, void**) = nullptr;
  CUresult (*getErrorString)(CUresult, const char**) = nullptr;
  CUresult (*ctxGetCurrent)(CUcontext*) = nullptr;
};
// Returns nullptr (with the error recorded) if an entry point is missing.
const DriverApi* driver();

// Scratch device memory from the caching pool, released in stream order.
struct Scratch {
  void* ptr = nullptr;
  cudaStream_t stream = nullptr;
  ~Scratch();
  int alloc(size_t nbytes, int device, cudaStream_t s);
};

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

#ifdef __CUDACC__
// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while the kernel before it on the stream is still
// running; grid_dependency_wait() blocks the calling thread until that kernel
// has completed and its memory operations are visible to this grid.  A kernel
// calls grid_launch_dependents() to let such a successor start before it
// ends.  Without a programmatic dependency both do nothing.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
#endif

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Attention of at most four query rows per (sequence, head) on the CUDA
// cores (attention_decode.cu): the decode-step form of tvr_attention_fwd.
// The caller has checked sizes, pointers, a positive finite scale and 16-byte
// aligned operands with strides that are multiples of 4 elements.
bool attention_decode_applies(int64_t seq_q, int64_t head_dim);
int attention_decode(const float* q, const float* k, const float* v, float* out, float* lse,
                     int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_k,
                     const int64_t* q_strides, const int64_t* k_strides,
                     const int64_t* v_strides, const int64_t* o_strides, float scale, int causal,
                     const int64_t* key_len, int key_len_add, cudaStream_t stream);

// Grid size for grid-stride elementwise kernels: enough blocks to cover the
// work, capped at `waves` resident waves of the device.
inline unsigned elementwise_grid(int64_t work_items, int threads, int device, int waves = 8) {
  int64_t blocks = ceil_div(work_items, threads);
  int64_t cap = static_cast<int64_t>(sm_count(device)) * waves;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<unsigned>(blocks);
}

}  // namespace tvr

#define TVR_CUDA_TRY(expr)                                                                  \
  do {                                                                                      \
    cudaError_t tvr_e_ = (expr);                                                            \
    if (tvr_e_ != cudaSuccess) {                                                            \
      return ::tvr::fail(TVR_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,                      \
                         cudaGetErrorString(tvr_e_), __FILE__, __LINE__);                   \
    }                                                                                       \
  } while (0)

#define TVR_CHECK(cond, ...)                                                                \
  do {                                                                                      \
    if (!(cond)) return ::tvr::fail(TVR_ERR_INVALID, __VA_ARGS__);                          \
  } while (0)

#define TVR_LAUNCH_CHECK() TVR_CUDA_TRY(cudaGetLastError())

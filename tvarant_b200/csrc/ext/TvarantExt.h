// Shared declarations of the tvarant PyTorch extension (_C.so).
//
// The extension owns no device code: every kernel, copy and allocation goes
// through the C ABI of libtvarant_cuda.so (include/tvarant.h).  It replaces
// the reference's csrc/runtime plumbing (Allocator/Guard/Hooks/Generator,
// Runtime.cpp) and csrc/aten op bodies with versions that pass raw device
// pointers, sizes and the current stream to that ABI.
#pragma once

#include <ATen/ATen.h>
#include <c10/core/Device.h>
#include <c10/core/Stream.h>
#include <c10/util/Exception.h>

#include <cstdint>
#include <vector>

#include "tvarant.h"

namespace tvarant {

// Throws c10::Error carrying the library's message when rc != TVR_OK.
void check_rc(int rc, const char* what);
#define TVR_TRY(expr) ::tvarant::check_rc((expr), #expr)

// ---- devices and streams (Runtime.cpp) ----
int device_count();
int current_device();
void set_device(int index);
int exchange_device(int index);
bool runtime_available();

// Stream ids: 0 is the device's legacy default stream; k >= 1 is entry k-1
// of a lazily created per-device pool of non-blocking streams.
void* stream_handle(c10::DeviceIndex device, c10::StreamId id);
c10::Stream current_stream(c10::DeviceIndex device = -1);
void set_current_stream(const c10::Stream& stream);
c10::Stream stream_from_pool(c10::DeviceIndex device, bool high_priority);
// Handle of the current stream of the current device (what kernels run on).
void* current_stream_handle();

// ---- allocator (Allocator.cpp) ----
c10::Allocator* allocator();

// ---- generator (Generator.cpp) ----
const at::Generator& default_generator(c10::DeviceIndex device);
at::Generator make_generator(c10::DeviceIndex device);

// ---- op helpers (Ops.cpp) ----
namespace ops {

void check_fp32(const at::Tensor& t, const char* op);
// float64 (and integer wrapped numbers) -> float32, as ensure_fp32 in the
// reference's csrc/aten/AtenCommon.h:20-29.
at::Tensor ensure_fp32(const at::Tensor& t, const char* op);
// Moves a CPU operand (a wrapped Python number or a CPU tensor) to the device
// of `like`.
at::Tensor to_device_like(const at::Tensor& t, const at::Tensor& like);
bool is_device(const at::Tensor& t);

// GEMM precision mode from torch.get_float32_matmul_precision(), unless
// TVARANT_GEMM_MODE is set (then AUTO lets the library read it).
int gemm_mode();

// C[m,n] = act(alpha * A[m,k] @ op(B) + beta * bias) — the reference's
// ops::gemm_bias_act (csrc/aten/AtenCommon.h:33-86).  B is [k,n], or [n,k]
// when trans_b.  A transposed B view is consumed without a copy.
// With `prog`, the pointwise program runs on the GEMM's output
// (tvr_gemm_pointwise): prog->inputs[prog->gemm_input] is unused and the
// other inputs are [m, n] with row strides prog->ld (0: broadcast row).
struct GemmProgram {
  std::vector<tvr_pw_node> nodes;
  int gemm_input = 0;
  std::vector<const float*> inputs;
  std::vector<int64_t> ld;
};
at::Tensor gemm_bias_act(const at::Tensor& a, const at::Tensor& b, const at::Tensor* bias,
                         float alpha, float beta, int act, bool trans_b,
                         const GemmProgram* prog = nullptr);

at::Tensor empty_like_contig(const at::Tensor& like, at::IntArrayRef sizes);
at::Tensor empty_device(at::IntArrayRef sizes, const at::TensorOptions& opts);
at::Tensor copy_from(const at::Tensor& self, const at::Tensor& dst, bool non_blocking);
at::Tensor& fill_scalar(at::Tensor& self, const at::Scalar& value);
at::Tensor add_tensor(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha);
at::Tensor add_scalar(const at::Tensor& self, const at::Scalar& other, const at::Scalar& alpha);
at::Tensor mul_tensor(const at::Tensor& self, const at::Tensor& other);
at::Tensor unary(const at::Tensor& self, int op, float scalar, const char* name);
at::Tensor contiguous_copy(const at::Tensor& self);

}  // namespace ops
}  // namespace tvarant

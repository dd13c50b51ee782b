// LLM-path ATen kernels of the tvarant device: silu, scalar mul/add,
// softmax, matmul / bmm, linear, native_layer_norm, embedding.
//
// Registration list and semantics follow the reference's csrc/aten/LlmOps.cpp
// (:288-301).  Differences by design:
//   - matmul does not materialise a broadcast 2-D right operand
//     (reference LlmOps.cpp:123-126): it is read with batch stride 0;
//   - transposed operands (k.transpose(-2, -1)) are consumed in place as the
//     other GEMM layout instead of being copied contiguous;
//   - embedding reads int64 (or int32) indices on the device; the reference
//     copies them to the host, narrows them to int32 and copies them back
//     (LlmOps.cpp:238-246).
#include <ATen/ATen.h>
#include <c10/core/DeviceGuard.h>
#include <torch/library.h>

#include <tuple>

#include "TvarantExt.h"

namespace tvarant::ops {
namespace {

at::Tensor silu_op(const at::Tensor& self) {
  check_fp32(self, "silu");
  return unary(self, TVR_UNARY_SILU, 0.f, "silu");
}

at::Tensor& silu_(at::Tensor& self) {
  at::Tensor r = silu_op(self);
  copy_from(r, self, false);
  return self;
}

at::Tensor& silu_out(const at::Tensor& self, at::Tensor& out) {
  at::Tensor r = silu_op(self);
  if (!out.sizes().equals(r.sizes())) out.resize_(r.sizes());
  copy_from(r, out, false);
  return out;
}

at::Tensor mul_scalar(const at::Tensor& self, const at::Scalar& other) {
  return unary(self, TVR_UNARY_SCALE, static_cast<float>(other.toDouble()), "mul");
}

at::Tensor add_scalar_op(const at::Tensor& self, const at::Scalar& other, const at::Scalar& alpha) {
  return add_scalar(self, other, alpha);
}

at::Tensor softmax_impl(const at::Tensor& self, int64_t dim, bool /*half_to_float*/) {
  check_fp32(self, "softmax");
  TORCH_CHECK(self.dim() > 0, "softmax: expected non-scalar");
  if (dim < 0) dim += self.dim();
  TORCH_CHECK(dim >= 0 && dim < self.dim(), "softmax dim out of range");
  c10::DeviceGuard guard(self.device());
  at::Tensor in = self.is_contiguous() ? self : contiguous_copy(self);
  int64_t outer = 1, inner = 1;
  for (int64_t i = 0; i < dim; ++i) outer *= in.size(i);
  for (int64_t i = dim + 1; i < in.dim(); ++i) inner *= in.size(i);
  at::Tensor out = empty_device(in.sizes(), in.options());
  TVR_TRY(tvr_softmax(static_cast<const float*>(in.data_ptr()), static_cast<float*>(out.data_ptr()),
                      outer, in.size(dim), inner, current_stream_handle()));
  return out;
}

at::Tensor softmax_int(const at::Tensor& self, int64_t dim, std::optional<at::ScalarType> dtype) {
  TORCH_CHECK(!dtype.has_value() || dtype.value() == at::kFloat,
              "Tvarant softmax supports float32 only");
  return softmax_impl(self, dim, false);
}

// Batch dimensions of `t` (all but the last two) collapse to one stride if
// each is nested in the next; returns that stride, or -1.
int64_t batch_stride(const at::Tensor& t) {
  const int64_t nb = t.dim() - 2;
  if (nb <= 0) return 0;
  int64_t stride = t.stride(nb - 1);
  for (int64_t d = nb - 2; d >= 0; --d) {
    if (t.size(d + 1) != 1 && t.stride(d) != t.stride(d + 1) * t.size(d + 1)) return -1;
  }
  return stride;
}

at::Tensor matmul_op(const at::Tensor& self, const at::Tensor& other) {
  check_fp32(self, "matmul");
  check_fp32(other, "matmul");
  TORCH_CHECK(self.dim() >= 2 && other.dim() >= 2, "matmul: expected at least 2D tensors");
  if (self.dim() == 2 && other.dim() == 2) {
    return gemm_bias_act(self, other, nullptr, 1.f, 0.f, TVR_ACT_NONE, false);
  }
  c10::DeviceGuard guard(self.device());
  const int64_t m = self.size(-2), k = self.size(-1), n = other.size(-1);
  TORCH_CHECK(other.size(-2) == k, "matmul: contracting dim mismatch ", self.sizes(), " vs ",
              other.sizes());
  // A: dense row-major matrices, batch dims collapsible.
  at::Tensor a = self;
  int64_t sa = batch_stride(a);
  if (!(a.stride(-1) == 1 && (m <= 1 || a.stride(-2) == k)) || sa < 0) {
    a = contiguous_copy(a);
    sa = m * k;
  }
  const int64_t a_batch = a.numel() / std::max<int64_t>(m * k, 1);
  // B: [k, n] row-major (trans_b = 0) or the transpose of a row-major
  // [n, k] (trans_b = 1), per batch; a 2-D B is shared by every batch entry.
  at::Tensor b = other;
  bool trans_b = false;
  int64_t sb;
  const bool row_major = b.stride(-1) == 1 && (k <= 1 || b.stride(-2) == n);
  const bool col_major = b.stride(-2) == 1 && (n <= 1 || b.stride(-1) == k);
  if (row_major || col_major) {
    trans_b = !row_major;
    sb = b.dim() == 2 ? 0 : batch_stride(b);
  } else {
    sb = -1;
  }
  if (sb < 0) {
    b = contiguous_copy(b);
    trans_b = false;
    sb = b.dim() == 2 ? 0 : k * n;
  }
  const int64_t b_batch = b.dim() == 2 ? a_batch : b.numel() / std::max<int64_t>(k * n, 1);
  TORCH_CHECK(a_batch == b_batch && (b.dim() == 2 || b.dim() == a.dim()),
              "matmul: batch mismatch ", self.sizes(), " vs ", other.sizes());
  if (b.dim() > 2) {
    for (int64_t d = 0; d < a.dim() - 2; ++d) {
      TORCH_CHECK(a.size(d) == b.size(d), "matmul: batch mismatch ", self.sizes(), " vs ",
                  other.sizes());
    }
  }
  auto out_sizes = a.sizes().vec();
  out_sizes.back() = n;
  at::Tensor out = empty_device(out_sizes, a.options());
  if (out.numel() == 0) return out;
  if (a_batch == 1) sa = m * k;
  TVR_TRY(tvr_bmm(static_cast<const float*>(a.data_ptr()), static_cast<const float*>(b.data_ptr()),
                  static_cast<float*>(out.data_ptr()), a_batch, m, n, k, sa, sb, m * n,
                  trans_b ? 1 : 0, gemm_mode(), current_stream_handle()));
  return out;
}

at::Tensor bmm_op(const at::Tensor& self, const at::Tensor& mat2) {
  TORCH_CHECK(self.dim() == 3 && mat2.dim() == 3, "bmm(): tensors must be 3D");
  return matmul_op(self, mat2);
}

at::Tensor linear_op(const at::Tensor& input, const at::Tensor& weight,
                  const std::optional<at::Tensor>& bias_opt) {
  check_fp32(input, "linear");
  check_fp32(weight, "linear");
  TORCH_CHECK(weight.dim() == 2, "linear: weight must be 2D");
  at::Tensor x = input.is_contiguous() ? input : contiguous_copy(input);
  const int64_t in_f = x.size(-1);
  TORCH_CHECK(in_f == weight.size(1), "linear: in_features mismatch");
  const int64_t out_f = weight.size(0);
  auto out_sizes = x.sizes().vec();
  out_sizes.back() = out_f;
  const int64_t m = in_f > 0 ? x.numel() / in_f : 0;
  at::Tensor x2 = x.reshape({m, in_f});
  const at::Tensor* bias = nullptr;
  at::Tensor bias_store;
  if (bias_opt.has_value() && bias_opt->defined()) {
    check_fp32(*bias_opt, "linear");
    bias_store = *bias_opt;
    bias = &bias_store;
  }
  return gemm_bias_act(x2, weight, bias, 1.f, 1.f, TVR_ACT_NONE, true).reshape(out_sizes);
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> native_layer_norm(
    const at::Tensor& input, c10::SymIntArrayRef normalized_shape_sym,
    const std::optional<at::Tensor>& weight, const std::optional<at::Tensor>& bias, double eps) {
  check_fp32(input, "layer_norm");
  auto normalized_shape = C10_AS_INTARRAYREF_SLOW(normalized_shape_sym);
  int64_t n = 1;
  for (auto d : normalized_shape) n *= d;
  TORCH_CHECK(n > 0 && input.numel() % n == 0, "layer_norm: invalid normalized_shape");
  TORCH_CHECK(static_cast<int64_t>(normalized_shape.size()) <= input.dim(),
              "layer_norm: normalized_shape longer than input");
  c10::DeviceGuard guard(input.device());
  const int64_t rows = input.numel() / n;
  at::Tensor in = input.is_contiguous() ? input : contiguous_copy(input);
  at::Tensor out = empty_device(in.sizes(), in.options());
  // statistics keep the normalised dimensions as size 1, as ATen does
  auto stat_sizes = in.sizes().vec();
  for (size_t i = stat_sizes.size() - normalized_shape.size(); i < stat_sizes.size(); ++i) {
    stat_sizes[i] = 1;
  }
  at::Tensor mean = empty_device(stat_sizes, in.options());
  at::Tensor rstd = empty_device(stat_sizes, in.options());
  at::Tensor w, b;
  const float* wptr = nullptr;
  const float* bptr = nullptr;
  if (weight.has_value() && weight->defined()) {
    check_fp32(*weight, "layer_norm");
    w = weight->is_contiguous() ? *weight : contiguous_copy(*weight);
    wptr = static_cast<const float*>(w.data_ptr());
  }
  if (bias.has_value() && bias->defined()) {
    check_fp32(*bias, "layer_norm");
    b = bias->is_contiguous() ? *bias : contiguous_copy(*bias);
    bptr = static_cast<const float*>(b.data_ptr());
  }
  TVR_TRY(tvr_layer_norm(static_cast<const float*>(in.data_ptr()), wptr, bptr,
                         static_cast<float*>(out.data_ptr()), static_cast<float*>(mean.data_ptr()),
                         static_cast<float*>(rstd.data_ptr()), rows, n, static_cast<float>(eps),
                         current_stream_handle()));
  return {out, mean, rstd};
}

at::Tensor embedding_op(const at::Tensor& weight, const at::Tensor& indices, c10::SymInt /*padding*/,
                     bool /*scale_grad_by_freq*/, bool /*sparse*/) {
  check_fp32(weight, "embedding");
  TORCH_CHECK(weight.dim() == 2, "embedding: weight must be 2D");
  TORCH_CHECK(indices.scalar_type() == at::kLong || indices.scalar_type() == at::kInt,
              "embedding: indices must be int64 or int32, got ", indices.scalar_type());
  c10::DeviceGuard guard(weight.device());
  at::Tensor idx = to_device_like(indices, weight);
  if (!idx.is_contiguous()) idx = contiguous_copy(idx);
  at::Tensor w = weight.is_contiguous() ? weight : contiguous_copy(weight);
  auto out_sizes = indices.sizes().vec();
  out_sizes.push_back(w.size(1));
  at::Tensor out = empty_device(out_sizes, w.options());
  if (idx.numel() == 0 || w.size(1) == 0) return out;
  TVR_TRY(tvr_embedding(static_cast<const float*>(w.data_ptr()), idx.data_ptr(),
                        idx.scalar_type() == at::kLong ? 64 : 32,
                        static_cast<float*>(out.data_ptr()), idx.numel(), w.size(1), w.size(0),
                        current_stream_handle()));
  return out;
}

}  // namespace
}  // namespace tvarant::ops

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("silu", TORCH_FN(tvarant::ops::silu_op));
  m.impl("silu_", TORCH_FN(tvarant::ops::silu_));
  m.impl("silu.out", TORCH_FN(tvarant::ops::silu_out));
  m.impl("mul.Scalar", TORCH_FN(tvarant::ops::mul_scalar));
  m.impl("add.Scalar", TORCH_FN(tvarant::ops::add_scalar_op));
  m.impl("_softmax", TORCH_FN(tvarant::ops::softmax_impl));
  m.impl("softmax.int", TORCH_FN(tvarant::ops::softmax_int));
  m.impl("matmul", TORCH_FN(tvarant::ops::matmul_op));
  m.impl("bmm", TORCH_FN(tvarant::ops::bmm_op));
  m.impl("linear", TORCH_FN(tvarant::ops::linear_op));
  m.impl("native_layer_norm", TORCH_FN(tvarant::ops::native_layer_norm));
  m.impl("embedding", TORCH_FN(tvarant::ops::embedding_op));
}

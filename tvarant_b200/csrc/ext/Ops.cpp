// Core ATen kernels of the tvarant device: tensor creation and views,
// copies in every direction, fill, add / mul with broadcasting, relu, mm,
// addmm, and the host-drawn random fills.
//
// Registration list and semantics follow the reference's csrc/aten/Ops.cpp
// (:469-497).  Differences by design:
//   - broadcasting happens inside the kernel (tvr_binary strides) instead of
//     expand().contiguous() copies (reference Ops.cpp:287-289);
//   - copies run on the device, including strided and dtype-converting
//     device-to-device copies (the reference staged them through host views,
//     Ops.cpp:185-212);
//   - there is no boxed CPU fallback (reference Ops.cpp:499-501): an op the
//     backend does not implement raises instead of silently running on CPU.
#include <ATen/ATen.h>
#include <ATen/EmptyTensor.h>
#include <ATen/ExpandUtils.h>
#include <ATen/InferSize.h>
#include <ATen/TensorUtils.h>
#include <ATen/CPUGeneratorImpl.h>
#include <ATen/detail/PrivateUse1HooksInterface.h>
#include <ATen/native/Resize.h>
#include <c10/core/DeviceGuard.h>
#include <torch/library.h>

#include <cstdlib>
#include <cstring>

#include "TvarantExt.h"

namespace tvarant::ops {
namespace {

c10::DispatchKeySet device_keys() {
  return c10::DispatchKeySet{c10::DispatchKey::PrivateUse1, c10::DispatchKey::AutogradPrivateUse1};
}

int type_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return 0;
    case at::kDouble: return 1;
    case at::kInt: return 2;
    case at::kLong: return 3;
    case at::kBool:
    case at::kByte: return 4;
    default: return -1;
  }
}

std::vector<int64_t> expanded_strides(const at::Tensor& t, at::IntArrayRef sizes) {
  return t.expand(sizes).strides().vec();
}

void strided_copy(const at::Tensor& dst, const at::Tensor& src_expanded) {
  TORCH_CHECK(dst.dim() <= TVR_MAX_DIMS, "tvarant copy supports at most ", TVR_MAX_DIMS,
              " dimensions, got ", dst.dim());
  const auto sizes = dst.sizes().vec();
  const auto ds = dst.strides().vec();
  const auto ss = src_expanded.strides().vec();
  TVR_TRY(tvr_strided_copy(dst.data_ptr(), src_expanded.data_ptr(),
                           static_cast<int64_t>(dst.element_size()),
                           static_cast<int>(sizes.size()), sizes.data(), ds.data(), ss.data(),
                           current_stream_handle()));
}

bool pinned(const at::Tensor& t) {
  int p = 0;
  return tvr_is_pinned(t.data_ptr(), &p) == TVR_OK && p != 0;
}

void sync_current_stream() { TVR_TRY(tvr_stream_synchronize(current_stream_handle())); }

// host -> device
void copy_h2d(const at::Tensor& src, const at::Tensor& dst, bool non_blocking) {
  c10::DeviceGuard guard(dst.device());
  at::Tensor s = src.to(dst.scalar_type()).expand(dst.sizes());
  const size_t nbytes = static_cast<size_t>(dst.numel()) * dst.element_size();
  at::Tensor target = dst.is_contiguous() ? dst : empty_device(dst.sizes(), dst.options());
  at::Tensor sc = s.contiguous();
  TVR_TRY(tvr_memcpy_h2d(target.data_ptr(), sc.data_ptr(), nbytes, current_stream_handle()));
  if (!target.is_same(dst)) strided_copy(dst, target);
  // A pinned source is read asynchronously; keep blocking semantics unless
  // the caller asked for a non-blocking copy.
  if (!non_blocking && pinned(sc)) sync_current_stream();
}

// device -> host
void copy_d2h(const at::Tensor& src, const at::Tensor& dst, bool non_blocking) {
  c10::DeviceGuard guard(src.device());
  at::Tensor s = src.is_contiguous() ? src : contiguous_copy(src);
  const size_t nbytes = static_cast<size_t>(s.numel()) * s.element_size();
  if (dst.is_contiguous() && dst.scalar_type() == s.scalar_type() && dst.sizes() == s.sizes()) {
    TVR_TRY(tvr_memcpy_d2h(dst.data_ptr(), s.data_ptr(), nbytes, current_stream_handle()));
    if (!(non_blocking && pinned(dst))) sync_current_stream();
    return;
  }
  at::Tensor tmp = at::empty(s.sizes(), s.options().device(at::kCPU));
  TVR_TRY(tvr_memcpy_d2h(tmp.data_ptr(), s.data_ptr(), nbytes, current_stream_handle()));
  sync_current_stream();
  dst.copy_(tmp);
}

// device -> device (same or different GPU)
void copy_d2d(const at::Tensor& src, const at::Tensor& dst) {
  if (src.device() != dst.device()) {
    at::Tensor host = at::empty(src.sizes(), src.options().device(at::kCPU));
    copy_d2h(src, host, false);
    copy_h2d(host, dst, false);
    return;
  }
  c10::DeviceGuard guard(dst.device());
  at::Tensor s = src;
  if (s.scalar_type() != dst.scalar_type()) {
    const int from = type_code(s.scalar_type()), to = type_code(dst.scalar_type());
    if (from < 0 || to < 0) {
      at::Tensor host = at::empty(src.sizes(), src.options().device(at::kCPU));
      copy_d2h(src, host, false);
      copy_h2d(host, dst, false);
      return;
    }
    at::Tensor sc = s.is_contiguous() ? s : contiguous_copy(s);
    at::Tensor conv = empty_device(sc.sizes(), dst.options());
    TVR_TRY(tvr_convert(conv.data_ptr(), to, sc.data_ptr(), from, sc.numel(),
                        current_stream_handle()));
    s = conv;
  }
  strided_copy(dst, s.expand(dst.sizes()));
}

}  // namespace

bool is_device(const at::Tensor& t) { return t.device().is_privateuseone(); }

void check_fp32(const at::Tensor& t, const char* op) {
  TORCH_CHECK(t.scalar_type() == at::kFloat, "Tvarant op '", op, "' supports float32 only, got ",
              t.scalar_type());
}

at::Tensor ensure_fp32(const at::Tensor& t, const char* op) {
  if (t.scalar_type() == at::kFloat) return t;
  if (t.scalar_type() == at::kDouble) return t.to(at::kFloat);
  // Python numbers arrive as 0-dim CPU tensors (wrapped numbers); accept
  // integer ones too so `x + 1` works.
  if (!is_device(t) && t.dim() == 0 && (at::isIntegralType(t.scalar_type(), true))) {
    return t.to(at::kFloat);
  }
  check_fp32(t, op);
  return t;
}

at::Tensor empty_device(at::IntArrayRef sizes, const at::TensorOptions& opts) {
  c10::DeviceGuard guard(opts.device());
  return at::detail::empty_generic(sizes, allocator(), device_keys(),
                                   c10::typeMetaToScalarType(opts.dtype()), std::nullopt);
}

at::Tensor empty_like_contig(const at::Tensor& like, at::IntArrayRef sizes) {
  return empty_device(sizes, like.options());
}

at::Tensor contiguous_copy(const at::Tensor& self) {
  at::Tensor out = empty_device(self.sizes(), self.options());
  if (self.numel() > 0) {
    c10::DeviceGuard guard(self.device());
    strided_copy(out, self);
  }
  return out;
}

at::Tensor to_device_like(const at::Tensor& t, const at::Tensor& like) {
  if (is_device(t)) return t;
  if (t.dim() == 0) {
    // A Python number or 0-dim CPU tensor: a fill kernel carries the value as
    // an argument, so no host buffer is read later by the device (a copy from
    // a temporary host scalar would be replayed from a dangling address by a
    // captured graph) and no host-to-device copy is queued.
    at::Tensor out = empty_device({}, t.options().device(like.device()));
    fill_scalar(out, t.item());
    return out;
  }
  at::Tensor c = t.contiguous();
  at::Tensor out = empty_device(c.sizes(), c.options().device(like.device()));
  copy_h2d(c, out, false);
  return out;
}

int gemm_mode() {
  const char* env = std::getenv("TVARANT_GEMM_MODE");
  if (env != nullptr && env[0] != '\0') return TVR_GEMM_AUTO;
  return at::globalContext().float32MatmulPrecision() == at::Float32MatmulPrecision::HIGHEST
             ? TVR_GEMM_3XTF32
             : TVR_GEMM_TF32;
}

at::Tensor gemm_bias_act(const at::Tensor& a_in, const at::Tensor& b_in, const at::Tensor* bias,
                         float alpha, float beta, int act, bool trans_b, const GemmProgram* prog) {
  TORCH_CHECK(a_in.dim() == 2 && b_in.dim() == 2, "gemm: expected 2D tensors");
  c10::DeviceGuard guard(a_in.device());
  at::Tensor a = a_in;
  const int64_t m = a.size(0), k = a.size(1);
  if (!(a.stride(1) == 1 && (m <= 1 || a.stride(0) >= k))) a = contiguous_copy(a);
  const int64_t lda = m <= 1 ? std::max<int64_t>(k, 1) : a.stride(0);
  // B as stored: a row-major matrix is used directly; a column-major one is
  // the transpose of a row-major matrix and flips trans_b instead of copying.
  at::Tensor b = b_in;
  bool trans = trans_b;
  int64_t ldb;
  const int64_t r = b.size(0), c = b.size(1);
  if (b.stride(1) == 1 && (r <= 1 || b.stride(0) >= c)) {
    ldb = r <= 1 ? std::max<int64_t>(c, 1) : b.stride(0);
  } else if (b.stride(0) == 1 && (c <= 1 || b.stride(1) >= r) && r > 1) {
    b = b.t();  // row-major [c, r] view of the same memory
    trans = !trans;
    ldb = c <= 1 ? std::max<int64_t>(r, 1) : b.stride(0);
  } else {
    b = contiguous_copy(b);
    ldb = std::max<int64_t>(c, 1);
  }
  const int64_t n = trans_b ? r : c;
  if (trans_b) {
    TORCH_CHECK(c == k, "gemm trans_b: K mismatch ", b_in.sizes(), " vs K=", k);
  } else {
    TORCH_CHECK(r == k, "gemm: K mismatch ", a_in.sizes(), " vs ", b_in.sizes());
  }
  at::Tensor bias_c;
  const void* bias_ptr = nullptr;
  float beta_use = 0.f;
  if (bias != nullptr && beta != 0.f) {
    bias_c = to_device_like(*bias, a);
    check_fp32(bias_c, "gemm");
    if (!bias_c.is_contiguous()) bias_c = contiguous_copy(bias_c);
    TORCH_CHECK(bias_c.numel() == n, "gemm bias must have ", n, " elements, got ",
                bias_c.numel());
    bias_ptr = bias_c.data_ptr();
    beta_use = beta;
  }
  at::Tensor out = empty_device({m, n}, a.options());
  if (m == 0 || n == 0) return out;
  if (prog != nullptr) {
    TVR_TRY(tvr_gemm_pointwise(
        static_cast<const float*>(a.data_ptr()), static_cast<const float*>(b.data_ptr()),
        static_cast<const float*>(bias_ptr), static_cast<float*>(out.data_ptr()), m, n, k, lda, ldb,
        n, alpha, beta_use, act, trans ? 1 : 0, gemm_mode(), prog->nodes.data(),
        static_cast<int>(prog->nodes.size()), static_cast<int>(prog->inputs.size()),
        prog->gemm_input, prog->inputs.data(), prog->ld.data(), current_stream_handle()));
    return out;
  }
  TVR_TRY(tvr_gemm_bias_act(static_cast<const float*>(a.data_ptr()),
                            static_cast<const float*>(b.data_ptr()),
                            static_cast<const float*>(bias_ptr),
                            static_cast<float*>(out.data_ptr()), m, n, k, lda, ldb, n, alpha,
                            beta_use, act, trans ? 1 : 0, gemm_mode(), current_stream_handle()));
  return out;
}

at::Tensor copy_from(const at::Tensor& self, const at::Tensor& dst, bool non_blocking) {
  TORCH_CHECK(self.defined() && dst.defined(), "copy: undefined tensor");
  if (self.numel() == 0 || dst.numel() == 0) return dst;
  const bool sd = is_device(self), dd = is_device(dst);
  if (sd && dd) {
    copy_d2d(self, dst);
  } else if (!sd && dd) {
    copy_h2d(self, dst, non_blocking);
  } else if (sd && !dd) {
    copy_d2h(self, dst, non_blocking);
  } else {
    TORCH_CHECK(false, "Unsupported Tvarant copy: ", self.device(), " -> ", dst.device());
  }
  return dst;
}

at::Tensor& fill_scalar(at::Tensor& self, const at::Scalar& value) {
  if (self.numel() == 0) return self;
  c10::DeviceGuard guard(self.device());
  at::Tensor v = at::scalar_tensor(value, self.options().device(at::kCPU));
  const int es = static_cast<int>(self.element_size());
  TORCH_CHECK(es == 1 || es == 2 || es == 4 || es == 8, "fill_: unsupported dtype ",
              self.scalar_type());
  if (self.is_non_overlapping_and_dense()) {
    TVR_TRY(tvr_fill(self.data_ptr(), v.data_ptr(), es, self.numel(), current_stream_handle()));
  } else {
    at::Tensor tmp = empty_device(self.sizes(), self.options());
    TVR_TRY(tvr_fill(tmp.data_ptr(), v.data_ptr(), es, tmp.numel(), current_stream_handle()));
    strided_copy(self, tmp);
  }
  return self;
}

namespace {

at::Tensor binary(const at::Tensor& self, const at::Tensor& other, int op, float alpha,
                  const char* name) {
  at::Tensor a = ensure_fp32(self, name);
  at::Tensor b = ensure_fp32(other, name);
  // tensor (op) Python number: the unary kernels take the number by value,
  // with the same fp32 rounding as the broadcast binary kernel
  // (a * s, and a + alpha * s with alpha * s rounded to fp32 first).
  auto host_scalar = [](const at::Tensor& t) { return !is_device(t) && t.dim() == 0; };
  if (is_device(a) && host_scalar(b)) {
    const float s = b.item<float>();
    if (op == TVR_BINARY_MUL) return unary(a, TVR_UNARY_SCALE, s, name);
    return unary(a, TVR_UNARY_ADD_SCALAR, alpha * s, name);
  }
  if (host_scalar(a) && is_device(b)) {
    const float s = a.item<float>();
    if (op == TVR_BINARY_MUL) return unary(b, TVR_UNARY_SCALE, s, name);
    if (alpha == 1.f) return unary(b, TVR_UNARY_ADD_SCALAR, s, name);
  }
  const at::Tensor& anchor = is_device(a) ? a : b;
  TORCH_CHECK(is_device(anchor), name, ": expected a tvarant tensor");
  a = to_device_like(a, anchor);
  b = to_device_like(b, anchor);
  TORCH_CHECK(a.device() == b.device(), name, ": tensors on different devices ", a.device(),
              " and ", b.device());
  c10::DeviceGuard guard(anchor.device());
  auto sizes = at::infer_size(a.sizes(), b.sizes());
  at::Tensor out = empty_device(sizes, anchor.options());
  if (out.numel() == 0) return out;
  if (static_cast<int>(sizes.size()) > TVR_MAX_DIMS) {
    a = contiguous_copy(a.expand(sizes)).view({-1});
    b = contiguous_copy(b.expand(sizes)).view({-1});
    sizes = {out.numel()};
  }
  const auto sa = expanded_strides(a, sizes);
  const auto sb = expanded_strides(b, sizes);
  TVR_TRY(tvr_binary(op, static_cast<const float*>(a.data_ptr()),
                     static_cast<const float*>(b.data_ptr()), static_cast<float*>(out.data_ptr()),
                     static_cast<int>(sizes.size()), sizes.data(), sa.data(), sb.data(), alpha,
                     current_stream_handle()));
  return out;
}

}  // namespace

at::Tensor add_tensor(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha) {
  return binary(self, other, TVR_BINARY_ADD, static_cast<float>(alpha.toDouble()), "add");
}

at::Tensor mul_tensor(const at::Tensor& self, const at::Tensor& other) {
  return binary(self, other, TVR_BINARY_MUL, 1.f, "mul");
}

at::Tensor unary(const at::Tensor& self, int op, float scalar, const char* name) {
  at::Tensor in = ensure_fp32(self, name);
  TORCH_CHECK(is_device(in), name, ": expected a tvarant tensor");
  c10::DeviceGuard guard(in.device());
  if (!in.is_contiguous()) in = contiguous_copy(in);
  at::Tensor out = empty_device(in.sizes(), in.options());
  TVR_TRY(tvr_unary(op, static_cast<const float*>(in.data_ptr()),
                    static_cast<float*>(out.data_ptr()), in.numel(), scalar,
                    current_stream_handle()));
  return out;
}

at::Tensor add_scalar(const at::Tensor& self, const at::Scalar& other, const at::Scalar& alpha) {
  return unary(self, TVR_UNARY_ADD_SCALAR, static_cast<float>(other.toDouble() * alpha.toDouble()),
               "add");
}

// ---- registered kernels ---------------------------------------------------------

namespace {

at::Tensor empty_memory_format(c10::SymIntArrayRef size, std::optional<c10::ScalarType> dtype,
                               std::optional<c10::Layout> layout,
                               std::optional<c10::Device> device, std::optional<bool> pin_memory,
                               std::optional<c10::MemoryFormat> memory_format) {
  const auto dev = c10::device_or_default(device);
  TORCH_CHECK(dev.is_privateuseone(), "empty(): expected tvarant device");
  TORCH_CHECK(c10::layout_or_default(layout) == c10::Layout::Strided,
              "Tvarant only supports strided layout");
  TORCH_CHECK(!c10::pinned_memory_or_default(pin_memory), "Pin memory is only supported on CPU");
  c10::DeviceGuard guard(dev);
  return at::detail::empty_generic(C10_AS_INTARRAYREF_SLOW(size), allocator(), device_keys(),
                                   c10::dtype_or_default(dtype), memory_format);
}

at::Tensor empty_strided(c10::SymIntArrayRef size, c10::SymIntArrayRef stride,
                         std::optional<c10::ScalarType> dtype, std::optional<c10::Layout> layout,
                         std::optional<c10::Device> device, std::optional<bool> pin_memory) {
  const auto dev = c10::device_or_default(device);
  TORCH_CHECK(dev.is_privateuseone(), "empty_strided(): expected tvarant device");
  TORCH_CHECK(c10::layout_or_default(layout) == c10::Layout::Strided,
              "Tvarant only supports strided layout");
  TORCH_CHECK(!c10::pinned_memory_or_default(pin_memory), "Pin memory is only supported on CPU");
  c10::DeviceGuard guard(dev);
  return at::detail::empty_strided_generic(C10_AS_INTARRAYREF_SLOW(size),
                                           C10_AS_INTARRAYREF_SLOW(stride), allocator(),
                                           device_keys(), c10::dtype_or_default(dtype));
}

at::Tensor view_of(const at::Tensor& self, at::IntArrayRef size, at::IntArrayRef stride,
                   int64_t offset) {
  auto result = at::detail::make_tensor<c10::TensorImpl>(
      c10::TensorImpl::VIEW, c10::Storage(self.storage()), self.key_set(), self.dtype());
  at::native::setStrided(result, size, stride, offset);
  return result;
}

at::Tensor as_strided(const at::Tensor& self, c10::SymIntArrayRef size,
                      c10::SymIntArrayRef stride, std::optional<c10::SymInt> storage_offset) {
  const int64_t off = storage_offset.has_value() ? storage_offset->expect_int()
                                                 : self.storage_offset();
  return view_of(self, C10_AS_INTARRAYREF_SLOW(size), C10_AS_INTARRAYREF_SLOW(stride), off);
}

const at::Tensor& resize_(const at::Tensor& self, c10::SymIntArrayRef size_sym,
                          std::optional<c10::MemoryFormat> memory_format) {
  auto size = C10_AS_INTARRAYREF_SLOW(size_sym);
  auto* impl = self.unsafeGetTensorImpl();
  impl->set_sizes_contiguous(size);
  const auto itemsize = self.dtype().itemsize();
  const size_t needed = at::detail::computeStorageNbytesContiguous(size, itemsize) +
                        static_cast<size_t>(self.storage_offset()) * itemsize;
  if (!self.storage() || self.storage().nbytes() < needed) {
    at::detail::getPrivateUse1Hooks().resizePrivateUse1Bytes(self.storage(), needed);
  }
  if (memory_format.has_value()) impl->empty_tensor_restride(*memory_format);
  return self;
}

at::Tensor reshape_alias(const at::Tensor& self, c10::SymIntArrayRef size,
                         c10::SymIntArrayRef stride) {
  return view_of(self, C10_AS_INTARRAYREF_SLOW(size), C10_AS_INTARRAYREF_SLOW(stride),
                 self.storage_offset());
}

at::Tensor view(const at::Tensor& self, c10::SymIntArrayRef size_sym) {
  auto inferred = at::infer_size(C10_AS_INTARRAYREF_SLOW(size_sym), self.numel());
  auto stride = at::detail::computeStride(self.sizes(), self.strides(), inferred);
  TORCH_CHECK(stride.has_value(),
              "view size is not compatible with input tensor's size and stride; use reshape() "
              "instead");
  return view_of(self, inferred, *stride, self.storage_offset());
}

at::Tensor copy_from_and_resize(const at::Tensor& self, const at::Tensor& dst) {
  resize_(dst, self.sym_sizes(), std::nullopt);
  return copy_from(self, dst, false);
}

at::Scalar local_scalar_dense(const at::Tensor& self) {
  TORCH_CHECK(self.numel() == 1, "item() only supports tensors with one element");
  c10::DeviceGuard guard(self.device());
  at::Tensor cpu = at::empty({}, self.options().device(at::kCPU));
  TVR_TRY(tvr_memcpy_d2h(cpu.data_ptr(), self.data_ptr(), self.element_size(),
                         current_stream_handle()));
  sync_current_stream();
  return cpu.item();
}

at::Tensor& set_source_tensor(at::Tensor& self, const at::Tensor& source) {
  self.unsafeGetTensorImpl()->set_storage_keep_dtype(source.storage());
  at::native::setStrided(self, source.sizes(), source.strides(), source.storage_offset());
  return self;
}

at::Tensor& set_source_storage(at::Tensor& self, at::Storage source) {
  const int64_t n = static_cast<int64_t>(source.nbytes() / self.dtype().itemsize());
  const int64_t one = 1;
  self.unsafeGetTensorImpl()->set_storage_keep_dtype(std::move(source));
  at::native::setStrided(self, at::IntArrayRef(&n, 1), at::IntArrayRef(&one, 1), int64_t(0));
  return self;
}

at::Tensor& set_source_storage_offset(at::Tensor& self, at::Storage source, c10::SymInt offset,
                                      c10::SymIntArrayRef size, c10::SymIntArrayRef stride) {
  self.unsafeGetTensorImpl()->set_storage_keep_dtype(std::move(source));
  at::native::setStrided(self, C10_AS_INTARRAYREF_SLOW(size), C10_AS_INTARRAYREF_SLOW(stride),
                         offset.expect_int());
  return self;
}

bool compatible_shallow_copy(const at::Tensor&, const at::Tensor&) { return true; }

at::Tensor& write_into(const at::Tensor& value, at::Tensor& out) {
  if (!out.sizes().equals(value.sizes())) at::native::resize_output(out, value.sizes());
  copy_from(value, out, false);
  return out;
}

at::Tensor& add_out(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha,
                    at::Tensor& out) {
  return write_into(add_tensor(self, other, alpha), out);
}

at::Tensor& mul_out(const at::Tensor& self, const at::Tensor& other, at::Tensor& out) {
  return write_into(mul_tensor(self, other), out);
}

at::Tensor relu_op(const at::Tensor& self) {
  check_fp32(self, "relu");
  return unary(self, TVR_UNARY_RELU, 0.f, "relu");
}

at::Tensor& relu_inplace(at::Tensor& self) {
  at::Tensor r = relu_op(self);
  tvarant::ops::copy_from(r, self, false);
  return self;
}

at::Tensor& relu_out(const at::Tensor& self, at::Tensor& out) {
  return write_into(relu_op(self), out);
}

at::Tensor mm(const at::Tensor& self, const at::Tensor& mat2) {
  check_fp32(self, "mm");
  check_fp32(mat2, "mm");
  TORCH_CHECK(self.dim() == 2 && mat2.dim() == 2, "mm(): tensors must be 2D");
  TORCH_CHECK(self.size(1) == mat2.size(0), "mm(): size mismatch ", self.sizes(), " and ",
              mat2.sizes());
  return gemm_bias_act(self, mat2, nullptr, 1.f, 0.f, TVR_ACT_NONE, false);
}

// beta*self + alpha*(mat1 @ mat2); a 1-D (or [1, N]) self is fused as the
// GEMM bias, anything else is added afterwards (reference Ops.cpp:373-397).
at::Tensor addmm(const at::Tensor& self, const at::Tensor& mat1, const at::Tensor& mat2,
                 const at::Scalar& beta, const at::Scalar& alpha) {
  check_fp32(mat1, "addmm");
  check_fp32(mat2, "addmm");
  const float a = alpha.toFloat(), b = beta.toFloat();
  if (b == 0.f) return gemm_bias_act(mat1, mat2, nullptr, a, 0.f, TVR_ACT_NONE, false);
  at::Tensor bias = self.to(mat1.scalar_type());
  if (bias.dim() == 1 || (bias.dim() == 2 && bias.size(0) == 1)) {
    at::Tensor flat = bias.reshape({-1});
    return gemm_bias_act(mat1, mat2, &flat, a, b, TVR_ACT_NONE, false);
  }
  at::Tensor out = gemm_bias_act(mat1, mat2, nullptr, a, 0.f, TVR_ACT_NONE, false);
  at::Tensor scaled = b == 1.f ? bias : unary(to_device_like(bias, out), TVR_UNARY_SCALE, b, "addmm");
  return add_tensor(scaled, out, 1);
}

// Random fills draw on the host generator (as the reference, whose device
// generator is a CPU generator) and copy the values to the device.
template <typename Fn>
void host_random(at::Tensor& self, std::optional<at::Generator> gen, Fn&& draw) {
  at::Tensor host = at::empty(self.sizes(), self.options().device(at::kCPU));
  if (gen.has_value() && gen->defined() && gen->device().is_privateuseone()) {
    at::Generator cpu_gen = at::make_generator<at::CPUGeneratorImpl>();
    {
      std::lock_guard<std::mutex> lock(gen->mutex());
      cpu_gen.set_state(gen->get_state());
    }
    draw(host, std::optional<at::Generator>(cpu_gen));
    std::lock_guard<std::mutex> lock(gen->mutex());
    gen->set_state(cpu_gen.get_state());
  } else {
    draw(host, gen);
  }
  copy_from(host, self, false);
}

// A use of `self` on another stream: its block returns to the pool only
// after the work queued on `s` so far has run.
void record_stream(at::Tensor& self, c10::Stream s) {
  TORCH_CHECK(s.device_type() == c10::DeviceType::PrivateUse1,
              "record_stream: expected a tvarant stream, got ", s);
  void* base = self.storage().data_ptr().get();
  if (base == nullptr) return;
  TVR_TRY(tvr_record_stream(base, stream_handle(s.device_index(), s.id())));
}

at::Tensor& normal_(at::Tensor& self, double mean, double std, std::optional<at::Generator> gen) {
  host_random(self, gen, [&](at::Tensor& h, std::optional<at::Generator> g) { h.normal_(mean, std, g); });
  return self;
}

at::Tensor& uniform_(at::Tensor& self, double from, double to, std::optional<at::Generator> gen) {
  host_random(self, gen, [&](at::Tensor& h, std::optional<at::Generator> g) { h.uniform_(from, to, g); });
  return self;
}

}  // namespace
}  // namespace tvarant::ops

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("empty.memory_format", TORCH_FN(tvarant::ops::empty_memory_format));
  m.impl("empty_strided", TORCH_FN(tvarant::ops::empty_strided));
  m.impl("as_strided", TORCH_FN(tvarant::ops::as_strided));
  m.impl("resize_", TORCH_FN(tvarant::ops::resize_));
  m.impl("_reshape_alias", TORCH_FN(tvarant::ops::reshape_alias));
  m.impl("view", TORCH_FN(tvarant::ops::view));
  m.impl("_copy_from", TORCH_FN(tvarant::ops::copy_from));
  m.impl("_copy_from_and_resize", TORCH_FN(tvarant::ops::copy_from_and_resize));
  m.impl("_local_scalar_dense", TORCH_FN(tvarant::ops::local_scalar_dense));
  m.impl("set_.source_Tensor", TORCH_FN(tvarant::ops::set_source_tensor));
  m.impl("set_.source_Storage", TORCH_FN(tvarant::ops::set_source_storage));
  m.impl("set_.source_Storage_storage_offset", TORCH_FN(tvarant::ops::set_source_storage_offset));
  m.impl("_has_compatible_shallow_copy_type", TORCH_FN(tvarant::ops::compatible_shallow_copy));
  m.impl("fill_.Scalar", TORCH_FN(tvarant::ops::fill_scalar));
  m.impl("add.Tensor", TORCH_FN(tvarant::ops::add_tensor));
  m.impl("add.out", TORCH_FN(tvarant::ops::add_out));
  m.impl("mul.Tensor", TORCH_FN(tvarant::ops::mul_tensor));
  m.impl("mul.out", TORCH_FN(tvarant::ops::mul_out));
  m.impl("relu", TORCH_FN(tvarant::ops::relu_op));
  m.impl("relu_", TORCH_FN(tvarant::ops::relu_inplace));
  m.impl("relu.out", TORCH_FN(tvarant::ops::relu_out));
  m.impl("mm", TORCH_FN(tvarant::ops::mm));
  m.impl("addmm", TORCH_FN(tvarant::ops::addmm));
  m.impl("normal_", TORCH_FN(tvarant::ops::normal_));
  m.impl("record_stream", TORCH_FN(tvarant::ops::record_stream));
  m.impl("uniform_", TORCH_FN(tvarant::ops::uniform_));
}

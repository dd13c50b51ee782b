// Factories, clone / contiguous, unary maps and sub for the tvarant device.
//
// Registration list and semantics follow the reference's
// csrc/aten/ExtendedOps.cpp (:362-392); sub is add with -alpha
// (ExtendedOps.cpp:261-280).  clone / contiguous of a strided view run the
// device strided-copy kernel instead of the reference's host-view copy.
#include <ATen/ATen.h>
#include <c10/core/DeviceGuard.h>
#include <torch/library.h>

#include "TvarantExt.h"

namespace tvarant::ops {
namespace {

at::Tensor make_filled(at::IntArrayRef size, const at::Scalar& value,
                       std::optional<c10::ScalarType> dtype, std::optional<c10::Layout> layout,
                       std::optional<c10::Device> device, std::optional<bool> pin_memory) {
  const auto dev = c10::device_or_default(device);
  TORCH_CHECK(dev.is_privateuseone(), "expected tvarant device");
  TORCH_CHECK(c10::layout_or_default(layout) == c10::Layout::Strided,
              "Tvarant only supports strided layout");
  TORCH_CHECK(!c10::pinned_memory_or_default(pin_memory), "Pin memory is only supported on CPU");
  at::Tensor t = empty_device(size, at::TensorOptions().dtype(c10::dtype_or_default(dtype)).device(dev));
  fill_scalar(t, value);
  return t;
}

at::Tensor make_filled_like(const at::Tensor& self, const at::Scalar& value,
                            std::optional<c10::ScalarType> dtype, std::optional<c10::Layout> layout,
                            std::optional<c10::Device> device, std::optional<bool> pin_memory) {
  return make_filled(self.sizes(), value, dtype.value_or(self.scalar_type()),
                     layout.value_or(self.layout()), device.value_or(self.device()), pin_memory);
}

at::Tensor zeros(c10::SymIntArrayRef size, std::optional<c10::ScalarType> dtype,
                 std::optional<c10::Layout> layout, std::optional<c10::Device> device,
                 std::optional<bool> pin_memory) {
  return make_filled(C10_AS_INTARRAYREF_SLOW(size), 0, dtype, layout, device, pin_memory);
}

at::Tensor ones(c10::SymIntArrayRef size, std::optional<c10::ScalarType> dtype,
                std::optional<c10::Layout> layout, std::optional<c10::Device> device,
                std::optional<bool> pin_memory) {
  return make_filled(C10_AS_INTARRAYREF_SLOW(size), 1, dtype, layout, device, pin_memory);
}

at::Tensor full(c10::SymIntArrayRef size, const at::Scalar& value,
                std::optional<c10::ScalarType> dtype, std::optional<c10::Layout> layout,
                std::optional<c10::Device> device, std::optional<bool> pin_memory) {
  // like ATen, an unspecified dtype follows the fill value
  const auto dt = dtype.has_value() ? dtype : std::optional<c10::ScalarType>(
                                                  value.isFloatingPoint() ? at::get_default_dtype_as_scalartype()
                                                  : value.isBoolean()     ? at::kBool
                                                  : value.isIntegral(false) ? at::kLong
                                                                            : at::get_default_dtype_as_scalartype());
  return make_filled(C10_AS_INTARRAYREF_SLOW(size), value, dt, layout, device, pin_memory);
}

at::Tensor zeros_like(const at::Tensor& self, std::optional<c10::ScalarType> dtype,
                      std::optional<c10::Layout> layout, std::optional<c10::Device> device,
                      std::optional<bool> pin_memory, std::optional<c10::MemoryFormat>) {
  return make_filled_like(self, 0, dtype, layout, device, pin_memory);
}

at::Tensor ones_like(const at::Tensor& self, std::optional<c10::ScalarType> dtype,
                     std::optional<c10::Layout> layout, std::optional<c10::Device> device,
                     std::optional<bool> pin_memory, std::optional<c10::MemoryFormat>) {
  return make_filled_like(self, 1, dtype, layout, device, pin_memory);
}

at::Tensor full_like(const at::Tensor& self, const at::Scalar& value,
                     std::optional<c10::ScalarType> dtype, std::optional<c10::Layout> layout,
                     std::optional<c10::Device> device, std::optional<bool> pin_memory,
                     std::optional<c10::MemoryFormat>) {
  return make_filled_like(self, value, dtype, layout, device, pin_memory);
}

at::Tensor clone(const at::Tensor& self, std::optional<c10::MemoryFormat> memory_format) {
  c10::DeviceGuard guard(self.device());
  at::Tensor out;
  const auto mf = memory_format.value_or(c10::MemoryFormat::Preserve);
  if (mf == c10::MemoryFormat::Preserve && self.is_non_overlapping_and_dense()) {
    out = at::detail::empty_strided_generic(
        self.sizes(), self.strides(), allocator(),
        c10::DispatchKeySet{c10::DispatchKey::PrivateUse1, c10::DispatchKey::AutogradPrivateUse1},
        self.scalar_type());
  } else {
    out = empty_device(self.sizes(), self.options());
  }
  return copy_from(self, out, false);
}

at::Tensor contiguous(const at::Tensor& self, c10::MemoryFormat memory_format) {
  if (self.is_contiguous(memory_format)) return self;
  TORCH_CHECK(memory_format == c10::MemoryFormat::Contiguous,
              "tvarant contiguous: only the default memory format is supported");
  return contiguous_copy(self);
}

// op(self), op_(self), op.out(self, out) for one TVR_UNARY_* id
template <int OP>
struct Unary {
  static at::Tensor fn(const at::Tensor& self) { return unary(self, OP, 0.f, name()); }
  static at::Tensor& fn_(at::Tensor& self) {
    at::Tensor r = fn(self);
    copy_from(r, self, false);
    return self;
  }
  static at::Tensor& fn_out(const at::Tensor& self, at::Tensor& out) {
    at::Tensor r = fn(self);
    if (!out.sizes().equals(r.sizes())) out.resize_(r.sizes());
    copy_from(r, out, false);
    return out;
  }
  static const char* name() {
    switch (OP) {
      case TVR_UNARY_NEG: return "neg";
      case TVR_UNARY_ABS: return "abs";
      case TVR_UNARY_EXP: return "exp";
      case TVR_UNARY_EXP2: return "exp2";
      case TVR_UNARY_SQRT: return "sqrt";
      case TVR_UNARY_RSQRT: return "rsqrt";
      case TVR_UNARY_SIGMOID: return "sigmoid";
      default: return "unary";
    }
  }
};

at::Tensor sub_tensor(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha) {
  return add_tensor(self, other, -alpha.toDouble());
}

at::Tensor& sub_out(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha,
                    at::Tensor& out) {
  at::Tensor r = sub_tensor(self, other, alpha);
  if (!out.sizes().equals(r.sizes())) out.resize_(r.sizes());
  copy_from(r, out, false);
  return out;
}

at::Tensor sub_scalar(const at::Tensor& self, const at::Scalar& other, const at::Scalar& alpha) {
  return add_scalar(self, other, -alpha.toDouble());
}

}  // namespace
}  // namespace tvarant::ops

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("zeros", TORCH_FN(tvarant::ops::zeros));
  m.impl("zeros_like", TORCH_FN(tvarant::ops::zeros_like));
  m.impl("ones", TORCH_FN(tvarant::ops::ones));
  m.impl("ones_like", TORCH_FN(tvarant::ops::ones_like));
  m.impl("full", TORCH_FN(tvarant::ops::full));
  m.impl("full_like", TORCH_FN(tvarant::ops::full_like));
  m.impl("clone", TORCH_FN(tvarant::ops::clone));
  m.impl("contiguous", TORCH_FN(tvarant::ops::contiguous));
#define TVR_REG_UNARY(NAME, OP)                                   \
  m.impl(#NAME, TORCH_FN(tvarant::ops::Unary<OP>::fn));                         \
  m.impl(#NAME "_", TORCH_FN(tvarant::ops::Unary<OP>::fn_));                    \
  m.impl(#NAME ".out", TORCH_FN(tvarant::ops::Unary<OP>::fn_out));
  TVR_REG_UNARY(neg, TVR_UNARY_NEG)
  TVR_REG_UNARY(abs, TVR_UNARY_ABS)
  TVR_REG_UNARY(exp, TVR_UNARY_EXP)
  TVR_REG_UNARY(exp2, TVR_UNARY_EXP2)
  TVR_REG_UNARY(sqrt, TVR_UNARY_SQRT)
  TVR_REG_UNARY(rsqrt, TVR_UNARY_RSQRT)
  TVR_REG_UNARY(sigmoid, TVR_UNARY_SIGMOID)
#undef TVR_REG_UNARY
  m.impl("sub.Tensor", TORCH_FN(tvarant::ops::sub_tensor));
  m.impl("sub.out", TORCH_FN(tvarant::ops::sub_out));
  m.impl("sub.Scalar", TORCH_FN(tvarant::ops::sub_scalar));
}

// where / masked_fill / tril / triu / argmax on the tvarant device.
//
// The reference has no kernels for these and runs them on the CPU through its
// boxed fallback (csrc/aten/Ops.cpp:499-501); this backend has no fallback,
// so they are native: tvr_where (broadcast select) and tvr_triangle.  They are
// what PyTorch itself calls to build attention masks (a boolean attn_mask is
// turned into an additive one with where; is_causal masks come from tril).
#include <ATen/ATen.h>
#include <ATen/ExpandUtils.h>
#include <c10/core/DeviceGuard.h>
#include <torch/library.h>

#include <vector>

#include "TvarantExt.h"

namespace tvarant::ops {
namespace {

int select_elem_size(at::ScalarType t) {
  switch (t) {
    case at::kFloat:
    case at::kInt:
      return 4;
    case at::kLong:
    case at::kDouble:
      return 8;
    case at::kBool:
    case at::kByte:
      return 1;
    default:
      TORCH_CHECK(false, "Tvarant where/masked_fill/tril/triu: unsupported dtype ", t);
  }
}

// Output dtype of where(cond, a, b): float32 once either side is floating,
// else the common integral / bool type.
at::ScalarType select_dtype(const at::Tensor& a, const at::Tensor& b) {
  if (at::isFloatingType(a.scalar_type()) || at::isFloatingType(b.scalar_type())) return at::kFloat;
  return at::promote_types(a.scalar_type(), b.scalar_type());
}

at::Tensor as_type_on(const at::Tensor& t, at::ScalarType dt, const at::Tensor& like) {
  at::Tensor x = t;
  if (x.scalar_type() != dt) {
    // conversions of device tensors run on the device (tvr_convert via _copy_from)
    x = x.to(dt);
  }
  return to_device_like(x, like);
}

at::Tensor where_self(const at::Tensor& condition, const at::Tensor& self, const at::Tensor& other) {
  const at::Tensor& anchor = is_device(self) ? self : (is_device(other) ? other : condition);
  TORCH_CHECK(is_device(anchor), "where: expected at least one tvarant tensor");
  c10::DeviceGuard guard(anchor.device());
  const at::ScalarType dt = select_dtype(self, other);
  at::Tensor a = as_type_on(self, dt, anchor);
  at::Tensor b = as_type_on(other, dt, anchor);
  at::Tensor c = as_type_on(condition, at::kBool, anchor);
  const auto shape = at::infer_size(at::infer_size(c.sizes(), a.sizes()), b.sizes());
  at::Tensor out = empty_device(shape, a.options());
  if (out.numel() == 0) return out;
  const at::Tensor ce = c.expand(shape), ae = a.expand(shape), be = b.expand(shape);
  TVR_TRY(tvr_where(ce.data_ptr(), ae.data_ptr(), be.data_ptr(), out.data_ptr(),
                    select_elem_size(dt), static_cast<int>(shape.size()), shape.data(),
                    ce.strides().data(), ae.strides().data(), be.strides().data(),
                    current_stream_handle()));
  return out;
}

at::Tensor& masked_fill_tensor_(at::Tensor& self, const at::Tensor& mask, const at::Tensor& value) {
  TORCH_CHECK(value.dim() == 0, "masked_fill_: value must be a 0-dim tensor, got ", value.dim(),
              " dimensions");
  c10::DeviceGuard guard(self.device());
  at::Tensor filled = where_self(mask, value, self);
  TORCH_CHECK(filled.sizes() == self.sizes(), "masked_fill_: mask ", mask.sizes(),
              " does not broadcast to ", self.sizes());
  self.copy_(filled);
  return self;
}

at::Tensor& masked_fill_scalar_(at::Tensor& self, const at::Tensor& mask, const at::Scalar& value) {
  return masked_fill_tensor_(self, mask, at::scalar_tensor(value, at::TensorOptions().dtype(
                                                                       self.scalar_type())));
}

at::Tensor triangle(const at::Tensor& self, int64_t diagonal, bool upper) {
  TORCH_CHECK(self.dim() >= 2, upper ? "triu" : "tril", ": input tensor must have at least 2 dimensions");
  c10::DeviceGuard guard(self.device());
  at::Tensor x = self.is_contiguous() ? self : contiguous_copy(self);
  at::Tensor out = empty_device(x.sizes(), x.options());
  const int64_t rows = x.size(-2), cols = x.size(-1);
  const int64_t batch = rows * cols > 0 ? x.numel() / (rows * cols) : 0;
  TVR_TRY(tvr_triangle(x.data_ptr(), out.data_ptr(), select_elem_size(x.scalar_type()), batch, rows,
                       cols, diagonal, upper ? 1 : 0, current_stream_handle()));
  return out;
}

at::Tensor tril(const at::Tensor& self, int64_t diagonal) { return triangle(self, diagonal, false); }
at::Tensor triu(const at::Tensor& self, int64_t diagonal) { return triangle(self, diagonal, true); }

at::Tensor& tril_(at::Tensor& self, int64_t diagonal) {
  self.copy_(triangle(self, diagonal, false));
  return self;
}

at::Tensor& triu_(at::Tensor& self, int64_t diagonal) {
  self.copy_(triangle(self, diagonal, true));
  return self;
}

// argmax over one dimension (or the flattened tensor when dim is None): the
// reduced dimension is made the last, contiguous one, then one row per
// remaining index (tvr_argmax_rows).
at::Tensor argmax(const at::Tensor& self, std::optional<int64_t> dim, bool keepdim) {
  check_fp32(self, "argmax");
  c10::DeviceGuard guard(self.device());
  TORCH_CHECK(self.numel() > 0, "argmax(): Expected reduction dim to be specified for input.numel() == 0.");
  at::Tensor x;
  std::vector<int64_t> out_shape;
  if (!dim.has_value()) {
    x = (self.is_contiguous() ? self : contiguous_copy(self)).reshape({1, self.numel()});
    if (keepdim) out_shape.assign(self.dim(), 1);
  } else {
    const int64_t d = at::maybe_wrap_dim(*dim, self.dim());
    at::Tensor moved = self.dim() == 0 ? self.reshape({1}) : self.movedim(d, -1);
    at::Tensor c = moved.is_contiguous() ? moved : contiguous_copy(moved);
    const int64_t n = c.dim() == 0 ? 1 : c.size(-1);
    x = c.reshape({c.numel() / n, n});
    out_shape = self.sizes().vec();
    if (self.dim() > 0) {
      if (keepdim) out_shape[d] = 1;
      else out_shape.erase(out_shape.begin() + d);
    }
  }
  at::Tensor out = empty_device({x.size(0)}, x.options().dtype(at::kLong));
  TVR_TRY(tvr_argmax_rows(static_cast<const float*>(x.data_ptr()),
                          static_cast<int64_t*>(out.data_ptr()), x.size(0), x.size(1),
                          current_stream_handle()));
  return out.reshape(out_shape);
}

at::Tensor logical_not(const at::Tensor& self) {
  c10::DeviceGuard guard(self.device());
  at::Tensor b = as_type_on(self, at::kBool, self);
  at::Tensor t = at::scalar_tensor(false, at::TensorOptions().dtype(at::kBool));
  at::Tensor f = at::scalar_tensor(true, at::TensorOptions().dtype(at::kBool));
  return where_self(b, t, f);
}

}  // namespace
}  // namespace tvarant::ops

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("where.self", TORCH_FN(tvarant::ops::where_self));
  m.impl("masked_fill_.Scalar", TORCH_FN(tvarant::ops::masked_fill_scalar_));
  m.impl("masked_fill_.Tensor", TORCH_FN(tvarant::ops::masked_fill_tensor_));
  m.impl("tril", TORCH_FN(tvarant::ops::tril));
  m.impl("triu", TORCH_FN(tvarant::ops::triu));
  m.impl("tril_", TORCH_FN(tvarant::ops::tril_));
  m.impl("triu_", TORCH_FN(tvarant::ops::triu_));
  m.impl("logical_not", TORCH_FN(tvarant::ops::logical_not));
  m.impl("argmax", TORCH_FN(tvarant::ops::argmax));
}

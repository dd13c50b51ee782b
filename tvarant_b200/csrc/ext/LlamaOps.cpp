// RMSNorm (aten::rms_norm, i.e. F.rms_norm) and rotary position embedding
// (tvarant::rope) on the tvarant device: tvr_rms_norm / tvr_rope.  The
// reference has neither op.
//
// aten::rms_norm is a composite op; the kernel is registered for the
// PrivateUse1 key and its autograd key, so tvarant tensors reach it instead
// of the pow / mean / rsqrt / mul decomposition.  Like the rest of this
// backend it computes forward values only.
#include <ATen/ATen.h>
#include <c10/core/DeviceGuard.h>
#include <torch/library.h>

#include <limits>

#include "TvarantExt.h"

namespace tvarant::ops {
namespace {

at::Tensor rms_norm(const at::Tensor& input, c10::SymIntArrayRef normalized_shape,
                    const std::optional<at::Tensor>& weight, std::optional<double> eps) {
  check_fp32(input, "rms_norm");
  const int64_t nd = static_cast<int64_t>(normalized_shape.size());
  TORCH_CHECK(nd >= 1 && nd <= input.dim(), "rms_norm: normalized_shape ", normalized_shape,
              " does not fit input of shape ", input.sizes());
  int64_t n = 1;
  for (int64_t i = 0; i < nd; ++i) {
    const int64_t want = normalized_shape[i].expect_int();
    TORCH_CHECK(input.size(input.dim() - nd + i) == want, "rms_norm: normalized_shape ",
                normalized_shape, " does not match the input's trailing sizes ", input.sizes());
    n *= want;
  }
  c10::DeviceGuard guard(input.device());
  at::Tensor x = input.is_contiguous() ? input : contiguous_copy(input);
  at::Tensor w;
  if (weight.has_value() && weight->defined()) {
    w = to_device_like(*weight, x);
    check_fp32(w, "rms_norm");
    TORCH_CHECK(w.numel() == n, "rms_norm: weight has ", w.numel(), " elements, expected ", n);
    if (!w.is_contiguous()) w = contiguous_copy(w);
  }
  at::Tensor y = empty_device(x.sizes(), x.options());
  const int64_t rows = n > 0 ? x.numel() / n : 0;
  if (rows == 0 || n == 0) return y;
  const float e = eps.has_value() ? static_cast<float>(*eps) : std::numeric_limits<float>::epsilon();
  TVR_TRY(tvr_rms_norm(static_cast<const float*>(x.data_ptr()),
                       w.defined() ? static_cast<const float*>(w.data_ptr()) : nullptr,
                       static_cast<float*>(y.data_ptr()), nullptr, rows, n, e,
                       current_stream_handle()));
  return y;
}

// x [B, H, S, D] (or [H, S, D], [S, D]; any strides with D contiguous): the
// rotation of position pos_offset + s by the angle tables cos / sin of shape
// [..., T, D/2] or [..., T, D] (only the first D/2 columns are read).
at::Tensor rope(const at::Tensor& x_in, const at::Tensor& cos, const at::Tensor& sin,
                int64_t pos_offset, bool interleaved) {
  check_fp32(x_in, "rope");
  TORCH_CHECK(x_in.dim() >= 2 && x_in.dim() <= 4, "rope: expected x of 2 to 4 dims, got ",
              x_in.sizes());
  c10::DeviceGuard guard(x_in.device());
  at::Tensor x = x_in.stride(-1) == 1 ? x_in : contiguous_copy(x_in);
  while (x.dim() < 4) x = x.unsqueeze(0);
  const int64_t B = x.size(0), H = x.size(1), S = x.size(2), D = x.size(3);
  TORCH_CHECK(D % 2 == 0, "rope: head dim ", D, " is odd");
  auto table = [&](const at::Tensor& t, const char* name) {
    at::Tensor u = to_device_like(t, x);
    check_fp32(u, "rope");
    TORCH_CHECK(u.dim() >= 2, "rope: ", name, " must be [T, D/2] or [T, D]");
    for (int64_t i = 0; i + 2 < u.dim(); ++i) {
      TORCH_CHECK(u.size(i) == 1, "rope: ", name, " ", u.sizes(), " must be one table");
    }
    u = u.reshape({u.size(-2), u.size(-1)});
    TORCH_CHECK(u.size(1) == D / 2 || u.size(1) == D, "rope: ", name, " has ", u.size(1),
                " columns, expected ", D / 2, " or ", D);
    return u.is_contiguous() ? u : contiguous_copy(u);
  };
  at::Tensor c = table(cos, "cos"), s = table(sin, "sin");
  TORCH_CHECK(c.sizes() == s.sizes(), "rope: cos ", c.sizes(), " and sin ", s.sizes(), " differ");
  at::Tensor y = empty_device(x_in.sizes(), x.options());
  at::Tensor yv = y;
  while (yv.dim() < 4) yv = yv.unsqueeze(0);
  const int64_t xs[3] = {x.stride(0), x.stride(2), x.stride(1)};   // batch, position, head
  const int64_t ys[3] = {yv.stride(0), yv.stride(2), yv.stride(1)};
  TVR_TRY(tvr_rope(static_cast<const float*>(x.data_ptr()), static_cast<float*>(y.data_ptr()),
                   static_cast<const float*>(c.data_ptr()), static_cast<const float*>(s.data_ptr()),
                   B, S, H, D, xs, ys, c.size(0), c.size(1), pos_offset, interleaved ? 1 : 0,
                   current_stream_handle()));
  return y;
}

}  // namespace
}  // namespace tvarant::ops

TORCH_LIBRARY_FRAGMENT(tvarant, m) {
  m.def("rope(Tensor x, Tensor cos, Tensor sin, int pos_offset=0, bool interleaved=False) -> Tensor");
}

TORCH_LIBRARY_IMPL(tvarant, PrivateUse1, m) { m.impl("rope", TORCH_FN(tvarant::ops::rope)); }

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) { m.impl("rms_norm", TORCH_FN(tvarant::ops::rms_norm)); }

TORCH_LIBRARY_IMPL(aten, AutogradPrivateUse1, m) {
  m.impl("rms_norm", TORCH_FN(tvarant::ops::rms_norm));
}

// The tvarant operator library: tvarant::linear_act, tvarant::pointwise,
// tvarant::linear_swiglu, tvarant::linear_pointwise and tvarant::softmax_add.
//
// Schemas are the reference's, verbatim (csrc/aten/CustomOps.cpp:101-106),
// so graphs produced by torch_tvarant.compiler run unchanged.  linear_act
// is one tcgen05 GEMM with bias and activation fused in the epilogue;
// pointwise compiles its SSA program with NVRTC (tvr_pointwise).  Opcodes
// 0-8 are the reference's (csrc/jit/Jit.h:11-21); 9 Sub, 10 Exp, 11 Abs are
// appended.
#include <ATen/ATen.h>
#include <c10/core/DeviceGuard.h>
#include <torch/library.h>

#include <string>
#include <vector>

#include "TvarantExt.h"

namespace tvarant::ops {
namespace {

// "none" / "identity" / "" -> 0, "relu" -> 1, "silu" / "swish" -> 2
// (reference csrc/jit/Jit.cpp:140-152).
int parse_act(const std::string& name) {
  if (name.empty() || name == "none" || name == "identity") return TVR_ACT_NONE;
  if (name == "relu") return TVR_ACT_RELU;
  if (name == "silu" || name == "swish") return TVR_ACT_SILU;
  TORCH_CHECK(false, "unknown activation '", name, "' (expected none|relu|silu)");
}

at::Tensor linear_act(const at::Tensor& x, const at::Tensor& weight,
                      const std::optional<at::Tensor>& bias, std::string act, bool trans_b) {
  check_fp32(x, "linear_act");
  check_fp32(weight, "linear_act");
  const int act_id = parse_act(act);
  TORCH_CHECK(x.dim() >= 1, "linear_act: expected at least 1D input");
  at::Tensor xc = x.is_contiguous() ? x : contiguous_copy(x);
  const int64_t k = xc.size(-1);
  const int64_t m = k > 0 ? xc.numel() / k : 0;
  at::Tensor x2 = xc.reshape({m, k});
  const at::Tensor* bptr = nullptr;
  at::Tensor bstore;
  if (bias.has_value() && bias->defined()) {
    check_fp32(*bias, "linear_act");
    bstore = *bias;
    bptr = &bstore;
  }
  at::Tensor y2 = gemm_bias_act(x2, weight, bptr, 1.f, 1.f, act_id, trans_b);
  auto out_sizes = xc.sizes().vec();
  out_sizes.back() = y2.size(1);
  return y2.reshape(out_sizes);
}

// silu(x . w_gate^T) * (x . w_up^T): the gated projection of a SwiGLU MLP as
// one GEMM (tvr_gemm_swiglu).  Weights are [N, K] (nn.Linear layout).  Not a
// reference op: the reference spells it linear_act(x, w_gate, None, "silu",
// True) * linear(x, w_up), which torch_tvarant.compiler rewrites into this.
at::Tensor linear_swiglu(const at::Tensor& x, const at::Tensor& w_gate, const at::Tensor& w_up) {
  check_fp32(x, "linear_swiglu");
  check_fp32(w_gate, "linear_swiglu");
  check_fp32(w_up, "linear_swiglu");
  TORCH_CHECK(x.dim() >= 1 && w_gate.dim() == 2 && w_up.dim() == 2,
              "linear_swiglu: expected x [..., K] and weights [N, K]");
  TORCH_CHECK(w_gate.sizes() == w_up.sizes(), "linear_swiglu: gate and up weights differ in shape (",
              w_gate.sizes(), " vs ", w_up.sizes(), ")");
  const int64_t k = x.size(-1);
  TORCH_CHECK(w_gate.size(1) == k, "linear_swiglu: x has ", k, " features, weights expect ",
              w_gate.size(1));
  TORCH_CHECK(x.device() == w_gate.device() && x.device() == w_up.device(),
              "linear_swiglu: operands on different devices");
  c10::DeviceGuard guard(x.device());
  at::Tensor xc = x.is_contiguous() ? x : contiguous_copy(x);
  at::Tensor wg = w_gate.stride(1) == 1 ? w_gate : contiguous_copy(w_gate);
  at::Tensor wu = w_up.stride(1) == 1 ? w_up : contiguous_copy(w_up);
  const int64_t n = wg.size(0);
  const int64_t m = k > 0 ? xc.numel() / k : 0;
  auto out_sizes = xc.sizes().vec();
  out_sizes.back() = n;
  at::Tensor out = empty_device(out_sizes, xc.options());
  if (m == 0 || n == 0) return out;
  TVR_TRY(tvr_gemm_swiglu(xc.data_ptr<float>(), wg.data_ptr<float>(), wu.data_ptr<float>(),
                          out.data_ptr<float>(), m, n, k, k, wg.stride(0), wu.stride(0), n,
                          gemm_mode(), current_stream_handle()));
  return out;
}

at::Tensor pointwise(at::TensorList inputs, at::IntArrayRef ops, at::IntArrayRef a,
                     at::IntArrayRef b, at::IntArrayRef input_ids, at::ArrayRef<double> alphas,
                     at::ArrayRef<double> consts) {
  TORCH_CHECK(!inputs.empty(), "pointwise: need at least one input");
  const size_t n_nodes = ops.size();
  TORCH_CHECK(a.size() == n_nodes && b.size() == n_nodes && input_ids.size() == n_nodes &&
                  alphas.size() == n_nodes && consts.size() == n_nodes,
              "pointwise: SSA arrays must all have the same length");
  TORCH_CHECK(n_nodes > 0, "pointwise: empty program");
  TORCH_CHECK(inputs.size() <= TVR_PW_MAX_INPUTS, "pointwise: at most ", TVR_PW_MAX_INPUTS,
              " inputs");
  std::vector<tvr_pw_node> prog(n_nodes);
  for (size_t i = 0; i < n_nodes; ++i) {
    prog[i].op = static_cast<int32_t>(ops[i]);
    prog[i].a = static_cast<int32_t>(a[i]);
    prog[i].b = static_cast<int32_t>(b[i]);
    prog[i].input_id = static_cast<int32_t>(input_ids[i]);
    prog[i].alpha = static_cast<float>(alphas[i]);
    prog[i].c = static_cast<float>(consts[i]);
  }
  // Inputs of equal numel are taken element by element (the reference's
  // contract); otherwise they are broadcast to a common shape first, which
  // the reference's fuser can produce but its kernel rejects.
  bool same_numel = true;
  std::vector<int64_t> shape = inputs[0].sizes().vec();
  for (const auto& t : inputs) {
    check_fp32(t, "pointwise");
    TORCH_CHECK(t.device().is_privateuseone(), "pointwise: expected tvarant tensors");
    same_numel = same_numel && t.numel() == inputs[0].numel();
    shape = at::infer_size(shape, t.sizes());
  }
  if (same_numel) shape = inputs[0].sizes().vec();
  c10::DeviceGuard guard(inputs[0].device());
  std::vector<at::Tensor> held;
  std::vector<const float*> ptrs;
  for (const auto& t : inputs) {
    at::Tensor c = t;
    if (!same_numel && !t.sizes().equals(shape)) c = contiguous_copy(t.expand(shape));
    else if (!c.is_contiguous()) c = contiguous_copy(c);
    ptrs.push_back(static_cast<const float*>(c.data_ptr()));
    held.push_back(std::move(c));
  }
  const int64_t numel = held[0].numel();
  at::Tensor out = empty_device(shape, inputs[0].options());
  TVR_TRY(tvr_pointwise(prog.data(), static_cast<int>(n_nodes), static_cast<int>(inputs.size()),
                        ptrs.data(), static_cast<float*>(out.data_ptr()), numel,
                        current_stream_handle()));
  return out;
}

// pointwise(inputs', program) where inputs' is `inputs` with
// linear_act(x, weight, bias, act, trans_b) inserted at position gemm_input:
// the GEMM -> pointwise pair torch_tvarant.compiler emits, as one call.  The
// program runs in the GEMM's epilogue (tvr_gemm_pointwise) when its other
// inputs are the GEMM output's size (contiguous) or one broadcast row of it;
// otherwise the two ops run as written.
at::Tensor linear_pointwise(const at::Tensor& x, const at::Tensor& weight,
                            const std::optional<at::Tensor>& bias, std::string act, bool trans_b,
                            int64_t gemm_input, at::TensorList inputs, at::IntArrayRef ops,
                            at::IntArrayRef a, at::IntArrayRef b, at::IntArrayRef input_ids,
                            at::ArrayRef<double> alphas, at::ArrayRef<double> consts) {
  check_fp32(x, "linear_pointwise");
  check_fp32(weight, "linear_pointwise");
  TORCH_CHECK(gemm_input >= 0 && gemm_input <= static_cast<int64_t>(inputs.size()),
              "linear_pointwise: gemm_input ", gemm_input, " out of range");
  TORCH_CHECK(x.dim() >= 1 && weight.dim() == 2, "linear_pointwise: expected x [..., K], weight 2D");
  const size_t n_nodes = ops.size();
  TORCH_CHECK(a.size() == n_nodes && b.size() == n_nodes && input_ids.size() == n_nodes &&
                  alphas.size() == n_nodes && consts.size() == n_nodes,
              "linear_pointwise: SSA arrays must all have the same length");
  c10::DeviceGuard guard(x.device());
  const int64_t n = trans_b ? weight.size(0) : weight.size(1);
  auto y_sizes = x.sizes().vec();
  y_sizes.back() = n;
  const int64_t numel = c10::multiply_integers(y_sizes);
  const int64_t m = n > 0 ? numel / n : 0;

  // Can the program run in the epilogue?  Every other input must be the
  // GEMM output's size (taken element by element, as tvarant::pointwise
  // does) or one row of n values that broadcasts to it.
  bool fused = n_nodes <= 12 && inputs.size() <= 2 && n_nodes > 0;
  bool same_numel = true;
  std::vector<int64_t> shape = y_sizes;
  for (const auto& t : inputs) {
    fused = fused && t.defined() && t.scalar_type() == at::kFloat && is_device(t) &&
            t.device() == x.device() && t.is_contiguous();
    if (!fused) break;
    if (t.numel() == numel) continue;
    same_numel = false;
    fused = t.numel() == n && at::infer_size(y_sizes, t.sizes()) == y_sizes;
  }
  if (fused) {
    // output shape: input 0's when all sizes agree, else the broadcast shape
    if (same_numel && gemm_input != 0) shape = inputs[0].sizes().vec();
    GemmProgram prog;
    prog.gemm_input = static_cast<int>(gemm_input);
    prog.nodes.resize(n_nodes);
    for (size_t i = 0; i < n_nodes; ++i) {
      prog.nodes[i].op = static_cast<int32_t>(ops[i]);
      prog.nodes[i].a = static_cast<int32_t>(a[i]);
      prog.nodes[i].b = static_cast<int32_t>(b[i]);
      prog.nodes[i].input_id = static_cast<int32_t>(input_ids[i]);
      prog.nodes[i].alpha = static_cast<float>(alphas[i]);
      prog.nodes[i].c = static_cast<float>(consts[i]);
    }
    size_t e = 0;
    for (int64_t i = 0; i <= static_cast<int64_t>(inputs.size()); ++i) {
      if (i == gemm_input) {
        prog.inputs.push_back(nullptr);
        prog.ld.push_back(0);
        continue;
      }
      const at::Tensor& t = inputs[e++];
      prog.inputs.push_back(static_cast<const float*>(t.data_ptr()));
      prog.ld.push_back(t.numel() == numel ? n : 0);
    }
    at::Tensor xc = x.is_contiguous() ? x : contiguous_copy(x);
    const int64_t k = xc.size(-1);
    const at::Tensor* bptr = nullptr;
    at::Tensor bstore;
    if (bias.has_value() && bias->defined()) {
      check_fp32(*bias, "linear_pointwise");
      bstore = *bias;
      bptr = &bstore;
    }
    at::Tensor y2 = gemm_bias_act(xc.reshape({m, k}), weight, bptr, 1.f, 1.f, parse_act(act),
                                  trans_b, &prog);
    return y2.reshape(shape);
  }
  std::vector<at::Tensor> all(inputs.begin(), inputs.end());
  all.insert(all.begin() + gemm_input, linear_act(x, weight, bias, act, trans_b));
  return pointwise(all, ops, a, b, input_ids, alphas, consts);
}

// softmax(x + mask, dim=-1) with the additive mask applied as each row is
// loaded (tvr_softmax_add): the attention-scores pattern
// softmax(q k^T * scale + mask) without the [.., L, S] round trip of the add.
// The mask must be a contiguous trailing block of x's shape (e.g. [L, S] for
// scores [B, H, L, S]); other shapes, and rows the fused kernel does not
// take, run the add and the softmax as written.
at::Tensor softmax_add(const at::Tensor& x, const at::Tensor& mask) {
  check_fp32(x, "softmax_add");
  TORCH_CHECK(x.dim() >= 1, "softmax_add: expected at least 1D scores");
  c10::DeviceGuard guard(x.device());
  at::Tensor m = to_device_like(mask, x);
  check_fp32(m, "softmax_add");
  const int64_t dim = x.size(-1);
  const int64_t k = x.dim() - m.dim();
  bool trailing = k >= 0 && m.dim() >= 1 && m.is_contiguous();
  for (int64_t i = 0; trailing && i < m.dim(); ++i) trailing = m.size(i) == x.size(k + i);
  if (trailing && dim > 0 && x.numel() > 0) {
    at::Tensor xc = x.is_contiguous() ? x : contiguous_copy(x);
    at::Tensor out = empty_device(xc.sizes(), xc.options());
    const int64_t rows = xc.numel() / dim;
    const int64_t mask_rows = m.numel() / dim;
    const int rc = tvr_softmax_add(static_cast<const float*>(xc.data_ptr()),
                                   static_cast<const float*>(m.data_ptr()),
                                   static_cast<float*>(out.data_ptr()), rows, dim, mask_rows,
                                   current_stream_handle());
    if (rc == TVR_OK) return out;
    TORCH_CHECK(rc == TVR_ERR_UNSUPPORTED, "tvarant: ", tvr_last_error());
  }
  return at::_softmax(at::add(x, m), -1, false);
}

}  // namespace
}  // namespace tvarant::ops

TORCH_LIBRARY(tvarant, m) {
  m.def("linear_act(Tensor x, Tensor weight, Tensor? bias, str act, bool trans_b=False) -> Tensor");
  m.def(
      "pointwise(Tensor[] inputs, int[] ops, int[] a, int[] b, int[] input_ids, float[] alphas, "
      "float[] consts) -> Tensor");
  m.def("all_reduce_(Tensor(a!) self, int comm) -> Tensor(a!)");
  m.def("linear_swiglu(Tensor x, Tensor w_gate, Tensor w_up) -> Tensor");
  m.def(
      "linear_pointwise(Tensor x, Tensor weight, Tensor? bias, str act, bool trans_b, "
      "int gemm_input, Tensor[] inputs, int[] ops, int[] a, int[] b, int[] input_ids, "
      "float[] alphas, float[] consts) -> Tensor");
  m.def("softmax_add(Tensor x, Tensor mask) -> Tensor");
}

TORCH_LIBRARY_IMPL(tvarant, PrivateUse1, m) {
  m.impl("linear_act", TORCH_FN(tvarant::ops::linear_act));
  m.impl("pointwise", TORCH_FN(tvarant::ops::pointwise));
  m.impl("linear_swiglu", TORCH_FN(tvarant::ops::linear_swiglu));
  m.impl("linear_pointwise", TORCH_FN(tvarant::ops::linear_pointwise));
  m.impl("softmax_add", TORCH_FN(tvarant::ops::softmax_add));
}

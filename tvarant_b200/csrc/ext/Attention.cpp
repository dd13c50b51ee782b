// F.scaled_dot_product_attention on the tvarant device.
//
// PyTorch routes SDPA on an out-of-tree device through two hooks: the
// `_fused_sdp_choice` dispatch stub picks a backend, and the "overrideable"
// backend calls aten::_scaled_dot_product_fused_attention_overrideable.  Here
// every fp32 4-D call without dropout takes the overrideable entry, which runs
// the fused tcgen05 attention kernel (tvr_attention_fwd: TF32, head dim 64)
// and otherwise composes the device's own ops — matmul (3xTF32 or TF32
// GEMMs), the additive causal / attention mask, softmax, matmul — the
// formulation the reference uses for attention (csrc/aten/LlmOps.cpp:68-148).
// Forward only.
#include <ATen/ATen.h>
#include <ATen/SDPBackend.h>
#include <ATen/native/DispatchStub.h>
#include <ATen/native/transformers/attention.h>
#include <c10/core/DeviceGuard.h>
#include <torch/library.h>

#include <array>
#include <cmath>
#include <limits>
#include <tuple>

#include "TvarantExt.h"

namespace tvarant::ops {

int64_t fused_sdp_choice(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                         const std::optional<at::Tensor>& attn_mask, double dropout_p,
                         bool is_causal, std::optional<double> scale, bool enable_gqa) {
  (void)attn_mask;
  (void)is_causal;
  (void)scale;
  const bool ok = q.scalar_type() == at::kFloat && k.scalar_type() == at::kFloat &&
                  v.scalar_type() == at::kFloat && q.dim() == 4 && k.dim() == 4 &&
                  v.dim() == 4 && dropout_p == 0.0 && (!enable_gqa || k.size(1) == q.size(1));
  return static_cast<int64_t>(ok ? at::SDPBackend::overrideable : at::SDPBackend::math);
}

namespace {

// Additive float mask on the device from a bool (true = attend) or float mask.
at::Tensor additive_mask(const at::Tensor& mask, const at::Tensor& like) {
  if (mask.scalar_type() == at::kBool) {
    at::Tensor host = mask.cpu();
    at::Tensor add = at::zeros(host.sizes(), host.options().dtype(at::kFloat));
    add.masked_fill_(host.logical_not(), -std::numeric_limits<float>::infinity());
    return add.to(like.device());
  }
  return ensure_fp32(to_device_like(mask, like), "scaled_dot_product_attention");
}

at::Tensor composed_attention(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                              const std::optional<at::Tensor>& attn_bias, bool is_causal,
                              double scale) {
  const int64_t L = q.size(2), S = k.size(2);
  at::Tensor scores = at::matmul(q, k.transpose(-2, -1)) * scale;
  if (is_causal) {
    at::Tensor causal = at::full({L, S}, -std::numeric_limits<float>::infinity(),
                                 at::TensorOptions().dtype(at::kFloat))
                            .triu(1)
                            .to(q.device());
    scores = scores + causal;
  }
  if (attn_bias.has_value() && attn_bias->defined()) scores = scores + additive_mask(*attn_bias, q);
  return at::matmul(at::_softmax(scores, -1, false), v);
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, c10::SymInt, c10::SymInt, at::Tensor,
           at::Tensor, at::Tensor>
sdpa_overrideable(const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
                  const std::optional<at::Tensor>& attn_bias, double dropout_p, bool is_causal,
                  bool return_debug_mask, std::optional<double> scale) {
  (void)return_debug_mask;
  TORCH_CHECK(dropout_p == 0.0,
              "scaled_dot_product_attention: dropout is not supported on the tvarant device");
  TORCH_CHECK(query.dim() == 4 && key.dim() == 4 && value.dim() == 4,
              "scaled_dot_product_attention: expected 4-D query, key and value");
  check_fp32(query, "scaled_dot_product_attention");
  check_fp32(key, "scaled_dot_product_attention");
  check_fp32(value, "scaled_dot_product_attention");
  const int64_t B = query.size(0), H = query.size(1), L = query.size(2), E = query.size(3);
  const int64_t S = key.size(2), Ev = value.size(3);
  TORCH_CHECK(key.size(0) == B && value.size(0) == B && key.size(1) == H && value.size(1) == H &&
                  value.size(2) == S && key.size(3) == E,
              "scaled_dot_product_attention: query ", query.sizes(), ", key ", key.sizes(),
              " and value ", value.sizes(), " do not match");
  const double sc = scale.has_value() ? *scale : 1.0 / std::sqrt(static_cast<double>(E));
  c10::DeviceGuard guard(query.device());
  const at::Tensor none = at::empty({0}, query.options());
  auto result = [&](const at::Tensor& out, const at::Tensor& lse) {
    return std::make_tuple(out, lse, none, none, c10::SymInt(L), c10::SymInt(S), none, none, none);
  };
  const bool masked = attn_bias.has_value() && attn_bias->defined();
  if (!masked && E == Ev && L > 0 && S > 0) {
    auto last_unit = [](const at::Tensor& t) { return t.stride(3) == 1 ? t : contiguous_copy(t); };
    const at::Tensor q = last_unit(query), k = last_unit(key), v = last_unit(value);
    // output laid out [B, L, H, E] and returned as the [B, H, L, E] view
    at::Tensor out_buf = empty_device({B, L, H, Ev}, query.options());
    at::Tensor out = out_buf.permute({0, 2, 1, 3});
    at::Tensor lse = empty_device({B, H, L}, query.options());
    const int64_t qs[3] = {q.stride(0), q.stride(1), q.stride(2)};
    const int64_t ks[3] = {k.stride(0), k.stride(1), k.stride(2)};
    const int64_t vs[3] = {v.stride(0), v.stride(1), v.stride(2)};
    const int64_t os[3] = {out.stride(0), out.stride(1), out.stride(2)};
    const int rc = tvr_attention_fwd(q.data_ptr<float>(), k.data_ptr<float>(), v.data_ptr<float>(),
                                     out.data_ptr<float>(), lse.data_ptr<float>(), B, H, L, S, E,
                                     qs, ks, vs, os, static_cast<float>(sc), is_causal ? 1 : 0,
                                     gemm_mode(), current_stream_handle());
    if (rc == TVR_OK) return result(out, lse);
    TORCH_CHECK(rc == TVR_ERR_UNSUPPORTED, "tvarant: ", tvr_last_error());
  }
  return result(composed_attention(query, key, value, attn_bias, is_causal, sc), none);
}

// ---- KV-cache decode pieces ----------------------------------------------
// Shapes stay fixed from step to step (the whole cache buffer, a position
// held in device memory), so a decode step can be captured once in a CUDA
// graph and replayed per token.

void check_pos(const at::Tensor& pos, const at::Tensor& like, const char* op) {
  TORCH_CHECK(pos.device() == like.device() && pos.scalar_type() == at::kLong && pos.numel() == 1,
              op, ": the position must be a one-element int64 tensor on the same device");
}

// cache[:, :, pos:pos+S] = src for cache [B, H, T, D] and src [B, H, S, D]
// (D contiguous in both), pos an int64 device scalar.
at::Tensor& kv_append_(at::Tensor& cache, const at::Tensor& src, const at::Tensor& pos) {
  check_fp32(cache, "kv_append_");
  check_fp32(src, "kv_append_");
  TORCH_CHECK(cache.dim() == 4 && src.dim() == 4 && cache.size(0) == src.size(0) &&
                  cache.size(1) == src.size(1) && cache.size(3) == src.size(3),
              "kv_append_: cache ", cache.sizes(), " and new entries ", src.sizes(),
              " must be [B, H, T, D] and [B, H, S, D]");
  TORCH_CHECK(cache.stride(3) == 1, "kv_append_: the cache's last dimension must be contiguous");
  check_pos(pos, cache, "kv_append_");
  c10::DeviceGuard guard(cache.device());
  at::Tensor s = src.stride(3) == 1 ? src : contiguous_copy(src);
  const int64_t cs[3] = {cache.stride(0), cache.stride(1), cache.stride(2)};
  const int64_t ss[3] = {s.stride(0), s.stride(1), s.stride(2)};
  TVR_TRY(tvr_kv_append(static_cast<float*>(cache.data_ptr()), static_cast<const float*>(s.data_ptr()),
                        s.size(0), s.size(1), s.size(2), s.size(3), cache.size(2), cs, ss,
                        static_cast<const int64_t*>(pos.data_ptr()), current_stream_handle()));
  return cache;
}

// Attention of q [B, H, Sq, D] to the first *key_len + key_len_add keys of
// k / v [B, H, T, D] (no mask; the fused TF32 kernel).
at::Tensor attention_keylen(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                            const at::Tensor& key_len, int64_t key_len_add, double scale) {
  for (const auto* t : {&q, &k, &v}) check_fp32(*t, "attention_keylen");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.sizes() == k.sizes() && q.size(0) == k.size(0) &&
                  q.size(1) == k.size(1) && q.size(3) == k.size(3),
              "attention_keylen: expected q [B, H, Sq, D] and k, v [B, H, T, D]");
  check_pos(key_len, q, "attention_keylen");
  TORCH_CHECK(gemm_mode() == TVR_GEMM_TF32,
              "attention_keylen runs the fused TF32 attention kernel: call "
              "torch.set_float32_matmul_precision('high')");
  c10::DeviceGuard guard(q.device());
  const int64_t B = q.size(0), H = q.size(1), L = q.size(2), E = q.size(3);
  at::Tensor out_buf = empty_device({B, L, H, E}, q.options());
  at::Tensor out = out_buf.permute({0, 2, 1, 3});
  auto st = [](const at::Tensor& t) {
    return std::array<int64_t, 3>{t.stride(0), t.stride(1), t.stride(2)};
  };
  const auto qs = st(q), ks = st(k), vs = st(v), os = st(out);
  TVR_TRY(tvr_attention_fwd_keylen(
      static_cast<const float*>(q.data_ptr()), static_cast<const float*>(k.data_ptr()),
      static_cast<const float*>(v.data_ptr()), static_cast<float*>(out.data_ptr()), B, H, L,
      k.size(2), E, qs.data(), ks.data(), vs.data(), os.data(), static_cast<float>(scale),
      static_cast<const int64_t*>(key_len.data_ptr()), static_cast<int>(key_len_add),
      TVR_GEMM_TF32, current_stream_handle()));
  return out;
}

// One decode step's attention with its cache append: k_new / v_new
// [B, H, 1, D] go into cache position *pos, and q [B, H, 1, D] attends to
// positions 0..*pos, in one launch (tvr_attention_decode_append).  Exactly
// kv_append_(k_cache, k_new, pos); kv_append_(v_cache, v_new, pos);
// attention_keylen(q, k_cache, v_cache, pos, 1, scale), which it runs when the
// fused kernel does not take the operands.
at::Tensor attention_decode_append(const at::Tensor& q, const at::Tensor& k_new,
                                   const at::Tensor& v_new, at::Tensor& k_cache,
                                   at::Tensor& v_cache, const at::Tensor& pos, double scale) {
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{
           &q, &k_new, &v_new, &k_cache, &v_cache}) {
    check_fp32(*t, "attention_decode_append");
  }
  TORCH_CHECK(q.dim() == 4 && q.size(2) == 1 && k_new.sizes() == q.sizes() &&
                  v_new.sizes() == q.sizes() && k_cache.dim() == 4 &&
                  v_cache.sizes() == k_cache.sizes() && k_cache.size(0) == q.size(0) &&
                  k_cache.size(1) == q.size(1) && k_cache.size(3) == q.size(3),
              "attention_decode_append: expected q, k_new, v_new [B, H, 1, D] and caches "
              "[B, H, T, D]");
  check_pos(pos, q, "attention_decode_append");
  c10::DeviceGuard guard(q.device());
  const bool inner = q.stride(3) == 1 && k_new.stride(3) == 1 && v_new.stride(3) == 1 &&
                     k_cache.stride(3) == 1 && v_cache.stride(3) == 1;
  if (inner) {
    const int64_t B = q.size(0), H = q.size(1), E = q.size(3);
    at::Tensor out_buf = empty_device({B, 1, H, E}, q.options());
    at::Tensor out = out_buf.permute({0, 2, 1, 3});
    auto st = [](const at::Tensor& t) {
      return std::array<int64_t, 3>{t.stride(0), t.stride(1), t.stride(2)};
    };
    const auto qs = st(q), kns = st(k_new), vns = st(v_new), kcs = st(k_cache),
               vcs = st(v_cache), os = st(out);
    const int rc = tvr_attention_decode_append(
        static_cast<const float*>(q.data_ptr()), static_cast<const float*>(k_new.data_ptr()),
        static_cast<const float*>(v_new.data_ptr()), static_cast<float*>(k_cache.data_ptr()),
        static_cast<float*>(v_cache.data_ptr()), static_cast<float*>(out.data_ptr()), B, H,
        k_cache.size(2), E, qs.data(), kns.data(), vns.data(), kcs.data(), vcs.data(), os.data(),
        static_cast<float>(scale), static_cast<const int64_t*>(pos.data_ptr()), gemm_mode(),
        current_stream_handle());
    if (rc == TVR_OK) return out;
    TORCH_CHECK(rc == TVR_ERR_UNSUPPORTED, "tvarant: ", tvr_last_error());
  }
  kv_append_(k_cache, k_new, pos);
  kv_append_(v_cache, v_new, pos);
  return attention_keylen(q, k_cache, v_cache, pos, 1, scale);
}

at::Tensor& counter_add_(at::Tensor& counter, int64_t delta) {
  TORCH_CHECK(is_device(counter) && counter.scalar_type() == at::kLong && counter.numel() == 1,
              "counter_add_: expected a one-element int64 tvarant tensor");
  c10::DeviceGuard guard(counter.device());
  TVR_TRY(tvr_counter_add(static_cast<int64_t*>(counter.data_ptr()), delta,
                          current_stream_handle()));
  return counter;
}

}  // namespace
}  // namespace tvarant::ops

TORCH_LIBRARY_FRAGMENT(tvarant, m) {
  m.def("kv_append_(Tensor(a!) cache, Tensor src, Tensor pos) -> Tensor(a!)");
  m.def("attention_keylen(Tensor q, Tensor k, Tensor v, Tensor key_len, int key_len_add, "
        "float scale) -> Tensor");
  m.def("counter_add_(Tensor(a!) counter, int delta) -> Tensor(a!)");
  m.def("attention_decode_append(Tensor q, Tensor k_new, Tensor v_new, Tensor(a!) k_cache, "
        "Tensor(b!) v_cache, Tensor pos, float scale) -> Tensor");
}

TORCH_LIBRARY_IMPL(tvarant, PrivateUse1, m) {
  m.impl("kv_append_", TORCH_FN(tvarant::ops::kv_append_));
  m.impl("attention_keylen", TORCH_FN(tvarant::ops::attention_keylen));
  m.impl("counter_add_", TORCH_FN(tvarant::ops::counter_add_));
  m.impl("attention_decode_append", TORCH_FN(tvarant::ops::attention_decode_append));
}

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("_scaled_dot_product_fused_attention_overrideable",
         TORCH_FN(tvarant::ops::sdpa_overrideable));
}

namespace at::native {
REGISTER_PRIVATEUSE1_DISPATCH(_fused_sdp_choice_stub, &tvarant::ops::fused_sdp_choice);
}  // namespace at::native

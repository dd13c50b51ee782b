// C-ABI entry points of the dense contractions: precision-mode resolution
// and the choice between the tcgen05 tensor-core kernel and the exact
// CUDA-core kernel.
//
// Replaces ops::gemm_bias_act (csrc/aten/AtenCommon.h:33-86) and the
// gemm_bias_act_kernel / bmm_kernel launches (csrc/runtime/CpuSimRuntime.cpp:166-188).
#include "internal.h"

#include <cstdlib>
#include <cstring>

#include "gemm_common.cuh"

namespace tvr {
namespace {

// TVR_GEMM_AUTO resolves from TVARANT_GEMM_MODE (tf32 | 3xtf32 | fp32),
// defaulting to the fp32-faithful 3xTF32 split.
int resolve_mode(int mode) {
  if (mode != TVR_GEMM_AUTO) return mode;
  const char* env = std::getenv("TVARANT_GEMM_MODE");
  if (env != nullptr) {
    if (std::strcmp(env, "tf32") == 0) return TVR_GEMM_TF32;
    if (std::strcmp(env, "3xtf32") == 0) return TVR_GEMM_3XTF32;
    if (std::strcmp(env, "fp32") == 0 || std::strcmp(env, "ieee") == 0) return TVR_GEMM_FP32;
  }
  return TVR_GEMM_3XTF32;
}

// Below this many multiply-adds a launch of the persistent tensor-core
// kernel costs more than it saves.
constexpr int64_t kSmallMacs = int64_t(1) << 21;

int run(const float* a, const float* b, const float* bias, float* c, int64_t m, int64_t n,
        int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int64_t batch, int64_t sa,
        int64_t sb, int64_t sc, float alpha, float beta, int act, bool trans_b, int mode,
        cudaStream_t stream, const EpiProg* prog = nullptr) {
  mode = resolve_mode(mode);
  // A pointwise program on the output: the tensor-core kernel applies it in
  // its epilogue; after the other kernels it runs as an in-place pass.
  auto then_prog = [&](int rc) {
    if (rc != TVR_OK || prog == nullptr) return rc;
    return epi_prog_inplace(*prog, c, ldc, m, n, stream);
  };
  if (mode != TVR_GEMM_TF32 && mode != TVR_GEMM_3XTF32 && mode != TVR_GEMM_FP32) {
    return fail(TVR_ERR_INVALID, "gemm: unknown precision mode %d", mode);
  }
  // At most 128 rows the weight read bounds the time.  One or two rows in
  // 3xTF32 mode: the fp32 FMA GEMV, as fast and closer to exact; otherwise
  // the weight-streaming tensor-core kernel, split over K across a CTA
  // cluster.  FP32 mode keeps the reference's sequential summation order.
  if (mode == TVR_GEMM_3XTF32 && batch == 1 &&
      gemm_skinny_applies(a, b, m, n, k, lda, ldb, trans_b)) {
    return then_prog(gemm_skinny(a, b, bias, c, m, n, k, lda, ldb, ldc, alpha, beta, act, stream));
  }
  if (mode != TVR_GEMM_FP32 && batch == 1 && gemm_ws_applies(a, b, m, n, k, lda, ldb, trans_b)) {
    // a residual add runs in the kernel's reduction epilogue (one launch less
    // in a decode step's attention projection and down projection)
    if (prog != nullptr && epi_is_residual_add(*prog)) {
      return gemm_ws(a, b, bias, c, m, n, k, lda, ldb, ldc, alpha, beta, act,
                     mode == TVR_GEMM_3XTF32, stream, prog->in[0], prog->ld[0]);
    }
    return then_prog(gemm_ws(a, b, bias, c, m, n, k, lda, ldb, ldc, alpha, beta, act,
                             mode == TVR_GEMM_3XTF32, stream));
  }
  const int64_t macs = batch * m * n * k;
  bool tensor = mode != TVR_GEMM_FP32 && macs > kSmallMacs;
  // Other skinny 3xTF32 problems (unaligned, batched): the exact CUDA-core
  // kernel reads each operand once and is as accurate.
  if (mode == TVR_GEMM_3XTF32 && m <= 16) tensor = false;
  if (tensor) {
    const int rc = gemm_tcgen05(a, b, bias, c, m, n, k, lda, ldb, ldc, batch, sa, sb, sc, alpha,
                                beta, act, trans_b, mode == TVR_GEMM_3XTF32, stream, prog);
    if (rc != TVR_ERR_UNSUPPORTED) return rc;
  }
  return then_prog(gemm_simt(a, b, bias, c, m, n, k, lda, ldb, ldc, batch, sa, sb, sc, alpha,
                             beta, act, trans_b, stream));
}

}  // namespace
}  // namespace tvr

using namespace tvr;

extern "C" {

int tvr_gemm_bias_act(const float* a, const float* b, const float* bias, float* c, int64_t m,
                      int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, float alpha,
                      float beta, int act, int trans_b, int mode, void* stream) {
  TVR_CHECK(m >= 0 && n >= 0 && k >= 0, "gemm: negative size (%lld, %lld, %lld)",
            (long long)m, (long long)n, (long long)k);
  TVR_CHECK(act >= 0 && act <= 2, "gemm: unknown activation %d", act);
  if (m == 0 || n == 0) return TVR_OK;
  TVR_CHECK(c != nullptr, "gemm: null output");
  TVR_CHECK(k == 0 || (a != nullptr && b != nullptr), "gemm: null operand");
  TVR_CHECK(lda >= k && ldc >= n, "gemm: leading dimension too small");
  TVR_CHECK(trans_b ? ldb >= k : ldb >= n, "gemm: leading dimension of B too small");
  return run(a, b, bias, c, m, n, k, lda, ldb, ldc, 1, 0, 0, 0, alpha, beta, act, trans_b != 0,
             mode, as_stream(stream));
}

int tvr_gemm_pointwise(const float* a, const float* b, const float* bias, float* c, int64_t m,
                       int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, float alpha,
                       float beta, int act, int trans_b, int mode, const tvr_pw_node* nodes,
                       int n_nodes, int n_inputs, int gemm_input, const float* const* inputs,
                       const int64_t* input_ld, void* stream) {
  TVR_CHECK(m >= 0 && n >= 0 && k >= 0, "gemm_pointwise: negative size (%lld, %lld, %lld)",
            (long long)m, (long long)n, (long long)k);
  TVR_CHECK(act >= 0 && act <= 2, "gemm_pointwise: unknown activation %d", act);
  if (m == 0 || n == 0) return TVR_OK;
  TVR_CHECK(c != nullptr, "gemm_pointwise: null output");
  TVR_CHECK(k == 0 || (a != nullptr && b != nullptr), "gemm_pointwise: null operand");
  TVR_CHECK(lda >= k && ldc >= n, "gemm_pointwise: leading dimension too small");
  TVR_CHECK(trans_b ? ldb >= k : ldb >= n, "gemm_pointwise: leading dimension of B too small");
  EpiProg prog;
  const int rc = build_epi_prog(nodes, n_nodes, n_inputs, gemm_input, inputs, input_ld, c, m, n,
                                ldc, &prog);
  if (rc != TVR_OK) return rc;
  return run(a, b, bias, c, m, n, k, lda, ldb, ldc, 1, 0, 0, 0, alpha, beta, act, trans_b != 0,
             mode, as_stream(stream), &prog);
}

int tvr_gemm_swiglu(const float* x, const float* w_gate, const float* w_up, float* out,
                    int64_t m, int64_t n, int64_t k, int64_t ldx, int64_t ldw_gate,
                    int64_t ldw_up, int64_t ldo, int mode, void* stream) {
  TVR_CHECK(m >= 0 && n >= 0 && k >= 0, "gemm_swiglu: negative size (%lld, %lld, %lld)",
            (long long)m, (long long)n, (long long)k);
  if (m == 0 || n == 0) return TVR_OK;
  TVR_CHECK(out != nullptr, "gemm_swiglu: null output");
  TVR_CHECK(k == 0 || (x != nullptr && w_gate != nullptr && w_up != nullptr),
            "gemm_swiglu: null operand");
  TVR_CHECK(ldx >= k && ldw_gate >= k && ldw_up >= k && ldo >= n,
            "gemm_swiglu: leading dimension too small");
  mode = resolve_mode(mode);
  TVR_CHECK(mode == TVR_GEMM_TF32 || mode == TVR_GEMM_3XTF32 || mode == TVR_GEMM_FP32,
            "gemm_swiglu: unknown precision mode %d", mode);
  cudaStream_t s = as_stream(stream);
  if (mode == TVR_GEMM_TF32 && m > 128 && k > 0) {
    const int rc = gemm_tcgen05_swiglu(x, w_gate, w_up, out, m, n, k, ldx, ldw_gate, ldw_up, ldo, s);
    if (rc != TVR_ERR_UNSUPPORTED) return rc;
  }
  // Composition: gate (with SiLU) and up into scratch, then their product
  // into out (through a third scratch block when out has a row stride).
  const bool dense_out = ldo == n;
  Scratch scratch;
  const size_t mn = static_cast<size_t>(m * n);
  int rc = scratch.alloc((dense_out ? 2 : 3) * mn * sizeof(float), current_device(), s);
  if (rc != TVR_OK) return rc;
  float* g = static_cast<float*>(scratch.ptr);
  float* u = g + mn;
  if ((rc = tvr_gemm_bias_act(x, w_gate, nullptr, g, m, n, k, ldx, ldw_gate, n, 1.f, 0.f,
                              TVR_ACT_SILU, 1, mode, stream)) != TVR_OK)
    return rc;
  if ((rc = tvr_gemm_bias_act(x, w_up, nullptr, u, m, n, k, ldx, ldw_up, n, 1.f, 0.f,
                              TVR_ACT_NONE, 1, mode, stream)) != TVR_OK)
    return rc;
  const int64_t sizes[2] = {m, n};
  const int64_t dense[2] = {n, 1};
  const int64_t strided[2] = {ldo, 1};
  float* prod = dense_out ? out : u + mn;
  if ((rc = tvr_binary(TVR_BINARY_MUL, g, u, prod, 2, sizes, dense, dense, 1.f, stream)) != TVR_OK)
    return rc;
  if (dense_out) return TVR_OK;
  return tvr_strided_copy(out, prod, 4, 2, sizes, strided, dense, stream);
}

int tvr_bmm(const float* a, const float* b, float* c, int64_t batch, int64_t m, int64_t n,
            int64_t k, int64_t stride_a, int64_t stride_b, int64_t stride_c, int trans_b,
            int mode, void* stream) {
  TVR_CHECK(batch >= 0 && m >= 0 && n >= 0 && k >= 0, "bmm: negative size");
  if (batch == 0 || m == 0 || n == 0) return TVR_OK;
  TVR_CHECK(c != nullptr, "bmm: null output");
  TVR_CHECK(k == 0 || (a != nullptr && b != nullptr), "bmm: null operand");
  const int64_t lda = k, ldb = trans_b ? k : n, ldc = n;
  return run(a, b, nullptr, c, m, n, k, lda, ldb, ldc, batch, stride_a, stride_b, stride_c, 1.f,
             0.f, 0, trans_b != 0, mode, as_stream(stream));
}

}  // extern "C"

// C entry points over the reference simulator's own kernels
// (samthakur587/Tvarant csrc/kernels/host/HostKernels.cpp and csrc/jit/Jit.cpp,
// compiled from the reference checkout by oracle/build.py into
// oracle/_ref/libtvr_ref.so).  Test infrastructure only: used to pin the C
// restatement in oracle/oracle.c and as the timed CPU baseline.
#include <cstdint>
#include <exception>
#include <vector>

#include "kernels/host/HostKernels.h"
#include "jit/Jit.h"

#define REF_API extern "C" __attribute__((visibility("default")))

REF_API void ref_gemm_bias_act(const float* a, const float* b, const float* bias, float* c,
                               int64_t m, int64_t n, int64_t k, float alpha, float beta,
                               int act, int trans_b) {
  tvarant::host::gemm_bias_act_f32(a, b, bias, c, m, n, k, alpha, beta, act, trans_b != 0);
}

REF_API void ref_bmm(const float* a, const float* b, float* c, int64_t batch, int64_t m,
                     int64_t n, int64_t k, int trans_b) {
  tvarant::host::bmm_f32(a, b, c, batch, m, n, k, trans_b != 0);
}

REF_API void ref_softmax(const float* in, float* out, int64_t outer, int64_t dim, int64_t inner) {
  tvarant::host::softmax_f32(in, out, outer, dim, inner);
}

REF_API void ref_layer_norm(const float* in, const float* w, const float* b, float* out,
                            float* mean, float* rstd, int64_t rows, int64_t n, float eps) {
  tvarant::host::layer_norm_f32(in, w, b, out, mean, rstd, rows, n, eps);
}

// The reference narrows indices to int32 before the kernel (LlmOps.cpp:238).
REF_API void ref_embedding(const float* w, const int64_t* idx, float* out, int64_t n_idx,
                           int64_t dim, int64_t vocab) {
  std::vector<int32_t> idx32(static_cast<size_t>(n_idx));
  for (int64_t i = 0; i < n_idx; ++i) idx32[static_cast<size_t>(i)] = static_cast<int32_t>(idx[i]);
  tvarant::host::embedding_f32(w, idx32.data(), out, n_idx, dim, vocab);
}

REF_API void ref_unary(int op, const float* x, float* y, int64_t n, float s) {
  using namespace tvarant::host;
  switch (op) {
    case 0: relu_f32(x, y, n); break;
    case 1: silu_f32(x, y, n); break;
    case 2: neg_f32(x, y, n); break;
    case 3: abs_f32(x, y, n); break;
    case 4: exp_f32(x, y, n); break;
    case 5: exp2_f32(x, y, n); break;
    case 6: sqrt_f32(x, y, n); break;
    case 7: rsqrt_f32(x, y, n); break;
    case 8: scale_f32(x, y, n, s); break;
    case 9: add_scalar_f32(x, y, n, s); break;
    default: copy_f32(y, x, n); break;
  }
}

REF_API void ref_binary(int op, const float* a, const float* b, float* out, int64_t n,
                        float alpha) {
  if (op == 0) tvarant::host::add_f32(a, b, out, n, alpha);
  else tvarant::host::mul_f32(a, b, out, n);
}

REF_API void ref_fill(float* out, float v, int64_t n) { tvarant::host::fill_f32(out, v, n); }

struct RefNode {
  int32_t op, a, b, input_id;
  float alpha, c;
};

// Reference interpreter (opcodes 0-8 only).  Returns 0, or -1 when the
// reference rejects the program.
REF_API int ref_pointwise(const RefNode* nodes, int n_nodes, int n_inputs,
                          const float* const* inputs, float* out, int64_t n) {
  tvarant::jit::PointwiseProgram prog;
  prog.n_inputs = n_inputs;
  prog.nodes.resize(static_cast<size_t>(n_nodes));
  for (int i = 0; i < n_nodes; ++i) {
    auto& nd = prog.nodes[static_cast<size_t>(i)];
    nd.op = static_cast<tvarant::jit::PwOp>(nodes[i].op);
    nd.a = nodes[i].a;
    nd.b = nodes[i].b;
    nd.input_id = nodes[i].input_id;
    nd.alpha = nodes[i].alpha;
    nd.c = nodes[i].c;
  }
  try {
    tvarant::jit::run_pointwise_host(prog, inputs, out, n);
  } catch (const std::exception&) {
    return -1;
  }
  return 0;
}

/*
 * oracle.c — CPU restatement of the reference simulator's kernels
 * (samthakur587/Tvarant, csrc/kernels/host/HostKernels.cpp and
 * csrc/jit/Jit.cpp), written in plain C.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels
 * of tvarant_b200: only tests/, __graft_entry__.smoke() and the CPU-baseline
 * leg of bench.py load it.  Nothing in the product path calls it.
 *
 * Built with -ffp-contract=off so every a*b+c is two roundings, as in the
 * reference (compiled for baseline x86-64, which has no FMA instructions).
 * Each function cites the reference lines it restates.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define TVO_API __attribute__((visibility("default")))

/* act 0 none, 1 relu, 2 silu — csrc/jit/Jit.h:48-56 */
static float tvo_act(float x, int act) {
  if (act == 1) return x > 0.f ? x : 0.f;
  if (act == 2) return x / (1.f + expf(-x));
  return x;
}

/* C = act(alpha * A*op(B) + beta * prev) — HostKernels.cpp:100-144.
 * The reference tiles i, j and p by 32, but each acc[i][j] still sums
 * p = 0..k-1 in increasing order, so a plain loop gives the same bits. */
TVO_API void tvo_gemm_bias_act(const float* a, const float* b, const float* bias, float* c,
                               int64_t m, int64_t n, int64_t k, float alpha, float beta,
                               int act, int trans_b) {
  for (int64_t i = 0; i < m; ++i) {
    for (int64_t j = 0; j < n; ++j) {
      float acc = 0.f;
      for (int64_t p = 0; p < k; ++p) {
        const float bv = trans_b ? b[j * k + p] : b[p * n + j];
        acc += a[i * k + p] * bv;
      }
      float prev = 0.f;
      if (bias != NULL) prev = bias[j];
      else if (beta != 0.f) prev = c[i * n + j];
      c[i * n + j] = tvo_act(alpha * acc + beta * prev, act);
    }
  }
}

/* Rows [row0, row1) of the GEMM only (rows are independent), for sampled
 * checks of large problems. */
TVO_API void tvo_gemm_rows(const float* a, const float* b, const float* bias, float* c,
                           int64_t row0, int64_t row1, int64_t n, int64_t k, float alpha,
                           float beta, int act, int trans_b) {
  tvo_gemm_bias_act(a + row0 * k, b, bias, c + row0 * n, row1 - row0, n, k, alpha, beta, act,
                    trans_b);
}

/* Batched — HostKernels.cpp:146-172. */
TVO_API void tvo_bmm(const float* a, const float* b, float* c, int64_t batch, int64_t m,
                     int64_t n, int64_t k, int trans_b) {
  for (int64_t bi = 0; bi < batch; ++bi) {
    tvo_gemm_bias_act(a + bi * m * k, b + bi * (trans_b ? n * k : k * n), NULL, c + bi * m * n,
                      m, n, k, 1.f, 0.f, 0, trans_b);
  }
}

/* Softmax over dim of (outer, dim, inner) — HostKernels.cpp:174-198. */
TVO_API void tvo_softmax(const float* in, float* out, int64_t outer, int64_t dim,
                         int64_t inner) {
  for (int64_t o = 0; o < outer; ++o) {
    for (int64_t i = 0; i < inner; ++i) {
      float mx = in[(o * dim) * inner + i];
      for (int64_t d = 1; d < dim; ++d) {
        const float v = in[(o * dim + d) * inner + i];
        if (mx < v) mx = v; /* std::max(m, v) */
      }
      float sum = 0.f;
      for (int64_t d = 0; d < dim; ++d) {
        const float e = expf(in[(o * dim + d) * inner + i] - mx);
        out[(o * dim + d) * inner + i] = e;
        sum += e;
      }
      const float inv = 1.f / sum;
      for (int64_t d = 0; d < dim; ++d) out[(o * dim + d) * inner + i] *= inv;
    }
  }
}

/* Layer norm over rows — HostKernels.cpp:200-242. */
TVO_API void tvo_layer_norm(const float* in, const float* w, const float* bias, float* out,
                            float* mean, float* rstd, int64_t rows, int64_t n, float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* x = in + r * n;
    float mu = 0.f;
    for (int64_t j = 0; j < n; ++j) mu += x[j];
    mu /= (float)n;
    float var = 0.f;
    for (int64_t j = 0; j < n; ++j) {
      const float d = x[j] - mu;
      var += d * d;
    }
    var /= (float)n;
    const float rs = 1.f / sqrtf(var + eps);
    if (mean) mean[r] = mu;
    if (rstd) rstd[r] = rs;
    float* y = out + r * n;
    for (int64_t j = 0; j < n; ++j) {
      float v = (x[j] - mu) * rs;
      if (w) v *= w[j];
      if (bias) v += bias[j];
      y[j] = v;
    }
  }
}

/* Row gather, index outside [0, vocab) -> zeros — HostKernels.cpp:244-260.
 * Indices are int64 here; the reference first narrows them to int32
 * (csrc/aten/LlmOps.cpp:238), which only matters beyond the int32 range. */
TVO_API void tvo_embedding(const float* w, const int64_t* idx, float* out, int64_t n_idx,
                           int64_t dim, int64_t vocab) {
  for (int64_t i = 0; i < n_idx; ++i) {
    const int64_t id = idx[i];
    float* dst = out + i * dim;
    if (id < 0 || id >= vocab) {
      memset(dst, 0, (size_t)dim * sizeof(float));
    } else {
      memcpy(dst, w + id * dim, (size_t)dim * sizeof(float));
    }
  }
}

/* Unary maps — HostKernels.cpp:17-98; op ids as TVR_UNARY_* in tvarant.h. */
TVO_API void tvo_unary(int op, const float* x, float* y, int64_t n, float s) {
  for (int64_t i = 0; i < n; ++i) {
    const float v = x[i];
    float r;
    switch (op) {
      case 0: r = v > 0.f ? v : 0.f; break;         /* relu  :39-43 */
      case 1: r = v / (1.f + expf(-v)); break;      /* silu  :45-50 */
      case 2: r = -v; break;                        /* neg   :64-68 */
      case 3: r = fabsf(v); break;                  /* abs   :70-74 */
      case 4: r = expf(v); break;                   /* exp   :76-80 */
      case 5: r = exp2f(v); break;                  /* exp2  :82-86 */
      case 6: r = sqrtf(v); break;                  /* sqrt  :88-92 */
      case 7: r = 1.f / sqrtf(v); break;            /* rsqrt :94-98 */
      case 8: r = v * s; break;                     /* scale :52-56 */
      case 9: r = v + s; break;                     /* add_scalar :58-62 */
      case 10: r = 1.f / (1.f + expf(-v)); break;   /* sigmoid (Jit.cpp:335-338) */
      default: r = v; break;                        /* copy  :23-25 */
    }
    y[i] = r;
  }
}

/* a + alpha*b, a*b on pre-broadcast contiguous buffers — HostKernels.cpp:27-37. */
TVO_API void tvo_binary(int op, const float* a, const float* b, float* out, int64_t n,
                        float alpha) {
  for (int64_t i = 0; i < n; ++i) out[i] = op == 0 ? a[i] + alpha * b[i] : a[i] * b[i];
}

/* Pointwise SSA interpreter — csrc/jit/Jit.cpp:34-87, with the appended
 * opcodes 9 Sub (a - alpha*b, evaluated as a + (-alpha)*b like the eager
 * sub, ExtendedOps.cpp:261-264), 10 Exp, 11 Abs.  Node layout matches
 * tvr_pw_node: op, a, b, input_id (int32), alpha, c (float).  Returns 0, or
 * -1 for an invalid program. */
typedef struct {
  int32_t op, a, b, input_id;
  float alpha, c;
} tvo_pw_node;

TVO_API int tvo_pointwise(const tvo_pw_node* nodes, int n_nodes, int n_inputs,
                          const float* const* inputs, float* out, int64_t n, float* regs) {
  if (n_nodes <= 0) return -1;
  for (int64_t i = 0; i < n; ++i) {
    for (int v = 0; v < n_nodes; ++v) {
      const tvo_pw_node* nd = &nodes[v];
      float r;
      switch (nd->op) {
        case 0:
          if (nd->input_id < 0 || nd->input_id >= n_inputs) return -1;
          r = inputs[nd->input_id][i];
          break;
        case 1: r = nd->c; break;
        case 2: r = regs[nd->a] + nd->alpha * regs[nd->b]; break;
        case 3: r = regs[nd->a] * regs[nd->b]; break;
        case 4: r = regs[nd->a] > 0.f ? regs[nd->a] : 0.f; break;
        case 5: r = regs[nd->a] / (1.f + expf(-regs[nd->a])); break;
        case 6: r = -regs[nd->a]; break;
        case 7: r = nd->alpha * regs[nd->a]; break;
        case 8: r = 1.f / (1.f + expf(-regs[nd->a])); break;
        case 9: r = regs[nd->a] + (-nd->alpha) * regs[nd->b]; break;
        case 10: r = expf(regs[nd->a]); break;
        case 11: r = fabsf(regs[nd->a]); break;
        default: return -1;
      }
      regs[v] = r;
    }
    out[i] = regs[n_nodes - 1];
  }
  return 0;
}

// Pointwise programs on a GEMM's output (tvr_gemm_pointwise): building the
// epilogue program from tvr_pw_node SSA nodes — as checked SSA for the pass
// below and as two-slot stack code for the tensor-core GEMM's epilogue
// (gemm_tc.cu) — and the in-place pass that applies it when the GEMM kernel
// cannot (split-K, CUDA-core or weight-streaming GEMMs, or a program that
// needs more than two stack slots or two extra inputs).  Both routes apply
// the same operations in the same order, written as the pointwise JIT emits
// them.
#include "internal.h"

#include <algorithm>

#include "epilogue_prog.cuh"
#include "gemm_common.cuh"

namespace tvr {
namespace {

constexpr int kThreads = 256;

// c = program(c, extras) over [m, n]; each thread takes four consecutive
// columns of one row.
__global__ void __launch_bounds__(kThreads) epi_prog_kernel(const __grid_constant__ EpiProg g,
                                                            float* __restrict__ c, int64_t ldc,
                                                            int m, int n, int c_vec) {
  const int64_t groups_per_row = (n + 3) / 4;
  const int64_t total = static_cast<int64_t>(m) * groups_per_row;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += stride) {
    const int64_t row = t / groups_per_row;
    const int col = static_cast<int>(t - row * groups_per_row) * 4;
    float* dst = c + row * ldc + col;
    const bool full4 = c_vec && col + 3 < n;
    float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
    if (full4) {
      y = *reinterpret_cast<const float4*>(dst);
    } else {
      y.x = dst[0];
      if (col + 1 < n) y.y = dst[1];
      if (col + 2 < n) y.z = dst[2];
      if (col + 3 < n) y.w = dst[3];
    }
    const float4 e0 = g.n_extra > 0 ? epi_load4(g, 0, row, col, m, n) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 e1 = g.n_extra > 1 ? epi_load4(g, 1, row, col, m, n) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 r = epi_eval4<EPI_MAX_NODES>(g, y, e0, e1);
    if (full4) {
      *reinterpret_cast<float4*>(dst) = r;
    } else {
      dst[0] = r.x;
      if (col + 1 < n) dst[1] = r.y;
      if (col + 2 < n) dst[2] = r.z;
      if (col + 3 < n) dst[3] = r.w;
    }
  }
}

// SSA program -> stack code over two slots (EpiProg::sop).  A node used
// twice is evaluated twice (programs are small and every operation is
// elementwise).  Operands of a binary node are evaluated in the order that
// needs fewer slots: the first-evaluated one sits in slot 1.
struct StackBuilder {
  const tvr_pw_node* nodes;
  const int* slot;  // input id -> extra slot (-1: the GEMM result)
  EpiProg* g;
  bool ok = true;

  static bool unary(int op) {
    return op == kEpiRelu || op == kEpiSilu || op == kEpiNeg || op == kEpiScale ||
           op == kEpiSigmoid || op == kEpiExp || op == kEpiAbs;
  }

  int need(int v) const {
    const tvr_pw_node& nd = nodes[v];
    if (nd.op == kEpiLoad || nd.op == kEpiConst) return 1;
    if (unary(nd.op)) return need(nd.a);
    const int na = need(nd.a), nb = need(nd.b);
    return std::min(std::max(na, 1 + nb), std::max(nb, 1 + na));
  }

  void put(int8_t op, int8_t rev, float val) {
    if (g->n_ops >= EPI_MAX_STACK_OPS) {
      ok = false;
      return;
    }
    g->sop[g->n_ops] = op;
    g->rev[g->n_ops] = rev;
    g->sval[g->n_ops] = val;
    ++g->n_ops;
  }

  void emit(int v) {
    if (!ok) return;
    const tvr_pw_node& nd = nodes[v];
    switch (nd.op) {
      case kEpiLoad: {
        const int e = slot[nd.input_id];
        if (e >= EPI_STACK_EXTRA) {
          ok = false;
          return;
        }
        put(e < 0 ? kStPushY : kStPushX, 0, 0.f);
        return;
      }
      case kEpiConst: put(kStPushC, 0, nd.c); return;
      case kEpiRelu: emit(nd.a); put(kStRelu, 0, 0.f); return;
      case kEpiSilu: emit(nd.a); put(kStSilu, 0, 0.f); return;
      case kEpiNeg: emit(nd.a); put(kStNeg, 0, 0.f); return;
      case kEpiScale: emit(nd.a); put(kStScale, 0, nd.alpha); return;
      case kEpiSigmoid: emit(nd.a); put(kStSigmoid, 0, 0.f); return;
      case kEpiExp: emit(nd.a); put(kStExp, 0, 0.f); return;
      case kEpiAbs: emit(nd.a); put(kStAbs, 0, 0.f); return;
      default: break;
    }
    const int na = need(nd.a), nb = need(nd.b);
    const bool swapped = std::max(nb, 1 + na) < std::max(na, 1 + nb);
    if (swapped) {
      emit(nd.b);
      emit(nd.a);
    } else {
      emit(nd.a);
      emit(nd.b);
    }
    const int8_t op = nd.op == kEpiAdd ? kStAdd : (nd.op == kEpiSub ? kStSub : kStMul);
    put(op, swapped ? 1 : 0, nd.alpha);
  }
};

bool overlaps(const float* p, int64_t p_elems, const float* q, int64_t q_elems) {
  const auto a0 = reinterpret_cast<uintptr_t>(p), a1 = a0 + 4 * static_cast<uintptr_t>(p_elems);
  const auto b0 = reinterpret_cast<uintptr_t>(q), b1 = b0 + 4 * static_cast<uintptr_t>(q_elems);
  return a0 < b1 && b0 < a1;
}

}  // namespace

int epi_prog_inplace(const EpiProg& prog, float* c, int64_t ldc, int64_t m, int64_t n,
                     cudaStream_t stream) {
  if (m == 0 || n == 0 || prog.n_nodes == 0) return TVR_OK;
  const int dev = current_device();
  const int64_t groups = m * ((n + 3) / 4);
  const int c_vec = (reinterpret_cast<uintptr_t>(c) % 16 == 0 && ldc % 4 == 0) ? 1 : 0;
  epi_prog_kernel<<<elementwise_grid(groups, kThreads, dev), kThreads, 0, stream>>>(
      prog, c, ldc, static_cast<int>(m), static_cast<int>(n), c_vec);
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

int build_epi_prog(const tvr_pw_node* nodes, int n_nodes, int n_inputs, int gemm_input,
                   const float* const* inputs, const int64_t* input_ld, const float* c,
                   int64_t m, int64_t n, int64_t ldc, EpiProg* out) {
  TVR_CHECK(nodes != nullptr && n_nodes > 0, "gemm_pointwise: empty program");
  TVR_CHECK(n_nodes <= EPI_MAX_NODES, "gemm_pointwise: %d nodes (at most %d)", n_nodes,
            EPI_MAX_NODES);
  TVR_CHECK(n_inputs >= 1 && n_inputs <= EPI_MAX_EXTRA + 1,
            "gemm_pointwise: %d inputs (the GEMM result and at most %d more)", n_inputs,
            EPI_MAX_EXTRA);
  TVR_CHECK(gemm_input >= 0 && gemm_input < n_inputs, "gemm_pointwise: gemm_input %d out of range",
            gemm_input);
  TVR_CHECK(n_inputs == 1 || (inputs != nullptr && input_ld != nullptr),
            "gemm_pointwise: null input arrays");
  EpiProg g;
  memset(&g, 0, sizeof(g));
  g.n_nodes = n_nodes;
  // input id -> extra slot (-1: the GEMM result)
  int slot[EPI_MAX_EXTRA + 1];
  int e = 0;
  for (int i = 0; i < n_inputs; ++i) {
    if (i == gemm_input) {
      slot[i] = -1;
      continue;
    }
    TVR_CHECK(inputs[i] != nullptr, "gemm_pointwise: null input %d", i);
    const int64_t ld = input_ld[i];
    TVR_CHECK(ld == 0 || ld >= n, "gemm_pointwise: input %d row stride %lld (0 or >= %lld)", i,
              (long long)ld, (long long)n);
    const int64_t extent = ld == 0 ? n : (m - 1) * ld + n;
    TVR_CHECK(!overlaps(inputs[i], extent, c, (m - 1) * ldc + n),
              "gemm_pointwise: input %d overlaps the output", i);
    g.in[e] = inputs[i];
    g.ld[e] = ld;
    g.vec[e] = (reinterpret_cast<uintptr_t>(inputs[i]) % 16 == 0 && ld % 4 == 0) ? 1 : 0;
    slot[i] = e++;
  }
  g.n_extra = e;
  for (int v = 0; v < n_nodes; ++v) {
    const tvr_pw_node& nd = nodes[v];
    const bool unary = nd.op == kEpiRelu || nd.op == kEpiSilu || nd.op == kEpiNeg ||
                       nd.op == kEpiScale || nd.op == kEpiSigmoid || nd.op == kEpiExp ||
                       nd.op == kEpiAbs;
    const bool binary = nd.op == kEpiAdd || nd.op == kEpiMul || nd.op == kEpiSub;
    g.op[v] = static_cast<int8_t>(nd.op);
    g.a[v] = -1;
    g.b[v] = -1;
    g.src[v] = -1;
    g.alpha[v] = nd.alpha;
    g.c[v] = nd.c;
    if (nd.op == kEpiLoad) {
      TVR_CHECK(nd.input_id >= 0 && nd.input_id < n_inputs,
                "gemm_pointwise: node %d loads input %d of %d", v, nd.input_id, n_inputs);
      g.src[v] = static_cast<int8_t>(slot[nd.input_id]);
    } else if (nd.op == kEpiConst) {
    } else if (unary || binary) {
      TVR_CHECK(nd.a >= 0 && nd.a < v, "gemm_pointwise: node %d operand a=%d is not an earlier node",
                v, nd.a);
      g.a[v] = static_cast<int8_t>(nd.a);
      if (binary) {
        TVR_CHECK(nd.b >= 0 && nd.b < v,
                  "gemm_pointwise: node %d operand b=%d is not an earlier node", v, nd.b);
        g.b[v] = static_cast<int8_t>(nd.b);
      }
    } else {
      return fail(TVR_ERR_INVALID, "gemm_pointwise: unknown pointwise op %d", nd.op);
    }
  }
  // the stack form the tensor-core epilogue runs (n_ops == 0 when the
  // program needs more than two slots or more than one extra input)
  StackBuilder sb{nodes, slot, &g};
  g.n_ops = 0;
  if (sb.need(n_nodes - 1) <= 2) sb.emit(n_nodes - 1);
  if (!sb.ok) g.n_ops = 0;
  *out = g;
  return TVR_OK;
}

}  // namespace tvr

extern "C" int tvr_gemm_pointwise_plan(const tvr_pw_node* nodes, int n_nodes, int n_inputs,
                                       int gemm_input, int* n_ops, int8_t* ops, int8_t* rev,
                                       float* vals, int cap) {
  using namespace tvr;
  TVR_CHECK(n_ops != nullptr, "gemm_pointwise_plan: null output count");
  TVR_CHECK(cap >= 0 && (cap == 0 || (ops && rev && vals)), "gemm_pointwise_plan: bad buffers");
  // the checks and the translation of build_epi_prog, with stand-in input
  // addresses (one row each, far from the stand-in output)
  static const float stand_in[2][4] = {};
  const float* inputs[EPI_MAX_EXTRA + 1] = {stand_in[0], stand_in[1], stand_in[1]};
  const int64_t lds[EPI_MAX_EXTRA + 1] = {0, 0, 0};
  static float out_stand_in[4];
  TVR_CHECK(n_inputs >= 1 && n_inputs <= EPI_MAX_EXTRA + 1,
            "gemm_pointwise_plan: %d inputs (the GEMM result and at most %d more)", n_inputs,
            EPI_MAX_EXTRA);
  EpiProg g;
  const int rc = build_epi_prog(nodes, n_nodes, n_inputs, gemm_input, inputs, lds, out_stand_in,
                                1, 4, 4, &g);
  if (rc != TVR_OK) return rc;
  *n_ops = g.n_ops;
  for (int i = 0; i < g.n_ops && i < cap; ++i) {
    ops[i] = g.sop[i];
    rev[i] = g.rev[i];
    vals[i] = g.sval[i];
  }
  return TVR_OK;
}

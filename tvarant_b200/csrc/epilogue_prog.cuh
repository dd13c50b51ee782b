// Pointwise programs evaluated in a GEMM epilogue (tvr_gemm_pointwise).
//
// The program is a tvr_pointwise SSA program (tvr_pw_node, opcodes of the
// reference's pointwise fuser, csrc/jit/Jit.h:11-21, plus Sub / Exp / Abs)
// one of whose inputs is the GEMM's result.  It is interpreted instead of
// compiled — one kernel serves every program, with no NVRTC compile — in
// two forms:
//   * stack code (EpiProg::sop) in the tensor-core GEMM's epilogue: each
//     operation is dispatched once for 16 values of a lane, which keeps the
//     epilogue of a 128 x 256 tile (~28 us for a six-operation chain) shorter
//     than the main loop of the next tile (~53 us at K = 4096), so it hides
//     behind the MMAs;
//   * the SSA nodes themselves (epi_eval4) in the in-place pass
//     (gemm_epilogue.cu), for what the stack form does not cover.
// Every operation is written as the pointwise JIT emits it
// (csrc/pointwise_jit.cu, codegen), with no contraction into FMAs.
//
// Node values live in registers: operands are read from earlier nodes by
// (unrolled) compile-time index or compare-and-select, never through an
// indexed array, which would put them in local memory.
#pragma once

#include <cstdint>

namespace tvr {

constexpr int EPI_MAX_NODES = 12;
constexpr int EPI_MAX_EXTRA = 2;

// The tensor-core GEMM runs a program in its epilogue as stack code of at
// most EPI_MAX_STACK_OPS operations over two stack slots and at most one
// extra input: each operation is applied to all 32 values a lane holds (8
// rows x 4 columns of a 32 x 32 chunk), so the dispatch of an operation is
// paid once per 32 values and the 32 are independent (instruction-level
// parallelism).  Programs that need a deeper stack or two extra inputs run
// as a pass over the GEMM's output (epi_prog_kernel) instead.
constexpr int EPI_MAX_STACK_OPS = 16;
constexpr int EPI_STACK_EXTRA = 1;

// Stack operations.  Pushes move slot 0 into slot 1 first; unary
// operations rewrite slot 0; binary operations combine the two slots into
// slot 0 — f(slot 1, slot 0), or f(slot 0, slot 1) when the operation's
// `rev` flag is set (the second operand was evaluated first).
enum EpiStackOp : int8_t {
  kStPushY = 0,  // the GEMM result (after bias and activation)
  kStPushX = 1,  // the extra input
  kStPushC = 2,  // constant sval
  kStAdd = 3,    // a + sval * b
  kStSub = 4,    // a - sval * b
  kStMul = 5,
  kStRelu = 6,
  kStSilu = 7,
  kStNeg = 8,
  kStScale = 9,  // sval * a
  kStSigmoid = 10,
  kStExp = 11,
  kStAbs = 12,
};

struct EpiProg {
  int n_nodes;  // 0: no program
  int n_extra;  // extra inputs (besides the GEMM result)
  int8_t op[EPI_MAX_NODES];
  int8_t a[EPI_MAX_NODES];
  int8_t b[EPI_MAX_NODES];
  int8_t src[EPI_MAX_NODES];  // Load: -1 the GEMM result, e >= 0 extra input e
  float alpha[EPI_MAX_NODES];
  float c[EPI_MAX_NODES];
  const float* in[EPI_MAX_EXTRA];
  int64_t ld[EPI_MAX_EXTRA];  // row stride; 0: one row [n] broadcast over all rows
  int vec[EPI_MAX_EXTRA];     // 1: 16-byte loads are aligned (base and row stride)
  // the same program as stack code (n_ops == 0: not expressible in two slots)
  int n_ops;
  int8_t sop[EPI_MAX_STACK_OPS];
  int8_t rev[EPI_MAX_STACK_OPS];
  float sval[EPI_MAX_STACK_OPS];
};

#ifdef __CUDACC__

// Pointwise opcodes (tvr_pw_node.op).
enum EpiOp {
  kEpiLoad = 0,
  kEpiConst = 1,
  kEpiAdd = 2,
  kEpiMul = 3,
  kEpiRelu = 4,
  kEpiSilu = 5,
  kEpiNeg = 6,
  kEpiScale = 7,
  kEpiSigmoid = 8,
  kEpiSub = 9,
  kEpiExp = 10,
  kEpiAbs = 11,
};

// True when the program is the residual add y + r (Load y, Load r, Add with
// alpha 1, in either operand order), r being extra input 0 as a full
// row-major matrix (row stride in[0] / ld[0], not a broadcast row).  The GEMM
// kernels add r in their own epilogues then; in IEEE arithmetic y + 1 * r is
// y + r in either order, so the result is bit-identical to the program.
inline bool epi_is_residual_add(const EpiProg& g) {
  return g.n_nodes == 3 && g.n_extra == 1 && g.op[0] == kEpiLoad && g.op[1] == kEpiLoad &&
         g.op[2] == kEpiAdd && g.alpha[2] == 1.f &&
         ((g.src[0] == -1 && g.src[1] == 0) || (g.src[0] == 0 && g.src[1] == -1)) &&
         ((g.a[2] == 0 && g.b[2] == 1) || (g.a[2] == 1 && g.b[2] == 0)) && g.in[0] != nullptr &&
         g.ld[0] != 0;
}

// Extra input e at (row, col..col+3); zeros outside [m) x [n).
__device__ __forceinline__ float4 epi_load4(const EpiProg& g, int e, int64_t row, int col, int m,
                                            int n) {
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
  if (row >= m || col >= n) return r;
  const float* src = g.in[e] + row * g.ld[e] + col;
  if (g.vec[e] && col + 3 < n) return *reinterpret_cast<const float4*>(src);
  r.x = src[0];
  if (col + 1 < n) r.y = src[1];
  if (col + 2 < n) r.z = src[2];
  if (col + 3 < n) r.w = src[3];
  return r;
}

// The program on four elements: y the GEMM results, e0 / e1 the extra inputs
// at the same positions.  Returns the value of the last node.  MAXN bounds
// the node count (the caller guarantees 0 < g.n_nodes <= MAXN).
//
// The node loop is unrolled, so every v[k] is a register.  An operand that
// is the previous node (the common case in a chain) is read directly; any
// other earlier node is picked by compare-and-select.  Branches depend only
// on the program (kernel parameters), so they are uniform across the warp.
template <int MAXN>
__device__ __forceinline__ float4 epi_eval4(const EpiProg& g, float4 y, float4 e0, float4 e1) {
  static_assert(MAXN <= EPI_MAX_NODES, "node bound");
  float v[MAXN][4];
  float r[4] = {0.f, 0.f, 0.f, 0.f};
  const float yv[4] = {y.x, y.y, y.z, y.w};
  const float e0v[4] = {e0.x, e0.y, e0.z, e0.w};
  const float e1v[4] = {e1.x, e1.y, e1.z, e1.w};
  const int last = g.n_nodes - 1;
#pragma unroll
  for (int k = 0; k < MAXN; ++k) {
    if (k > last) continue;  // uniform; keeps the loop fully unrolled (no break)
    float A[4] = {0.f, 0.f, 0.f, 0.f}, B[4] = {0.f, 0.f, 0.f, 0.f};
    if (k > 0) {
      const int ia = g.a[k], ib = g.b[k];
      if (ia == k - 1) {
#pragma unroll
        for (int q = 0; q < 4; ++q) A[q] = v[k - 1][q];
      } else {
#pragma unroll
        for (int j = 0; j + 1 < k; ++j) {
#pragma unroll
          for (int q = 0; q < 4; ++q) A[q] = ia == j ? v[j][q] : A[q];
        }
      }
      if (ib == k - 1) {
#pragma unroll
        for (int q = 0; q < 4; ++q) B[q] = v[k - 1][q];
      } else if (ib >= 0) {
#pragma unroll
        for (int j = 0; j + 1 < k; ++j) {
#pragma unroll
          for (int q = 0; q < 4; ++q) B[q] = ib == j ? v[j][q] : B[q];
        }
      }
    }
    const float al = g.alpha[k];
    switch (g.op[k]) {
      case kEpiLoad: {
        const int s = g.src[k];
#pragma unroll
        for (int q = 0; q < 4; ++q) v[k][q] = s < 0 ? yv[q] : (s == 0 ? e0v[q] : e1v[q]);
        break;
      }
      case kEpiConst:
#pragma unroll
        for (int q = 0; q < 4; ++q) v[k][q] = g.c[k];
        break;
      case kEpiAdd:
#pragma unroll
        for (int q = 0; q < 4; ++q) v[k][q] = __fadd_rn(A[q], __fmul_rn(al, B[q]));
        break;
      case kEpiMul:
#pragma unroll
        for (int q = 0; q < 4; ++q) v[k][q] = __fmul_rn(A[q], B[q]);
        break;
      case kEpiRelu:
#pragma unroll
        for (int q = 0; q < 4; ++q) v[k][q] = A[q] > 0.f ? A[q] : 0.f;
        break;
      case kEpiSilu:
#pragma unroll
        for (int q = 0; q < 4; ++q) v[k][q] = A[q] / (1.f + expf(-A[q]));
        break;
      case kEpiNeg:
#pragma unroll
        for (int q = 0; q < 4; ++q) v[k][q] = -A[q];
        break;
      case kEpiScale:
#pragma unroll
        for (int q = 0; q < 4; ++q) v[k][q] = __fmul_rn(al, A[q]);
        break;
      case kEpiSigmoid:
#pragma unroll
        for (int q = 0; q < 4; ++q) v[k][q] = 1.f / (1.f + expf(-A[q]));
        break;
      case kEpiSub:
#pragma unroll
        for (int q = 0; q < 4; ++q) v[k][q] = __fadd_rn(A[q], __fmul_rn(-al, B[q]));
        break;
      case kEpiExp:
#pragma unroll
        for (int q = 0; q < 4; ++q) v[k][q] = expf(A[q]);
        break;
      default:  // kEpiAbs
#pragma unroll
        for (int q = 0; q < 4; ++q) v[k][q] = fabsf(A[q]);
        break;
    }
    if (k == last) {
#pragma unroll
      for (int q = 0; q < 4; ++q) r[q] = v[k][q];
    }
  }
  return make_float4(r[0], r[1], r[2], r[3]);
}

#endif  // __CUDACC__

}  // namespace tvr

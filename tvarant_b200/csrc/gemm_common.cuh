// Epilogue arithmetic shared by the GEMM kernels.
#pragma once

#include "epilogue_prog.cuh"

#include <cuda_runtime.h>

#include <cstdint>

namespace tvr {

// act(alpha*acc + beta*prev) with the reference's operation order
// (csrc/kernels/host/HostKernels.cpp:130-140, csrc/jit/Jit.h:48-56): two
// separately rounded products and one sum, then relu (x > 0 ? x : 0) or
// silu (x / (1 + exp(-x))).
__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == 1) return v > 0.f ? v : 0.f;
  if (act == 2) return v / (1.f + expf(-v));
  return v;
}

__device__ __forceinline__ float epilogue_value(float acc, float prev, float alpha, float beta,
                                                int act) {
  return apply_act(__fadd_rn(__fmul_rn(alpha, acc), __fmul_rn(beta, prev)), act);
}

// The same on four values with the activation fixed at compile time, for
// the tensor-core epilogue.  SiLU there uses the fast exponential and
// division intrinsics (a few ulp, inside the GEMM tolerances) so that the
// epilogue keeps pace with output bandwidth; the CUDA-core kernel keeps the
// reference's IEEE expression.
template <int ACT>
__device__ __forceinline__ float act_fixed(float v) {
  if constexpr (ACT == 1) return v > 0.f ? v : 0.f;
  else if constexpr (ACT == 2) return __fdividef(v, 1.f + __expf(-v));
  else return v;
}

template <int ACT>
__device__ __forceinline__ void epilogue4(float4& x, const float4& prev, float alpha, float beta) {
  x.x = act_fixed<ACT>(__fadd_rn(__fmul_rn(alpha, x.x), __fmul_rn(beta, prev.x)));
  x.y = act_fixed<ACT>(__fadd_rn(__fmul_rn(alpha, x.y), __fmul_rn(beta, prev.y)));
  x.z = act_fixed<ACT>(__fadd_rn(__fmul_rn(alpha, x.z), __fmul_rn(beta, prev.z)));
  x.w = act_fixed<ACT>(__fadd_rn(__fmul_rn(alpha, x.w), __fmul_rn(beta, prev.w)));
}

// Entry points of the individual GEMM implementations (host side).
int gemm_simt(const float* a, const float* b, const float* bias, float* c, int64_t m,
              int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int64_t batch,
              int64_t sa, int64_t sb, int64_t sc, float alpha, float beta, int act,
              bool trans_b, cudaStream_t stream);

// fp32 FMA GEMV for one or two rows against a K-major weight; applies when
// gemm_skinny_applies() holds (16-byte aligned rows, K % 4 == 0).
bool gemm_skinny_applies(const float* a, const float* b, int64_t m, int64_t n, int64_t k,
                         int64_t lda, int64_t ldb, bool trans_b);
int gemm_skinny(const float* a, const float* b, const float* bias, float* c, int64_t m, int64_t n,
                int64_t k, int64_t lda, int64_t ldb, int64_t ldc, float alpha, float beta,
                int act, cudaStream_t stream);

// Weight-streaming tcgen05 GEMM for at most 128 rows against a K-major
// weight (split-K over a thread-block cluster, reduced in distributed shared
// memory); applies when gemm_ws_applies() holds.  A non-null `resid` [m, n]
// (row stride resid_ld) is added to the result in the epilogue.
bool gemm_ws_applies(const float* x, const float* w, int64_t m, int64_t n, int64_t k,
                     int64_t ldx, int64_t ldw, bool trans_b);
int gemm_ws(const float* x, const float* w, const float* bias, float* c, int64_t m, int64_t n,
            int64_t k, int64_t ldx, int64_t ldw, int64_t ldc, float alpha, float beta, int act,
            bool split3, cudaStream_t stream, const float* resid = nullptr,
            int64_t resid_ld = 0);

// silu(x . Wg^T) * (x . Wu^T) in one TF32 tcgen05 pass (K-major weights);
// TVR_ERR_UNSUPPORTED when the operands cannot be described by TMA maps.
int gemm_tcgen05_swiglu(const float* x, const float* wg, const float* wu, float* out, int64_t m,
                        int64_t n, int64_t k, int64_t ldx, int64_t ldwg, int64_t ldwu,
                        int64_t ldo, cudaStream_t stream);

// C = A . B^T (TF32, K-major B) summed over `world` ranks through NVLink
// SHARP in the same kernel; tvr_gemm_nvls_all_reduce_f32 validates the
// cross-rank arguments.  Checks the shapes, then advances the epoch counter
// on the stream and launches (nothing is launched when a check fails).
int gemm_tcgen05_nvls(const float* a, const float* b, float* c, void* c_multicast, int64_t m,
                      int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                      void* const* peer_flags, int rank, int world, uint32_t* epoch,
                      int reduce_ctas, cudaStream_t stream);

// Returns TVR_ERR_UNSUPPORTED (without recording an error) when the
// operands cannot be described by TMA tensor maps; the caller then uses
// gemm_simt.  With a pointwise program (prog non-null with nodes), the
// program is applied to the output: in the epilogue when possible, else by
// epi_prog_inplace after the GEMM.
int gemm_tcgen05(const float* a, const float* b, const float* bias, float* c, int64_t m,
                 int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int64_t batch,
                 int64_t sa, int64_t sb, int64_t sc, float alpha, float beta, int act,
                 bool trans_b, bool split3, cudaStream_t stream, const EpiProg* prog = nullptr);

// c[r, j] = program(c[r, j], extra inputs at (r, j)) over [m, n] (row stride
// ldc), in place (gemm_epilogue.cu).
int epi_prog_inplace(const EpiProg& prog, float* c, int64_t ldc, int64_t m, int64_t n,
                     cudaStream_t stream);

// Checks a tvr_pw_node program whose input gemm_input is the GEMM result and
// whose other inputs are [m, n] fp32 with row strides input_ld (0: one row
// broadcast), none overlapping the output c, and packs it (gemm_epilogue.cu).
int build_epi_prog(const tvr_pw_node* nodes, int n_nodes, int n_inputs, int gemm_input,
                   const float* const* inputs, const int64_t* input_ld, const float* c,
                   int64_t m, int64_t n, int64_t ldc, EpiProg* out);

}  // namespace tvr

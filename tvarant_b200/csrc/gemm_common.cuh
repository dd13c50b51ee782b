// Epilogue arithmetic shared by the GEMM kernels.
#pragma once

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

// Entry points of the individual GEMM implementations (host side).
int gemm_simt(const float* a, const float* b, const float* bias, float* c, int64_t m,
              int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int64_t batch,
              int64_t sa, int64_t sb, int64_t sc, float alpha, float beta, int act,
              bool trans_b, cudaStream_t stream);

// Returns TVR_ERR_UNSUPPORTED (without recording an error) when the
// operands cannot be described by TMA tensor maps; the caller then uses
// gemm_simt.
int gemm_tcgen05(const float* a, const float* b, const float* bias, float* c, int64_t m,
                 int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int64_t batch,
                 int64_t sa, int64_t sb, int64_t sc, float alpha, float beta, int act,
                 bool trans_b, bool split3, cudaStream_t stream);

}  // namespace tvr

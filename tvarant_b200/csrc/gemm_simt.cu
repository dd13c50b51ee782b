// CUDA-core fp32 GEMM used for TVR_GEMM_FP32, for tiny problems, and for
// operands the tensor-core path cannot address with TMA (unaligned rows).
//
// Each output is accumulated over k = 0, 1, ..., K-1 in order with a
// separately rounded multiply and add, then `alpha*acc + beta*prev` and the
// activation — the exact operation sequence of the reference's
// host::gemm_bias_act_f32 (csrc/kernels/host/HostKernels.cpp:100-144), so
// this path reproduces the reference simulator bit for bit.
#include "internal.h"

#include "gemm_common.cuh"

namespace tvr {
namespace {

constexpr int TM = 64, TN = 64, TK = 16, THREADS = 256;

template <bool TRANS_B>
__global__ void __launch_bounds__(THREADS) gemm_simt_kernel(
    const float* __restrict__ A, const float* __restrict__ B, const float* __restrict__ bias,
    float* __restrict__ C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
    int64_t ldc, int64_t sa, int64_t sb, int64_t sc, int batch, float alpha, float beta,
    int act, int use_prev) {
  __shared__ float As[TK][TM + 4];
  __shared__ float Bs[TK][TN + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  for (int bz = blockIdx.z; bz < batch; bz += gridDim.z) {
    const float* Ab = A + bz * sa;
    const float* Bb = B + bz * sb;
    float* Cb = C + bz * sc;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * TM;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * TN;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    for (int64_t k0 = 0; k0 < K; k0 += TK) {
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int idx = threadIdx.x + t * THREADS;
        const int r = idx / TK, c = idx % TK;
        const int64_t gm = m0 + r, gk = k0 + c;
        As[c][r] = (gm < M && gk < K) ? Ab[gm * lda + gk] : 0.f;
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int idx = threadIdx.x + t * THREADS;
        if (TRANS_B) {
          const int r = idx / TK, c = idx % TK;  // r: n, c: k
          const int64_t gn = n0 + r, gk = k0 + c;
          Bs[c][r] = (gn < N && gk < K) ? Bb[gn * ldb + gk] : 0.f;
        } else {
          const int r = idx / TN, c = idx % TN;  // r: k, c: n
          const int64_t gk = k0 + r, gn = n0 + c;
          Bs[r][c] = (gk < K && gn < N) ? Bb[gk * ldb + gn] : 0.f;
        }
      }
      __syncthreads();
      const int kmax = static_cast<int>(K - k0 < TK ? K - k0 : TK);
      for (int kk = 0; kk < kmax; ++kk) {
        float av[4], bv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(av[i], bv[j]));
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t gm = m0 + ty * 4 + i;
      if (gm >= M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t gn = n0 + tx * 4 + j;
        if (gn >= N) continue;
        float prev = 0.f;
        if (bias != nullptr) prev = bias[gn];
        else if (use_prev) prev = Cb[gm * ldc + gn];
        Cb[gm * ldc + gn] = epilogue_value(acc[i][j], prev, alpha, beta, act);
      }
    }
  }
}

}  // namespace

int gemm_simt(const float* a, const float* b, const float* bias, float* c, int64_t m,
              int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int64_t batch,
              int64_t sa, int64_t sb, int64_t sc, float alpha, float beta, int act,
              bool trans_b, cudaStream_t stream) {
  const int use_prev = (bias == nullptr && beta != 0.f) ? 1 : 0;
  const int64_t gx = ceil_div(n, TN), gy = ceil_div(m, TM);
  TVR_CHECK(gx <= 0x7fffffff && gy <= 65535, "gemm: output too large for the CUDA-core path");
  const unsigned gz = static_cast<unsigned>(batch < 65535 ? batch : 65535);
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy), gz);
  if (trans_b) {
    gemm_simt_kernel<true><<<grid, THREADS, 0, stream>>>(a, b, bias, c, m, n, k, lda, ldb, ldc,
                                                         sa, sb, sc, static_cast<int>(batch),
                                                         alpha, beta, act, use_prev);
  } else {
    gemm_simt_kernel<false><<<grid, THREADS, 0, stream>>>(a, b, bias, c, m, n, k, lda, ldb,
                                                          ldc, sa, sb, sc,
                                                          static_cast<int>(batch), alpha, beta,
                                                          act, use_prev);
  }
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

}  // namespace tvr

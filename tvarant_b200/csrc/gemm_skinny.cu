// Decode-row GEMV: one or two activation rows against a K-major weight
// (nn.Linear layout), C[m,n] = act(alpha * sum_k A[m,k] * W[n,k] + beta * P[m,n]),
// in fp32 FMA on the CUDA cores.
//
// With one or two rows the weight is read once from HBM and the arithmetic is
// negligible (N = K = 4096: 64 MB for 16 MFLOP), so the 3xTF32 mode uses this
// kernel: as fast as the tensor-core weight-streaming kernel and closer to
// exact fp32.  Layout of the work:
//   * a warp owns C = 8 output columns and one of KS = 8 slices of K; lane l
//     reads the 16-byte slices 32i + l of its 8 weight rows (one 512-byte run
//     per row and load) and of the activation rows, and keeps an MT x C
//     block of accumulators;
//   * the weight loads of the next step are issued before the FMAs of the
//     current one, and bypass L1 so that the activation rows stay there;
//   * a CTA holds 8 warps, one per K slice, over the same 8 columns.  Lanes
//     are combined by recursive halving over shuffles, the K slices through
//     shared memory in a fixed order (the result does not depend on
//     scheduling), then bias / alpha / beta / activation are applied with
//     the reference's epilogue (csrc/kernels/host/HostKernels.cpp:130-140).
#include "internal.h"

#include "gemm_common.cuh"

namespace tvr {
namespace {

constexpr int WARPS = 8;

__device__ __forceinline__ float4 ld_stream(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float dot4(const float4& a, const float4& b, float acc) {
  acc = fmaf(a.x, b.x, acc);
  acc = fmaf(a.y, b.y, acc);
  acc = fmaf(a.z, b.z, acc);
  return fmaf(a.w, b.w, acc);
}

// Sums each of the V (a power of two) per-lane values over the warp.  The
// halving steps hand half of the live values to the partner lane, so lane l
// ends up owning the sums of values (l >> S) * P + j, j < P, where
// P = max(1, V/32) and S = 5 - min(5, log2 V); when V < 32 the remaining
// offsets finish with plain butterflies and lane l holds a valid sum if its
// low S bits are zero.
template <int V>
struct LaneSums {
  static constexpr int LOG = V >= 32 ? 5 : (V >= 16 ? 4 : V >= 8 ? 3 : V >= 4 ? 2 : V >= 2 ? 1 : 0);
  static constexpr int P = V >= 32 ? V / 32 : 1;
  static constexpr int S = 5 - LOG;
};

template <int V>
__device__ __forceinline__ void warp_reduce(float (&v)[V], int lane) {
  int cur = V;
#pragma unroll
  for (int step = 0; step < 5; ++step) {
    const int off = 16 >> step;
    if (step < LaneSums<V>::LOG) {
      const bool upper = (lane & off) != 0;
      const int h = cur >> 1;
#pragma unroll
      for (int i = 0; i < V / 2; ++i) {
        if (i < h) {
          const float send = upper ? v[i] : v[i + h];
          const float keep = upper ? v[i + h] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      cur = h;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
  }
}

template <int MT, int C, int KS>
__global__ void __launch_bounds__(WARPS * 32) gemm_skinny_kernel(
    const float* __restrict__ A, const float* __restrict__ W, const float* __restrict__ bias,
    float* __restrict__ out, int m, int n, int k4, int64_t lda, int64_t ldw, int64_t ldc,
    float alpha, float beta, int act, int use_prev) {
  constexpr int CG = WARPS / KS;
  constexpr int V = MT * C;
  using LS = LaneSums<V>;
  __shared__ float partial[KS > 1 ? KS - 1 : 1][CG][V];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cg = warp % CG, ks = warp / CG;
  const int n0 = (blockIdx.x * CG + cg) * C;

  const float* wrow[C];
#pragma unroll
  for (int c = 0; c < C; ++c) wrow[c] = W + static_cast<int64_t>(min(n0 + c, n - 1)) * ldw;
  const float4* arow = reinterpret_cast<const float4*>(A);
  const int64_t lda4 = lda / 4;

  // this warp's slice of K, in 16-byte units, a multiple of 32 units long
  const int per = ((k4 + KS - 1) / KS + 31) / 32 * 32;
  const int kbeg = ks * per;
  const int kend = min(k4, kbeg + per);

  float acc[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = 0.f;

  int q = kbeg + lane;
  float4 wn[C];
  if (q < kend) {
#pragma unroll
    for (int c = 0; c < C; ++c) wn[c] = ld_stream(wrow[c] + 4 * static_cast<int64_t>(q));
  }
  while (q < kend) {
    float4 w[C];
#pragma unroll
    for (int c = 0; c < C; ++c) w[c] = wn[c];
    const int qn = q + 32;
    if (qn < kend) {
#pragma unroll
      for (int c = 0; c < C; ++c) wn[c] = ld_stream(wrow[c] + 4 * static_cast<int64_t>(qn));
    }
#pragma unroll
    for (int r = 0; r < MT; ++r) {
      if (r < m) {
        const float4 x = __ldg(arow + r * lda4 + q);
#pragma unroll
        for (int c = 0; c < C; ++c) acc[r * C + c] = dot4(x, w[c], acc[r * C + c]);
      }
    }
    q = qn;
  }
  warp_reduce<V>(acc, lane);

  const bool owner = (lane & ((1 << LS::S) - 1)) == 0;
  const int base = (lane >> LS::S) * LS::P;
  if constexpr (KS > 1) {
    if (ks > 0 && owner) {
#pragma unroll
      for (int j = 0; j < LS::P; ++j) partial[ks - 1][cg][base + j] = acc[j];
    }
    __syncthreads();
    if (ks > 0) return;
  }
  if (!owner) return;
#pragma unroll
  for (int j = 0; j < LS::P; ++j) {
    const int idx = base + j;
    float sum = acc[j];
#pragma unroll
    for (int s = 0; s < KS - 1; ++s) sum += partial[s][cg][idx];
    const int r = idx / C, col = n0 + idx % C;
    if (r >= m || col >= n) continue;
    float* dst = out + static_cast<int64_t>(r) * ldc + col;
    float prev = 0.f;
    if (bias != nullptr) prev = bias[col];
    else if (use_prev) prev = *dst;
    *dst = epilogue_value(sum, prev, alpha, beta, act);
  }
}

struct Args {
  const float* a;
  const float* w;
  const float* bias;
  float* c;
  int m, n, k4;
  int64_t lda, ldw, ldc;
  float alpha, beta;
  int act, use_prev;
};

template <int MT>
void launch(const Args& g, cudaStream_t stream) {
  constexpr int C = 8, KS = 8;
  constexpr int cols_per_cta = C * (WARPS / KS);
  const unsigned grid = static_cast<unsigned>(ceil_div(g.n, cols_per_cta));
  gemm_skinny_kernel<MT, C, KS><<<grid, WARPS * 32, 0, stream>>>(
      g.a, g.w, g.bias, g.c, g.m, g.n, g.k4, g.lda, g.ldw, g.ldc, g.alpha, g.beta, g.act,
      g.use_prev);
}

}  // namespace

bool gemm_skinny_applies(const float* a, const float* b, int64_t m, int64_t n, int64_t k,
                         int64_t lda, int64_t ldb, bool trans_b) {
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return trans_b && m >= 1 && m <= 2 && n >= 1 && k >= 4 && k % 4 == 0 && lda % 4 == 0 &&
         ldb % 4 == 0 && al16(a) && al16(b) && n < (int64_t(1) << 30) &&
         k < (int64_t(1) << 31) - 256;
}

int gemm_skinny(const float* a, const float* b, const float* bias, float* c, int64_t m, int64_t n,
                int64_t k, int64_t lda, int64_t ldb, int64_t ldc, float alpha, float beta,
                int act, cudaStream_t stream) {
  Args g{a, b, bias, c, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k / 4),
         lda, ldb, ldc, alpha, beta, act, (bias == nullptr && beta != 0.f) ? 1 : 0};
  if (m <= 1) launch<1>(g, stream);
  else launch<2>(g, stream);
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

}  // namespace tvr

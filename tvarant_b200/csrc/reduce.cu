// Row reductions and gathers: softmax, layer norm, embedding.
//
// Reference semantics (csrc/kernels/host/HostKernels.cpp):
//   softmax_f32    :174-198  m = max; e = exp(x - m); out = e * (1/sum e)
//   layer_norm_f32 :200-242  two-pass mean / biased variance,
//                            rstd = 1/sqrt(var + eps), y = (x-mu)*rstd [*w] [+b]
//   embedding_f32  :244-260  row copy, index outside [0, vocab) -> zero row
// The reference loops are scalar and sequential; here each row is read from
// HBM exactly once into registers (16-byte loads), reduced with warp
// shuffles (+ shared memory across warps) and written once, so the kernels
// run at the 1-read + 1-write HBM bound.  Only the order of the fp32 sums
// differs from the reference (tree instead of left-to-right).
#include "internal.h"

#include <cfloat>
#include <cmath>

namespace tvr {
namespace {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reductions; `red` holds one slot per warp (<= 32 warps).
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nwarps ? red[lane] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nwarps ? red[lane] : -INFINITY;
  return warp_max(t);
}

// ---- softmax: one warp per row, the row held in registers ---------------------
// The second half of a warp's row: v holds the lane's float4s of the row (the
// mask already added), m their maximum.  Row maximum and sum by shuffles,
// then exp(v - max) * (1 / sum) streamed to yr.
template <int VPL>
__device__ __forceinline__ void softmax_row_finish(float4 (&v)[VPL], float m, int n4, int lane,
                                                   float4* __restrict__ yr) {
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int c = lane + 32 * j;
    if (c < n4) {
      v[j].x = expf(v[j].x - m);
      v[j].y = expf(v[j].y - m);
      v[j].z = expf(v[j].z - m);
      v[j].w = expf(v[j].w - m);
      s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    }
  }
  s = warp_sum(s);
  const float inv = 1.f / s;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int c = lane + 32 * j;
    if (c < n4) {
      float4 o;
      o.x = v[j].x * inv;
      o.y = v[j].y * inv;
      o.z = v[j].z * inv;
      o.w = v[j].w * inv;
      __stcs(yr + c, o);
    }
  }
}

// x + a with one fp32 rounding per element, as a separate add computes it.
__device__ __forceinline__ float4 add4_rn(float4 v, float4 a) {
  v.x = __fadd_rn(v.x, a.x);
  v.y = __fadd_rn(v.y, a.y);
  v.z = __fadd_rn(v.z, a.z);
  v.w = __fadd_rn(v.w, a.w);
  return v;
}

__device__ __forceinline__ float max4(float m, float4 v) {
  return fmaxf(m, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
}

// VPL float4 per lane; requires dim % 4 == 0, 16-byte aligned rows,
// dim <= 128 * VPL.  MASK: softmax(x + mask[row % mask_rows]) — the additive
// mask (e.g. a causal mask shared by every batch entry and head) is added as
// the row is loaded, with the same single fp32 rounding as a separate add.
template <int VPL, bool MASK = false>
__global__ void __launch_bounds__(256) softmax_warp_kernel(const float* __restrict__ x,
                                                           float* __restrict__ y, int64_t rows,
                                                           int dim,
                                                           const float* __restrict__ mask = nullptr,
                                                           int64_t mask_rows = 1) {
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int n4 = dim >> 2;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       row < rows; row += warps_total) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * dim);
    const float4* mr = MASK ? reinterpret_cast<const float4*>(mask + (row % mask_rows) * dim)
                            : nullptr;
    float4 v[VPL];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (c < n4) {
        v[j] = __ldcs(xr + c);
        if constexpr (MASK) v[j] = add4_rn(v[j], __ldg(mr + c));
        m = max4(m, v[j]);
      }
    }
    softmax_row_finish<VPL>(v, m, n4, lane, reinterpret_cast<float4*>(y + row * dim));
  }
}

// softmax(x + mask[row % mask_rows]) when at least kMaskShare rows share each
// mask row (scores of every batch entry and head under one [L, S] mask).
// A unit is one mask row and kMaskShare of the rows that share it: the block
// stages that mask row in shared memory (two buffers, one barrier per unit),
// and warp w softmaxes the unit's row w with the row in registers as above.
// Against a warp that reads its own mask row from L2, the mask crosses L2
// once per 8 rows instead of once per row ([64, 1024, 1024] scores with a
// [1024, 1024] causal mask on a B200: 0.75-0.79 -> 0.885 of the measured copy
// rate; GPT-2 with bmm attention 0.91 -> 0.94 M tokens/s).  The register cap
// keeps the 1024-wide class at three blocks per SM without spills (four
// blocks at 64 registers spill and ran slower).  Each row's arithmetic is the
// other kernel's, so both give the same bits.
constexpr int kMaskShare = 8;

template <int VPL>
__global__ void __launch_bounds__(32 * kMaskShare, VPL <= 4 ? 4 : (VPL <= 8 ? 3 : 2))
    softmax_shared_mask_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t rows,
                               int dim, const float* __restrict__ mask, int64_t mask_rows) {
  __shared__ float4 ms[2][32 * VPL];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int n4 = dim >> 2;
  const int64_t share = rows / mask_rows;  // rows per mask row
  const int64_t groups = (share + kMaskShare - 1) / kMaskShare;
  const int64_t units = mask_rows * groups;
  int buf = 0;
  for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
    const int64_t mrow = u / groups;
    const int64_t k = (u - mrow * groups) * kMaskShare + warp;  // which of the sharing rows
    const bool active = k < share;
    const int64_t row = k * mask_rows + mrow;  // row % mask_rows == mrow
    float4 v[VPL];
    if (active) {
      const float4* xr = reinterpret_cast<const float4*>(x + row * dim);
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int c = lane + 32 * j;
        if (c < n4) v[j] = __ldcs(xr + c);
      }
    }
    // The row loads above stay in flight while the block stages the mask row.
    // Two buffers: a warp writing buffer b in unit i + 2 has passed unit i + 1's
    // barrier, so every warp has finished reading b in unit i.
    const float4* mg = reinterpret_cast<const float4*>(mask + mrow * dim);
    for (int c = threadIdx.x; c < n4; c += blockDim.x) ms[buf][c] = __ldg(mg + c);
    __syncthreads();
    if (active) {
      float m = -INFINITY;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int c = lane + 32 * j;
        if (c < n4) {
          v[j] = add4_rn(v[j], ms[buf][c]);
          m = max4(m, v[j]);
        }
      }
      softmax_row_finish<VPL>(v, m, n4, lane, reinterpret_cast<float4*>(y + row * dim));
    }
    buf ^= 1;
  }
}

// One block per row, VPT float4 per thread (dim <= 4 * VPT * blockDim).
template <int VPT>
__global__ void __launch_bounds__(1024) softmax_block_kernel(const float* __restrict__ x,
                                                             float* __restrict__ y, int dim) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int n4 = dim >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + row * dim);
  float4 v[VPT];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = threadIdx.x + blockDim.x * j;
    if (c < n4) {
      v[j] = __ldcs(xr + c);
      m = fmaxf(m, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
    }
  }
  m = block_max(m, red);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = threadIdx.x + blockDim.x * j;
    if (c < n4) {
      v[j].x = expf(v[j].x - m);
      v[j].y = expf(v[j].y - m);
      v[j].z = expf(v[j].z - m);
      v[j].w = expf(v[j].w - m);
      s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    }
  }
  s = block_sum(s, red);
  const float inv = 1.f / s;
  float4* yr = reinterpret_cast<float4*>(y + row * dim);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = threadIdx.x + blockDim.x * j;
    if (c < n4) {
      float4 o;
      o.x = v[j].x * inv;
      o.y = v[j].y * inv;
      o.z = v[j].z * inv;
      o.w = v[j].w * inv;
      __stcs(yr + c, o);
    }
  }
}

// Any (outer, dim, inner) layout: one thread per (outer, inner) column,
// adjacent threads on adjacent inner indices (coalesced), online max/sum in
// one pass, then a second pass that writes.  Also the path for rows that do
// not fit the register kernels.  A -inf element adds nothing to the sum, so it
// is skipped: while the running maximum is still -inf (a column that starts
// with masked positions), exp(-inf - -inf) would be NaN.  A column of only
// -inf still ends with s = 0 and NaN outputs, as the reference's max-first
// softmax (HostKernels.cpp:174-198) gives.
__global__ void __launch_bounds__(256) softmax_generic_kernel(const float* __restrict__ x,
                                                              float* __restrict__ y,
                                                              int64_t outer, int64_t dim,
                                                              int64_t inner) {
  const int64_t cols = outer * inner;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < cols;
       t += stride) {
    const int64_t o = t / inner, i = t % inner;
    const float* xc = x + o * dim * inner + i;
    float* yc = y + o * dim * inner + i;
    float m = -INFINITY, s = 0.f;
    for (int64_t d = 0; d < dim; ++d) {
      const float v = xc[d * inner];
      if (v > m) {
        s = s * expf(m - v) + 1.f;
        m = v;
      } else if (v != -INFINITY) {
        s += expf(v - m);
      }
    }
    const float inv = 1.f / s;
    for (int64_t d = 0; d < dim; ++d) yc[d * inner] = expf(xc[d * inner] - m) * inv;
  }
}

// Long rows with inner == 1: one block per row, two passes over the row.
__global__ void __launch_bounds__(1024) softmax_long_row_kernel(const float* __restrict__ x,
                                                                float* __restrict__ y,
                                                                int64_t dim) {
  __shared__ float red[32];
  const float* xr = x + static_cast<int64_t>(blockIdx.x) * dim;
  float* yr = y + static_cast<int64_t>(blockIdx.x) * dim;
  float m = -INFINITY;
  for (int64_t d = threadIdx.x; d < dim; d += blockDim.x) m = fmaxf(m, xr[d]);
  m = block_max(m, red);
  float s = 0.f;
  for (int64_t d = threadIdx.x; d < dim; d += blockDim.x) s += expf(xr[d] - m);
  s = block_sum(s, red);
  const float inv = 1.f / s;
  for (int64_t d = threadIdx.x; d < dim; d += blockDim.x) yr[d] = expf(xr[d] - m) * inv;
}

template <int VPL>
void launch_softmax_warp(const float* x, float* y, int64_t rows, int dim, cudaStream_t s,
                         int dev, const float* mask = nullptr, int64_t mask_rows = 1) {
  const int warps_per_block = 8;
  int64_t blocks = ceil_div(rows, warps_per_block);
  const int64_t cap = static_cast<int64_t>(sm_count(dev)) * 32;
  if (blocks > cap) blocks = cap;
  if (mask != nullptr && rows / mask_rows >= kMaskShare) {
    // persistent: as many blocks as fit on the SMs at once, each walking units
    static int per_sm = [] {
      int n = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, softmax_shared_mask_kernel<VPL>,
                                                        32 * kMaskShare, 0) != cudaSuccess ||
          n < 1) {
        n = 1;
      }
      return n;
    }();
    const int64_t units = mask_rows * ceil_div(rows / mask_rows, int64_t(kMaskShare));
    const int64_t grid = std::min<int64_t>(units, static_cast<int64_t>(sm_count(dev)) * per_sm);
    softmax_shared_mask_kernel<VPL><<<static_cast<unsigned>(grid), 32 * kMaskShare, 0, s>>>(
        x, y, rows, dim, mask, mask_rows);
  } else if (mask != nullptr) {
    softmax_warp_kernel<VPL, true><<<static_cast<unsigned>(blocks), 32 * warps_per_block, 0, s>>>(
        x, y, rows, dim, mask, mask_rows);
  } else {
    softmax_warp_kernel<VPL><<<static_cast<unsigned>(blocks), 32 * warps_per_block, 0, s>>>(
        x, y, rows, dim);
  }
}

// ---- layer norm, rows up to 1024 wide: one warp per row -----------------------
// A block per row spends most of a short row's time in its two block-wide
// reductions (shared memory and __syncthreads); here a warp holds the row in
// registers (VPL float4 per lane), reduces with shuffles, and a block of 8
// warps walks rows in a grid-stride loop.  Same arithmetic per element as the
// block kernel below.
template <int VPL>
__global__ void __launch_bounds__(256) layer_norm_warp_kernel(
    const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
    float* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out,
    int64_t rows, int n, float eps) {
  // a few-row GEMM launched as a programmatic dependent (decode steps) may
  // start streaming its weights now
  if (threadIdx.x == 0) grid_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int n4 = n >> 2;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  const int64_t step = static_cast<int64_t>(gridDim.x) * 8;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5); row < rows;
       row += step) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * n);
    float4 v[VPL];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (c < n4) {
        v[j] = __ldcs(xr + c);
        s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
      } else {
        v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    const float mu = warp_sum(s) / static_cast<float>(n);
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      if (lane + 32 * j < n4) {
        const float a = v[j].x - mu, b = v[j].y - mu, cc = v[j].z - mu, d = v[j].w - mu;
        q += (__fmul_rn(a, a) + __fmul_rn(b, b)) + (__fmul_rn(cc, cc) + __fmul_rn(d, d));
      }
    }
    const float var = warp_sum(q) / static_cast<float>(n);
    const float rs = 1.f / sqrtf(var + eps);
    if (lane == 0) {
      if (mean_out) mean_out[row] = mu;
      if (rstd_out) rstd_out[row] = rs;
    }
    float4* yr = reinterpret_cast<float4*>(y + row * n);
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (c < n4) {
        float4 o;
        o.x = __fmul_rn(v[j].x - mu, rs);
        o.y = __fmul_rn(v[j].y - mu, rs);
        o.z = __fmul_rn(v[j].z - mu, rs);
        o.w = __fmul_rn(v[j].w - mu, rs);
        if (gamma) {
          const float4 g = __ldg(g4 + c);
          o.x = __fmul_rn(o.x, g.x);
          o.y = __fmul_rn(o.y, g.y);
          o.z = __fmul_rn(o.z, g.z);
          o.w = __fmul_rn(o.w, g.w);
        }
        if (beta) {
          const float4 bb = __ldg(b4 + c);
          o.x = __fadd_rn(o.x, bb.x);
          o.y = __fadd_rn(o.y, bb.y);
          o.z = __fadd_rn(o.z, bb.z);
          o.w = __fadd_rn(o.w, bb.w);
        }
        __stcs(yr + c, o);
      }
    }
  }
}

// ---- layer norm: one block per row, the row held in registers ---------------

template <int VPT>
__global__ void __launch_bounds__(1024) layer_norm_kernel(
    const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
    float* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out, int n,
    float eps) {
  __shared__ float red[32];
  // a few-row GEMM launched as a programmatic dependent (decode steps) may
  // start streaming its weights now
  if (threadIdx.x == 0) grid_launch_dependents();
  const int64_t row = blockIdx.x;
  const int n4 = n >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + row * n);
  float4 v[VPT];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = threadIdx.x + blockDim.x * j;
    if (c < n4) {
      v[j] = __ldcs(xr + c);
      s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    } else {
      v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  const float mu = block_sum(s, red) / static_cast<float>(n);
  float q = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = threadIdx.x + blockDim.x * j;
    if (c < n4) {
      const float a = v[j].x - mu, b = v[j].y - mu, cc = v[j].z - mu, d = v[j].w - mu;
      q += (__fmul_rn(a, a) + __fmul_rn(b, b)) + (__fmul_rn(cc, cc) + __fmul_rn(d, d));
    }
  }
  const float var = block_sum(q, red) / static_cast<float>(n);
  const float rs = 1.f / sqrtf(var + eps);
  if (threadIdx.x == 0) {
    if (mean_out) mean_out[row] = mu;
    if (rstd_out) rstd_out[row] = rs;
  }
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  float4* yr = reinterpret_cast<float4*>(y + row * n);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = threadIdx.x + blockDim.x * j;
    if (c < n4) {
      float4 o;
      o.x = __fmul_rn(v[j].x - mu, rs);
      o.y = __fmul_rn(v[j].y - mu, rs);
      o.z = __fmul_rn(v[j].z - mu, rs);
      o.w = __fmul_rn(v[j].w - mu, rs);
      if (gamma) {
        const float4 g = __ldg(g4 + c);
        o.x = __fmul_rn(o.x, g.x);
        o.y = __fmul_rn(o.y, g.y);
        o.z = __fmul_rn(o.z, g.z);
        o.w = __fmul_rn(o.w, g.w);
      }
      if (beta) {
        const float4 b = __ldg(b4 + c);
        o.x = __fadd_rn(o.x, b.x);
        o.y = __fadd_rn(o.y, b.y);
        o.z = __fadd_rn(o.z, b.z);
        o.w = __fadd_rn(o.w, b.w);
      }
      __stcs(yr + c, o);
    }
  }
}

// Any n / alignment: three passes over the row from global memory.
__global__ void __launch_bounds__(256) layer_norm_generic_kernel(
    const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
    float* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out, int64_t n,
    float eps) {
  __shared__ float red[32];
  if (threadIdx.x == 0) grid_launch_dependents();
  const float* xr = x + static_cast<int64_t>(blockIdx.x) * n;
  float* yr = y + static_cast<int64_t>(blockIdx.x) * n;
  float s = 0.f;
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x) s += xr[j];
  const float mu = block_sum(s, red) / static_cast<float>(n);
  float q = 0.f;
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x) {
    const float d = xr[j] - mu;
    q += __fmul_rn(d, d);
  }
  const float var = block_sum(q, red) / static_cast<float>(n);
  const float rs = 1.f / sqrtf(var + eps);
  if (threadIdx.x == 0) {
    if (mean_out) mean_out[blockIdx.x] = mu;
    if (rstd_out) rstd_out[blockIdx.x] = rs;
  }
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x) {
    float o = __fmul_rn(xr[j] - mu, rs);
    if (gamma) o = __fmul_rn(o, gamma[j]);
    if (beta) o = __fadd_rn(o, beta[j]);
    yr[j] = o;
  }
}

// ---- embedding ----------------------------------------------------------------

template <typename I, bool VEC>
__global__ void __launch_bounds__(256) embedding_kernel(const float* __restrict__ w,
                                                        const I* __restrict__ idx,
                                                        float* __restrict__ out, int64_t n_idx,
                                                        int64_t dim, int64_t vocab,
                                                        int rows_per_block) {
  // Threads of a block are split into `rows_per_block` groups, one row each.
  const int group = threadIdx.x / (blockDim.x / rows_per_block);
  const int gthreads = blockDim.x / rows_per_block;
  const int t = threadIdx.x % gthreads;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * rows_per_block + group; row < n_idx;
       row += static_cast<int64_t>(gridDim.x) * rows_per_block) {
    const int64_t id = static_cast<int64_t>(idx[row]);
    const bool valid = id >= 0 && id < vocab;
    if constexpr (VEC) {
      const int64_t d4 = dim >> 2;
      const float4* src = reinterpret_cast<const float4*>(w + (valid ? id : 0) * dim);
      float4* dst = reinterpret_cast<float4*>(out + row * dim);
      for (int64_t c = t; c < d4; c += gthreads) {
        __stcs(dst + c, valid ? __ldg(src + c) : make_float4(0.f, 0.f, 0.f, 0.f));
      }
    } else {
      const float* src = w + (valid ? id : 0) * dim;
      float* dst = out + row * dim;
      for (int64_t c = t; c < dim; c += gthreads) dst[c] = valid ? src[c] : 0.f;
    }
  }
}

template <typename I>
int launch_embedding(const float* w, const I* idx, float* out, int64_t n_idx, int64_t dim,
                     int64_t vocab, cudaStream_t s, int dev) {
  const bool vec = dim % 4 == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  const int64_t units = vec ? dim / 4 : dim;
  int rows_per_block = 1;
  while (rows_per_block < 8 && units * rows_per_block * 2 <= 256) rows_per_block *= 2;
  int64_t blocks = ceil_div(n_idx, rows_per_block);
  const int64_t cap = static_cast<int64_t>(sm_count(dev)) * 16;
  if (blocks > cap) blocks = cap;
  if (vec) {
    embedding_kernel<I, true><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        w, idx, out, n_idx, dim, vocab, rows_per_block);
  } else {
    embedding_kernel<I, false><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        w, idx, out, n_idx, dim, vocab, rows_per_block);
  }
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace tvr

using namespace tvr;

extern "C" {

int tvr_softmax(const float* x, float* y, int64_t outer, int64_t dim, int64_t inner,
                void* stream) {
  TVR_CHECK(outer >= 0 && dim >= 0 && inner >= 0, "tvr_softmax: negative size");
  if (outer == 0 || dim == 0 || inner == 0) return TVR_OK;
  TVR_CHECK(x && y, "tvr_softmax: null pointer");
  const int dev = current_device();
  cudaStream_t s = as_stream(stream);
  if (inner == 1 && dim % 4 == 0 && aligned16(x) && aligned16(y) && dim <= 2048) {
    const int d = static_cast<int>(dim);
    const int vpl = static_cast<int>(ceil_div(dim, 128));
    switch (vpl) {
      case 1: launch_softmax_warp<1>(x, y, outer, d, s, dev); break;
      case 2: launch_softmax_warp<2>(x, y, outer, d, s, dev); break;
      case 3: case 4: launch_softmax_warp<4>(x, y, outer, d, s, dev); break;
      case 5: case 6: case 7: case 8: launch_softmax_warp<8>(x, y, outer, d, s, dev); break;
      default: launch_softmax_warp<16>(x, y, outer, d, s, dev); break;
    }
    TVR_LAUNCH_CHECK();
    return TVR_OK;
  }
  if (inner == 1 && dim % 4 == 0 && aligned16(x) && aligned16(y) && dim <= 16384 &&
      outer <= 0x7fffffff) {
    const int d = static_cast<int>(dim);
    const int threads = 256;
    const int vpt = static_cast<int>(ceil_div(dim, 4 * threads));
    const unsigned blocks = static_cast<unsigned>(outer);
    if (vpt <= 4) softmax_block_kernel<4><<<blocks, threads, 0, s>>>(x, y, d);
    else if (vpt <= 8) softmax_block_kernel<8><<<blocks, threads, 0, s>>>(x, y, d);
    else softmax_block_kernel<16><<<blocks, threads, 0, s>>>(x, y, d);
    TVR_LAUNCH_CHECK();
    return TVR_OK;
  }
  if (inner == 1 && outer <= 0x7fffffff && dim >= 4096) {
    softmax_long_row_kernel<<<static_cast<unsigned>(outer), 512, 0, s>>>(x, y, dim);
    TVR_LAUNCH_CHECK();
    return TVR_OK;
  }
  softmax_generic_kernel<<<elementwise_grid(outer * inner, 256, dev), 256, 0, s>>>(
      x, y, outer, dim, inner);
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

int tvr_softmax_add(const float* x, const float* mask, float* y, int64_t rows, int64_t dim,
                    int64_t mask_rows, void* stream) {
  TVR_CHECK(rows >= 0 && dim >= 0, "tvr_softmax_add: negative size");
  TVR_CHECK(mask_rows >= 1 && rows % mask_rows == 0,
            "tvr_softmax_add: %lld rows are not a whole number of %lld mask rows",
            (long long)rows, (long long)mask_rows);
  if (rows == 0 || dim == 0) return TVR_OK;
  TVR_CHECK(x && mask && y, "tvr_softmax_add: null pointer");
  if (!(dim % 4 == 0 && dim <= 2048 && aligned16(x) && aligned16(y) && aligned16(mask))) {
    return TVR_ERR_UNSUPPORTED;  // the caller adds, then calls tvr_softmax
  }
  const int dev = current_device();
  cudaStream_t s = as_stream(stream);
  const int d = static_cast<int>(dim);
  switch (static_cast<int>(ceil_div(dim, 128))) {
    case 1: launch_softmax_warp<1>(x, y, rows, d, s, dev, mask, mask_rows); break;
    case 2: launch_softmax_warp<2>(x, y, rows, d, s, dev, mask, mask_rows); break;
    case 3: case 4: launch_softmax_warp<4>(x, y, rows, d, s, dev, mask, mask_rows); break;
    case 5: case 6: case 7: case 8: launch_softmax_warp<8>(x, y, rows, d, s, dev, mask, mask_rows); break;
    default: launch_softmax_warp<16>(x, y, rows, d, s, dev, mask, mask_rows); break;
  }
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

int tvr_layer_norm(const float* x, const float* gamma, const float* beta, float* y,
                   float* mean, float* rstd, int64_t rows, int64_t n, float eps,
                   void* stream) {
  TVR_CHECK(rows >= 0 && n > 0, "tvr_layer_norm: invalid shape rows=%lld n=%lld",
            (long long)rows, (long long)n);
  if (rows == 0) return TVR_OK;
  TVR_CHECK(x && y, "tvr_layer_norm: null pointer");
  TVR_CHECK(rows <= 0x7fffffff, "tvr_layer_norm: too many rows");
  cudaStream_t s = as_stream(stream);
  const unsigned blocks = static_cast<unsigned>(rows);
  const bool vec = n % 4 == 0 && aligned16(x) && aligned16(y) && (!gamma || aligned16(gamma)) &&
                   (!beta || aligned16(beta));
  if (vec && n <= 1024 && rows >= 1024) {
    // a warp per row for many short rows (GPT-2's forward: 8192 x 768); a
    // few rows (a decode step's 8) keep a block per row, spread over as many
    // SMs (one block of 8 row-warps made a decode step 75 us slower)
    const int n4 = static_cast<int>(n / 4);
    const int vpl = (n4 + 31) / 32;
    const int64_t cap = static_cast<int64_t>(sm_count(current_device())) * 8;
    const unsigned wblocks = static_cast<unsigned>(std::min<int64_t>(ceil_div(rows, 8), cap));
    const int ni = static_cast<int>(n);
    if (vpl <= 1) {
      layer_norm_warp_kernel<1><<<wblocks, 256, 0, s>>>(x, gamma, beta, y, mean, rstd, rows, ni, eps);
    } else if (vpl <= 2) {
      layer_norm_warp_kernel<2><<<wblocks, 256, 0, s>>>(x, gamma, beta, y, mean, rstd, rows, ni, eps);
    } else if (vpl <= 4) {
      layer_norm_warp_kernel<4><<<wblocks, 256, 0, s>>>(x, gamma, beta, y, mean, rstd, rows, ni, eps);
    } else if (vpl <= 6) {
      layer_norm_warp_kernel<6><<<wblocks, 256, 0, s>>>(x, gamma, beta, y, mean, rstd, rows, ni, eps);
    } else {
      layer_norm_warp_kernel<8><<<wblocks, 256, 0, s>>>(x, gamma, beta, y, mean, rstd, rows, ni, eps);
    }
  } else if (vec && n <= 16384) {
    const int n4 = static_cast<int>(n / 4);
    int vpt = 1;
    while (vpt < 16 && ceil_div(n4, vpt) > 256) vpt *= 2;
    int threads = static_cast<int>(ceil_div(ceil_div(n4, vpt), 32) * 32);
    const int ni = static_cast<int>(n);
    switch (vpt) {
      case 1: layer_norm_kernel<1><<<blocks, threads, 0, s>>>(x, gamma, beta, y, mean, rstd, ni, eps); break;
      case 2: layer_norm_kernel<2><<<blocks, threads, 0, s>>>(x, gamma, beta, y, mean, rstd, ni, eps); break;
      case 4: layer_norm_kernel<4><<<blocks, threads, 0, s>>>(x, gamma, beta, y, mean, rstd, ni, eps); break;
      case 8: layer_norm_kernel<8><<<blocks, threads, 0, s>>>(x, gamma, beta, y, mean, rstd, ni, eps); break;
      default: layer_norm_kernel<16><<<blocks, threads, 0, s>>>(x, gamma, beta, y, mean, rstd, ni, eps); break;
    }
  } else {
    layer_norm_generic_kernel<<<blocks, 256, 0, s>>>(x, gamma, beta, y, mean, rstd, n, eps);
  }
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

int tvr_embedding(const float* weight, const void* indices, int index_bits, float* out,
                  int64_t n_idx, int64_t dim, int64_t vocab, void* stream) {
  TVR_CHECK(n_idx >= 0 && dim >= 0 && vocab >= 0, "tvr_embedding: negative size");
  TVR_CHECK(index_bits == 32 || index_bits == 64, "tvr_embedding: index_bits must be 32 or 64");
  if (n_idx == 0 || dim == 0) return TVR_OK;
  TVR_CHECK(indices && out, "tvr_embedding: null pointer");
  TVR_CHECK(weight || vocab == 0, "tvr_embedding: null weight");
  const int dev = current_device();
  cudaStream_t s = as_stream(stream);
  if (index_bits == 64) {
    return launch_embedding<int64_t>(weight, static_cast<const int64_t*>(indices), out, n_idx,
                                     dim, vocab, s, dev);
  }
  return launch_embedding<int32_t>(weight, static_cast<const int32_t*>(indices), out, n_idx,
                                   dim, vocab, s, dev);
}

}  // extern "C"

// RMSNorm and rotary position embedding (RoPE): the two row operations a
// Llama-style decoder adds to the reference's op set.  The reference has
// neither; a model on it would compose RMSNorm from pow / mean / rsqrt / mul
// and RoPE from slices, negation, cat and multiplies, each a pass over HBM.
// Here each is one pass, at the 1-read + 1-write HBM bound.
//
//   rms_norm: y = x * (1 / sqrt(mean(x^2) + eps)) [* w], per row of n values;
//             the row in registers (16-byte loads), the sum of squares by a
//             block reduction.
//   rope:     for each (batch, position, head) vector of `dim` values and
//             each rotation pair (a, b) with angle table cos / sin at the
//             position:  a' = a*cos - b*sin,  b' = b*cos + a*sin.
//             Pairs are (i, i + dim/2) ("rotate half", as in GPT-NeoX and
//             Hugging Face Llama) or (2i, 2i + 1) (interleaved, as in GPT-J).
// Products and sums are separately rounded (__fmul_rn / __fadd_rn), the
// order a chain of elementwise framework ops produces.
#include "internal.h"

#include <cmath>

#include "fastdiv.cuh"

namespace tvr {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const float t = lane < nwarps ? red[lane] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ float sq4(float4 v) {
  return (__fmul_rn(v.x, v.x) + __fmul_rn(v.y, v.y)) + (__fmul_rn(v.z, v.z) + __fmul_rn(v.w, v.w));
}

// One block per row, VPT float4 per thread (n % 4 == 0, 16-byte aligned rows).
template <int VPT>
__global__ void __launch_bounds__(1024) rms_norm_kernel(const float* __restrict__ x,
                                                        const float* __restrict__ w,
                                                        float* __restrict__ y,
                                                        float* __restrict__ rstd_out, int n,
                                                        float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int n4 = n >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + row * n);
  float4 v[VPT];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = threadIdx.x + blockDim.x * j;
    v[j] = c < n4 ? __ldcs(xr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    s += sq4(v[j]);
  }
  const float ms = block_sum(s, red) / static_cast<float>(n);
  const float rs = 1.f / sqrtf(ms + eps);
  if (threadIdx.x == 0 && rstd_out) rstd_out[row] = rs;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4* yr = reinterpret_cast<float4*>(y + row * n);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = threadIdx.x + blockDim.x * j;
    if (c < n4) {
      float4 o = make_float4(__fmul_rn(v[j].x, rs), __fmul_rn(v[j].y, rs), __fmul_rn(v[j].z, rs),
                             __fmul_rn(v[j].w, rs));
      if (w) {
        const float4 g = __ldg(w4 + c);
        o = make_float4(__fmul_rn(o.x, g.x), __fmul_rn(o.y, g.y), __fmul_rn(o.z, g.z),
                        __fmul_rn(o.w, g.w));
      }
      __stcs(yr + c, o);
    }
  }
}

// Any n / alignment: two passes over the row in global memory.
__global__ void __launch_bounds__(256) rms_norm_generic_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ w,
                                                               float* __restrict__ y,
                                                               float* __restrict__ rstd_out,
                                                               int64_t n, float eps) {
  __shared__ float red[32];
  const float* xr = x + static_cast<int64_t>(blockIdx.x) * n;
  float* yr = y + static_cast<int64_t>(blockIdx.x) * n;
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += __fmul_rn(xr[i], xr[i]);
  const float ms = block_sum(s, red) / static_cast<float>(n);
  const float rs = 1.f / sqrtf(ms + eps);
  if (threadIdx.x == 0 && rstd_out) rstd_out[blockIdx.x] = rs;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float o = __fmul_rn(xr[i], rs);
    yr[i] = w ? __fmul_rn(o, __ldg(w + i)) : o;
  }
}

struct RopeDims {
  int64_t seq, heads, half;      // positions, heads, dim / 2
  int64_t xs_b, xs_s, xs_h;      // input strides (elements) of batch, position, head
  int64_t ys_b, ys_s, ys_h;      // output strides
  int64_t pos_offset;            // position of sequence index 0 in the tables
  int64_t table_stride;          // row stride (elements) of cos / sin
};

// One thread per rotation pair; consecutive threads take consecutive pairs
// of one vector, so loads and stores of a warp are contiguous.
// x and y may be the same buffer (each thread reads its pair before writing it).
template <bool INTERLEAVED>
__global__ void __launch_bounds__(256) rope_kernel(const float* x, float* y,
                                                   const float* __restrict__ cos_t,
                                                   const float* __restrict__ sin_t, RopeDims d,
                                                   int64_t total) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += stride) {
    const int64_t i = t % d.half;
    int64_t r = t / d.half;
    const int64_t h = r % d.heads;
    r /= d.heads;
    const int64_t s = r % d.seq;
    const int64_t b = r / d.seq;
    const float* xv = x + b * d.xs_b + s * d.xs_s + h * d.xs_h;
    float* yv = y + b * d.ys_b + s * d.ys_s + h * d.ys_h;
    const int64_t ia = INTERLEAVED ? 2 * i : i;
    const int64_t ib = INTERLEAVED ? 2 * i + 1 : i + d.half;
    const int64_t ti = (s + d.pos_offset) * d.table_stride + i;
    const float c = __ldg(cos_t + ti), sn = __ldg(sin_t + ti);
    const float a = xv[ia], bb = xv[ib];
    yv[ia] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(bb, sn));
    yv[ib] = __fadd_rn(__fmul_rn(bb, c), __fmul_rn(a, sn));
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Rotate-half with 4 pairs per thread: float4 loads of both halves and of the
// tables (half % 4 == 0, every stride and base 16-byte aligned), 32-bit
// index arithmetic (fewer than 2^31 quads, offsets below 2^31).
struct RopeVec {
  FastDiv quads, heads, seq;
  uint32_t half;
  uint32_t xs_b, xs_s, xs_h, ys_b, ys_s, ys_h;
  uint32_t pos_offset, table_stride;
};

__global__ void __launch_bounds__(256) rope_half_vec_kernel(const float* x, float* y,
                                                            const float* __restrict__ cos_t,
                                                            const float* __restrict__ sin_t,
                                                            RopeVec d, uint32_t total) {
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    uint32_t r = fast_div(t, d.quads);
    const uint32_t i = 4 * (t - r * d.quads.d);
    const uint32_t r2 = fast_div(r, d.heads);
    const uint32_t h = r - r2 * d.heads.d;
    const uint32_t b = fast_div(r2, d.seq);
    const uint32_t s = r2 - b * d.seq.d;
    const float* xv = x + b * d.xs_b + s * d.xs_s + h * d.xs_h;
    float* yv = y + b * d.ys_b + s * d.ys_s + h * d.ys_h;
    const uint32_t ti = (s + d.pos_offset) * d.table_stride + i;
    const float4 a = *reinterpret_cast<const float4*>(xv + i);
    const float4 bb = *reinterpret_cast<const float4*>(xv + i + d.half);
    const float4 c = __ldg(reinterpret_cast<const float4*>(cos_t + ti));
    const float4 sn = __ldg(reinterpret_cast<const float4*>(sin_t + ti));
    float4 oa, ob;
    oa.x = __fsub_rn(__fmul_rn(a.x, c.x), __fmul_rn(bb.x, sn.x));
    oa.y = __fsub_rn(__fmul_rn(a.y, c.y), __fmul_rn(bb.y, sn.y));
    oa.z = __fsub_rn(__fmul_rn(a.z, c.z), __fmul_rn(bb.z, sn.z));
    oa.w = __fsub_rn(__fmul_rn(a.w, c.w), __fmul_rn(bb.w, sn.w));
    ob.x = __fadd_rn(__fmul_rn(bb.x, c.x), __fmul_rn(a.x, sn.x));
    ob.y = __fadd_rn(__fmul_rn(bb.y, c.y), __fmul_rn(a.y, sn.y));
    ob.z = __fadd_rn(__fmul_rn(bb.z, c.z), __fmul_rn(a.z, sn.z));
    ob.w = __fadd_rn(__fmul_rn(bb.w, c.w), __fmul_rn(a.w, sn.w));
    *reinterpret_cast<float4*>(yv + i) = oa;
    *reinterpret_cast<float4*>(yv + i + d.half) = ob;
  }
}

}  // namespace
}  // namespace tvr

using namespace tvr;

extern "C" {

int tvr_rms_norm(const float* x, const float* weight, float* y, float* rstd, int64_t rows,
                 int64_t n, float eps, void* stream) {
  TVR_CHECK(rows >= 0 && n > 0, "tvr_rms_norm: invalid shape rows=%lld n=%lld", (long long)rows,
            (long long)n);
  if (rows == 0) return TVR_OK;
  TVR_CHECK(x && y, "tvr_rms_norm: null pointer");
  TVR_CHECK(rows <= 0x7fffffff, "tvr_rms_norm: too many rows");
  cudaStream_t s = as_stream(stream);
  const unsigned blocks = static_cast<unsigned>(rows);
  const bool vec = n % 4 == 0 && aligned16(x) && aligned16(y) && (!weight || aligned16(weight));
  if (vec && n <= 16 * 4 * 1024) {
    // up to 256 threads, more float4 per thread as rows grow (as for layer norm)
    const int ni = static_cast<int>(n);
    const int64_t n4 = n / 4;
    int vpt = 1;
    while (vpt < 16 && ceil_div(n4, vpt) > 256) vpt *= 2;
    const int threads = static_cast<int>(ceil_div(ceil_div(n4, vpt), 32) * 32);
    switch (vpt) {
      case 1: rms_norm_kernel<1><<<blocks, threads, 0, s>>>(x, weight, y, rstd, ni, eps); break;
      case 2: rms_norm_kernel<2><<<blocks, threads, 0, s>>>(x, weight, y, rstd, ni, eps); break;
      case 4: rms_norm_kernel<4><<<blocks, threads, 0, s>>>(x, weight, y, rstd, ni, eps); break;
      case 8: rms_norm_kernel<8><<<blocks, threads, 0, s>>>(x, weight, y, rstd, ni, eps); break;
      default: rms_norm_kernel<16><<<blocks, threads, 0, s>>>(x, weight, y, rstd, ni, eps); break;
    }
  } else {
    rms_norm_generic_kernel<<<blocks, 256, 0, s>>>(x, weight, y, rstd, n, eps);
  }
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

int tvr_rope(const float* x, float* y, const float* cos_table, const float* sin_table,
             int64_t batch, int64_t seq, int64_t heads, int64_t dim, const int64_t* x_strides,
             const int64_t* y_strides, int64_t table_rows, int64_t table_stride,
             int64_t pos_offset, int interleaved, void* stream) {
  TVR_CHECK(batch >= 0 && seq >= 0 && heads >= 0 && dim >= 0, "tvr_rope: negative size");
  TVR_CHECK(dim % 2 == 0, "tvr_rope: dim %lld is odd", (long long)dim);
  TVR_CHECK(pos_offset >= 0 && pos_offset + seq <= table_rows,
            "tvr_rope: positions %lld..%lld exceed the %lld table rows", (long long)pos_offset,
            (long long)(pos_offset + seq), (long long)table_rows);
  TVR_CHECK(table_stride >= dim / 2, "tvr_rope: table row stride %lld < dim/2",
            (long long)table_stride);
  const int64_t total = batch * seq * heads * (dim / 2);
  if (total == 0) return TVR_OK;
  TVR_CHECK(x && y && cos_table && sin_table && x_strides && y_strides, "tvr_rope: null pointer");
  RopeDims d{seq, heads, dim / 2, x_strides[0], x_strides[1], x_strides[2], y_strides[0],
             y_strides[1], y_strides[2], pos_offset, table_stride};
  const int dev = current_device();
  cudaStream_t s = as_stream(stream);
  const int64_t half = dim / 2;
  auto fits = [](int64_t v) { return v >= 0 && v < (int64_t(1) << 31); };
  const int64_t x_span = (batch - 1) * x_strides[0] + (seq - 1) * x_strides[1] +
                         (heads - 1) * x_strides[2] + dim;
  const int64_t y_span = (batch - 1) * y_strides[0] + (seq - 1) * y_strides[1] +
                         (heads - 1) * y_strides[2] + dim;
  bool vec = !interleaved && half % 4 == 0 && table_stride % 4 == 0 && aligned16(x) &&
             aligned16(y) && aligned16(cos_table) && aligned16(sin_table) &&
             fits(total / 4) && fits(x_span) && fits(y_span) && fits(table_rows * table_stride);
  for (int k = 0; vec && k < 3; ++k) {
    vec = x_strides[k] % 4 == 0 && y_strides[k] % 4 == 0 && x_strides[k] >= 0 && y_strides[k] >= 0;
  }
  if (vec) {
    RopeVec v;
    v.quads = make_fastdiv(static_cast<uint32_t>(half / 4));
    v.heads = make_fastdiv(static_cast<uint32_t>(heads));
    v.seq = make_fastdiv(static_cast<uint32_t>(seq));
    v.half = static_cast<uint32_t>(half);
    v.xs_b = static_cast<uint32_t>(x_strides[0]);
    v.xs_s = static_cast<uint32_t>(x_strides[1]);
    v.xs_h = static_cast<uint32_t>(x_strides[2]);
    v.ys_b = static_cast<uint32_t>(y_strides[0]);
    v.ys_s = static_cast<uint32_t>(y_strides[1]);
    v.ys_h = static_cast<uint32_t>(y_strides[2]);
    v.pos_offset = static_cast<uint32_t>(pos_offset);
    v.table_stride = static_cast<uint32_t>(table_stride);
    const uint32_t quads = static_cast<uint32_t>(total / 4);
    rope_half_vec_kernel<<<elementwise_grid(quads, 256, dev), 256, 0, s>>>(x, y, cos_table,
                                                                           sin_table, v, quads);
    TVR_LAUNCH_CHECK();
    return TVR_OK;
  }
  const unsigned grid = elementwise_grid(total, 256, dev);
  if (interleaved) rope_kernel<true><<<grid, 256, 0, s>>>(x, y, cos_table, sin_table, d, total);
  else rope_kernel<false><<<grid, 256, 0, s>>>(x, y, cos_table, sin_table, d, total);
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

}  // extern "C"

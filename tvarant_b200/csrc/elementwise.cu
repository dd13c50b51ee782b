// Elementwise kernels: unary maps, fill, broadcasting binary ops, strided
// copies and dtype conversion.
//
// The reference runs these as scalar loops (csrc/kernels/host/HostKernels.cpp:17-98)
// or one-work-item-per-element OpenCL kernels (csrc/runtime/OpenCLRuntime.cpp:32-88),
// after materialising broadcasts with expand().contiguous() (csrc/aten/Ops.cpp:287-289).
// Here every kernel is a grid-stride loop over 16-byte vectors where the
// operands allow it, broadcasting is done by index arithmetic in the kernel,
// and all indices are 64-bit.  These ops are HBM-bound: the only goal is to
// move each byte once at full width.
//
// Arithmetic keeps the reference's expression shapes with explicit
// round-to-nearest intrinsics so that nvcc does not contract a*b+c into an
// FMA the reference (compiled for baseline x86-64, no FMA) never performs.
#include "internal.h"

#include "fastdiv.cuh"

#include <cmath>

namespace tvr {
namespace {

constexpr int kThreads = 256;

template <int OP>
__device__ __forceinline__ float unary_op(float x, float s) {
  if constexpr (OP == TVR_UNARY_RELU) {
    return x > 0.f ? x : 0.f;
  } else if constexpr (OP == TVR_UNARY_SILU) {
    return x / (1.f + expf(-x));
  } else if constexpr (OP == TVR_UNARY_NEG) {
    return -x;
  } else if constexpr (OP == TVR_UNARY_ABS) {
    return fabsf(x);
  } else if constexpr (OP == TVR_UNARY_EXP) {
    return expf(x);
  } else if constexpr (OP == TVR_UNARY_EXP2) {
    return exp2f(x);
  } else if constexpr (OP == TVR_UNARY_SQRT) {
    return sqrtf(x);
  } else if constexpr (OP == TVR_UNARY_RSQRT) {
    return 1.f / sqrtf(x);
  } else if constexpr (OP == TVR_UNARY_SCALE) {
    return __fmul_rn(x, s);
  } else if constexpr (OP == TVR_UNARY_ADD_SCALAR) {
    return __fadd_rn(x, s);
  } else if constexpr (OP == TVR_UNARY_SIGMOID) {
    return 1.f / (1.f + expf(-x));
  } else {
    return x;
  }
}

template <int OP>
__global__ void __launch_bounds__(kThreads) unary_vec4_kernel(const float4* __restrict__ x,
                                                              float4* __restrict__ y, int64_t n4,
                                                              float s) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += stride) {
    float4 v = x[i];
    v.x = unary_op<OP>(v.x, s);
    v.y = unary_op<OP>(v.y, s);
    v.z = unary_op<OP>(v.z, s);
    v.w = unary_op<OP>(v.w, s);
    y[i] = v;
  }
}

template <int OP>
__global__ void __launch_bounds__(kThreads) unary_scalar_kernel(const float* __restrict__ x,
                                                                float* __restrict__ y, int64_t n,
                                                                float s) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    y[i] = unary_op<OP>(x[i], s);
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int OP>
int launch_unary(const float* x, float* y, int64_t n, float s, cudaStream_t stream, int dev) {
  if (n <= 0) return TVR_OK;
  int64_t head = 0;
  if (aligned16(x) && aligned16(y)) {
    const int64_t n4 = n / 4;
    if (n4 > 0) {
      unary_vec4_kernel<OP><<<elementwise_grid(n4, kThreads, dev), kThreads, 0, stream>>>(
          reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), n4, s);
      TVR_LAUNCH_CHECK();
    }
    head = n4 * 4;
  }
  if (head < n) {
    const int64_t rest = n - head;
    unary_scalar_kernel<OP><<<elementwise_grid(rest, kThreads, dev), kThreads, 0, stream>>>(
        x + head, y + head, rest, s);
    TVR_LAUNCH_CHECK();
  }
  return TVR_OK;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) fill_kernel(T* __restrict__ dst, T value, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    dst[i] = value;
  }
}

// ---- broadcasting binary ---------------------------------------------------

struct Index8 {
  int64_t size[TVR_MAX_DIMS];
  int64_t sa[TVR_MAX_DIMS];
  int64_t sb[TVR_MAX_DIMS];
};

// Index arithmetic of the N-d kernels when every extent and element offset
// fits in 32 bits.
struct Index8Fast {
  FastDiv div[TVR_MAX_DIMS];
  uint32_t sa[TVR_MAX_DIMS];
  uint32_t sb[TVR_MAX_DIMS];
};

template <int OP>
__device__ __forceinline__ float binary_op(float a, float b, float alpha) {
  if constexpr (OP == TVR_BINARY_ADD) {
    return __fadd_rn(a, __fmul_rn(alpha, b));
  } else {
    return __fmul_rn(a, b);
  }
}

// Both operands dense with the output.
template <int OP>
__global__ void __launch_bounds__(kThreads) binary_dense_vec4_kernel(
    const float4* __restrict__ a, const float4* __restrict__ b, float4* __restrict__ out,
    int64_t n4, float alpha) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += stride) {
    const float4 x = a[i];
    const float4 w = b[i];
    float4 r;
    r.x = binary_op<OP>(x.x, w.x, alpha);
    r.y = binary_op<OP>(x.y, w.y, alpha);
    r.z = binary_op<OP>(x.z, w.z, alpha);
    r.w = binary_op<OP>(x.w, w.w, alpha);
    out[i] = r;
  }
}

// General case: `ndim` collapsed dimensions; the innermost is handled
// `VEC` elements at a time when VEC == 4 (inner size % 4 == 0, each operand's
// inner stride 0 or 1, aligned).
template <int OP, int VEC>
__global__ void __launch_bounds__(kThreads) binary_nd_kernel(const float* __restrict__ a,
                                                             const float* __restrict__ b,
                                                             float* __restrict__ out,
                                                             Index8 ix, int ndim,
                                                             int64_t n_vec, float alpha) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_vec;
       i += stride) {
    int64_t rem = i;
    int64_t oa = 0, ob = 0;
    // innermost dimension counts vectors
    {
      const int64_t inner = ix.size[ndim - 1] / VEC;
      const int64_t c = rem % inner;
      rem /= inner;
      oa += c * VEC * ix.sa[ndim - 1];
      ob += c * VEC * ix.sb[ndim - 1];
    }
    for (int d = ndim - 2; d >= 0; --d) {
      const int64_t c = rem % ix.size[d];
      rem /= ix.size[d];
      oa += c * ix.sa[d];
      ob += c * ix.sb[d];
    }
    if constexpr (VEC == 4) {
      float4 x, w;
      if (ix.sa[ndim - 1] == 1) x = *reinterpret_cast<const float4*>(a + oa);
      else x = make_float4(a[oa], a[oa], a[oa], a[oa]);
      if (ix.sb[ndim - 1] == 1) w = *reinterpret_cast<const float4*>(b + ob);
      else w = make_float4(b[ob], b[ob], b[ob], b[ob]);
      float4 r;
      r.x = binary_op<OP>(x.x, w.x, alpha);
      r.y = binary_op<OP>(x.y, w.y, alpha);
      r.z = binary_op<OP>(x.z, w.z, alpha);
      r.w = binary_op<OP>(x.w, w.w, alpha);
      reinterpret_cast<float4*>(out)[i] = r;
    } else {
      out[i] = binary_op<OP>(a[oa], b[ob], alpha);
    }
  }
}

// The same with 32-bit index arithmetic (FastDiv); dimension d's divisor is
// its extent (the innermost counted in vectors).
template <int OP, int VEC>
__global__ void __launch_bounds__(kThreads) binary_nd_fast_kernel(const float* __restrict__ a,
                                                                  const float* __restrict__ b,
                                                                  float* __restrict__ out,
                                                                  Index8Fast ix, int ndim,
                                                                  uint32_t n_vec, float alpha) {
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n_vec; i += stride) {
    uint32_t rem = i;
    uint32_t oa = 0, ob = 0;
    for (int d = ndim - 1; d >= 0; --d) {
      const uint32_t q = fast_div(rem, ix.div[d]);
      const uint32_t c = rem - q * ix.div[d].d;
      rem = q;
      oa += c * ix.sa[d];
      ob += c * ix.sb[d];
    }
    if constexpr (VEC == 4) {
      const bool a_vec = ix.sa[ndim - 1] == VEC, b_vec = ix.sb[ndim - 1] == VEC;
      float4 x, w;
      if (a_vec) x = *reinterpret_cast<const float4*>(a + oa);
      else x = make_float4(a[oa], a[oa], a[oa], a[oa]);
      if (b_vec) w = *reinterpret_cast<const float4*>(b + ob);
      else w = make_float4(b[ob], b[ob], b[ob], b[ob]);
      float4 r;
      r.x = binary_op<OP>(x.x, w.x, alpha);
      r.y = binary_op<OP>(x.y, w.y, alpha);
      r.z = binary_op<OP>(x.z, w.z, alpha);
      r.w = binary_op<OP>(x.w, w.w, alpha);
      reinterpret_cast<float4*>(out)[i] = r;
    } else {
      out[i] = binary_op<OP>(a[oa], b[ob], alpha);
    }
  }
}

// Collapses adjacent dimensions that are contiguous for the output and for
// both operands, and drops size-1 dimensions.  Returns the new rank.
int collapse_binary(int ndim, const int64_t* sizes, const int64_t* sa, const int64_t* sb,
                    Index8* ix) {
  int r = 0;
  for (int d = 0; d < ndim; ++d) {
    if (sizes[d] == 1) continue;
    if (r > 0) {
      const int p = r - 1;
      // merge if dim p is "outer" of dim d for all operands: stride_p == stride_d * size_d
      if (ix->sa[p] == sa[d] * sizes[d] && ix->sb[p] == sb[d] * sizes[d]) {
        ix->size[p] *= sizes[d];
        ix->sa[p] = sa[d];
        ix->sb[p] = sb[d];
        continue;
      }
    }
    ix->size[r] = sizes[d];
    ix->sa[r] = sa[d];
    ix->sb[r] = sb[d];
    ++r;
  }
  if (r == 0) {
    ix->size[0] = 1;
    ix->sa[0] = 0;
    ix->sb[0] = 0;
    r = 1;
  }
  return r;
}

template <int OP>
int launch_binary(const float* a, const float* b, float* out, int ndim, const int64_t* sizes,
                  const int64_t* sa, const int64_t* sb, float alpha, cudaStream_t stream,
                  int dev) {
  int64_t numel = 1;
  for (int d = 0; d < ndim; ++d) numel *= sizes[d];
  if (numel == 0) return TVR_OK;
  Index8 ix;
  const int r = collapse_binary(ndim, sizes, sa, sb, &ix);
  const bool a_dense = (r == 1 && ix.sa[0] == 1) || numel == 1;
  const bool b_dense = (r == 1 && ix.sb[0] == 1) || numel == 1;
  if (a_dense && b_dense && aligned16(a) && aligned16(b) && aligned16(out) && numel % 4 == 0) {
    const int64_t n4 = numel / 4;
    binary_dense_vec4_kernel<OP><<<elementwise_grid(n4, kThreads, dev), kThreads, 0, stream>>>(
        reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b),
        reinterpret_cast<float4*>(out), n4, alpha);
    TVR_LAUNCH_CHECK();
    return TVR_OK;
  }
  const int64_t inner = ix.size[r - 1];
  const bool vec_ok = inner % 4 == 0 && (ix.sa[r - 1] == 0 || ix.sa[r - 1] == 1) &&
                      (ix.sb[r - 1] == 0 || ix.sb[r - 1] == 1) && aligned16(out) &&
                      (ix.sa[r - 1] == 0 || aligned16(a)) && (ix.sb[r - 1] == 0 || aligned16(b));
  bool outer_aligned = true;
  for (int d = 0; d < r - 1; ++d) {
    if ((ix.sa[r - 1] == 1 && ix.sa[d] % 4 != 0) || (ix.sb[r - 1] == 1 && ix.sb[d] % 4 != 0)) {
      outer_aligned = false;
    }
  }
  const int vec = (vec_ok && outer_aligned) ? 4 : 1;
  // 32-bit index arithmetic when every element offset fits
  bool fits = numel / vec < (int64_t(1) << 31);
  int64_t max_a = 0, max_b = 0;  // largest element offset of each operand
  for (int d = 0; fits && d < r; ++d) {
    fits = ix.sa[d] >= 0 && ix.sb[d] >= 0 && ix.size[d] < (int64_t(1) << 31) &&
           ix.sa[d] < (int64_t(1) << 31) && ix.sb[d] < (int64_t(1) << 31);
    max_a += (ix.size[d] - 1) * ix.sa[d];
    max_b += (ix.size[d] - 1) * ix.sb[d];
  }
  fits = fits && max_a + 4 < (int64_t(1) << 31) && max_b + 4 < (int64_t(1) << 31);
  if (fits) {
    Index8Fast fx;
    for (int d = 0; d < r; ++d) {
      const int64_t ext = d == r - 1 ? ix.size[d] / vec : ix.size[d];
      fx.div[d] = make_fastdiv(static_cast<uint32_t>(ext));
      fx.sa[d] = static_cast<uint32_t>(d == r - 1 ? ix.sa[d] * vec : ix.sa[d]);
      fx.sb[d] = static_cast<uint32_t>(d == r - 1 ? ix.sb[d] * vec : ix.sb[d]);
    }
    const int64_t nv = numel / vec;
    if (vec == 4) {
      binary_nd_fast_kernel<OP, 4><<<elementwise_grid(nv, kThreads, dev), kThreads, 0, stream>>>(
          a, b, out, fx, r, static_cast<uint32_t>(nv), alpha);
    } else {
      binary_nd_fast_kernel<OP, 1><<<elementwise_grid(nv, kThreads, dev), kThreads, 0, stream>>>(
          a, b, out, fx, r, static_cast<uint32_t>(nv), alpha);
    }
  } else if (vec == 4) {
    const int64_t nv = numel / 4;
    binary_nd_kernel<OP, 4><<<elementwise_grid(nv, kThreads, dev), kThreads, 0, stream>>>(
        a, b, out, ix, r, nv, alpha);
  } else {
    binary_nd_kernel<OP, 1><<<elementwise_grid(numel, kThreads, dev), kThreads, 0, stream>>>(
        a, b, out, ix, r, numel, alpha);
  }
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

// ---- strided copy ------------------------------------------------------------

struct CopyIndex {
  int64_t size[TVR_MAX_DIMS];
  int64_t sd[TVR_MAX_DIMS];
  int64_t ss[TVR_MAX_DIMS];
};

template <typename T>
__global__ void __launch_bounds__(kThreads) strided_copy_kernel(T* __restrict__ dst,
                                                                const T* __restrict__ src,
                                                                CopyIndex ix, int ndim,
                                                                int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    int64_t rem = i;
    int64_t od = 0, os = 0;
    for (int d = ndim - 1; d >= 0; --d) {
      const int64_t c = rem % ix.size[d];
      rem /= ix.size[d];
      od += c * ix.sd[d];
      os += c * ix.ss[d];
    }
    dst[od] = src[os];
  }
}

struct CopyIndexFast {
  FastDiv div[TVR_MAX_DIMS];
  uint32_t sd[TVR_MAX_DIMS];
  uint32_t ss[TVR_MAX_DIMS];
};

template <typename T>
__global__ void __launch_bounds__(kThreads) strided_copy_fast_kernel(T* __restrict__ dst,
                                                                     const T* __restrict__ src,
                                                                     CopyIndexFast ix, int ndim,
                                                                     uint32_t n) {
  // Four elements per thread and step, all four loads issued before the
  // stores, so each thread keeps four reads in flight.
  constexpr int U = 4;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < n; i0 += U * stride) {
    uint32_t od[U], os[U];
    T v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t i = i0 + u * stride;
      uint32_t rem = i < n ? i : 0;
      uint32_t a = 0, b = 0;
      for (int d = ndim - 1; d >= 0; --d) {
        const uint32_t q = fast_div(rem, ix.div[d]);
        const uint32_t c = rem - q * ix.div[d].d;
        rem = q;
        a += c * ix.sd[d];
        b += c * ix.ss[d];
      }
      od[u] = a;
      os[u] = b;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (i0 + u * stride < n) v[u] = src[os[u]];
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (i0 + u * stride < n) dst[od[u]] = v[u];
    }
  }
}

// ---- head splits and merges: a transpose of contiguous runs ------------------
// A permutation that keeps a run of L 16-byte elements contiguous in both
// tensors, where the destination's next dimension A (destination stride L)
// is not the source's next dimension B (source stride L): [B, S, 3, H, D] ->
// [3, B, H, S, D] to split attention heads, [B, H, S, D] -> [B, S, H, D] to
// merge them.  Copied in destination order it reads L-element runs at a
// stride of kilobytes (0.64 of the copy rate for GPT-2's head split).  Here
// a block moves a TA x TB tile of runs through shared memory: it reads TB
// runs that are contiguous in the source for each A index, then writes TA
// runs that are contiguous in the destination for each B index.
struct TransposeIndex {
  FastDiv outer[TVR_MAX_DIMS];  // the other dimensions, outermost first
  uint32_t outer_sd[TVR_MAX_DIMS];
  uint32_t outer_ss[TVR_MAX_DIMS];
  int n_outer;
  uint32_t na, nb, run;  // extents of A and B; run length L
  uint32_t a_ss, b_sd;   // A's source stride, B's destination stride
  uint32_t ta, tb;       // tile extents
  uint32_t tiles_a, tiles_b, tiles;
  FastDiv div_run, div_tb_run, div_ta_run, div_tiles_a, div_tiles_b;
};

constexpr int kTransposeTileUnits = 2048;  // 32 KB of shared memory per block

__global__ void __launch_bounds__(kThreads) copy_transpose_kernel(uint4* __restrict__ dst,
                                                                  const uint4* __restrict__ src,
                                                                  TransposeIndex ix) {
  extern __shared__ uint4 tile[];  // [ta][tb][run]
  const uint32_t units = ix.ta * ix.tb * ix.run;
  const uint32_t tb_run = ix.tb * ix.run, ta_run = ix.ta * ix.run;
  for (uint32_t t = blockIdx.x; t < ix.tiles; t += gridDim.x) {
    const uint32_t q = fast_div(t, ix.div_tiles_b);
    const uint32_t b0 = (t - q * ix.tiles_b) * ix.tb;
    uint32_t rem = fast_div(q, ix.div_tiles_a);
    const uint32_t a0 = (q - rem * ix.tiles_a) * ix.ta;
    uint32_t so = 0, dso = 0;
    for (int d = ix.n_outer - 1; d >= 0; --d) {
      const uint32_t qq = fast_div(rem, ix.outer[d]);
      const uint32_t c = rem - qq * ix.outer[d].d;
      rem = qq;
      so += c * ix.outer_ss[d];
      dso += c * ix.outer_sd[d];
    }
    // tile index (a, b, v), v fastest: consecutive threads read consecutive
    // source elements; a thread issues all U of its loads before it stores
    // any of them, so a full tile (2048 elements over 256 threads) is in
    // flight at once
    constexpr int U = kTransposeTileUnits / kThreads;
    for (uint32_t i0 = threadIdx.x; i0 < units; i0 += U * blockDim.x) {
      uint4 val[U];
      bool ok[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t i = i0 + u * blockDim.x;
        const uint32_t a = fast_div(i, ix.div_tb_run);
        const uint32_t r = i - a * tb_run;
        const uint32_t b = fast_div(r, ix.div_run);
        const uint32_t v = r - b * ix.run;
        ok[u] = i < units && a0 + a < ix.na && b0 + b < ix.nb;
        if (ok[u]) val[u] = src[so + (a0 + a) * ix.a_ss + (b0 + b) * ix.run + v];
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (ok[u]) tile[i0 + u * blockDim.x] = val[u];
      }
    }
    __syncthreads();
    // (b, a, v), v fastest: consecutive threads write consecutive destination
    // elements
#pragma unroll 4
    for (uint32_t i = threadIdx.x; i < units; i += blockDim.x) {
      const uint32_t b = fast_div(i, ix.div_ta_run);
      const uint32_t r = i - b * ta_run;
      const uint32_t a = fast_div(r, ix.div_run);
      const uint32_t v = r - a * ix.run;
      if (a0 + a < ix.na && b0 + b < ix.nb) {
        dst[dso + (b0 + b) * ix.b_sd + (a0 + a) * ix.run + v] = tile[(a * ix.tb + b) * ix.run + v];
      }
    }
    __syncthreads();  // the next tile overwrites the shared memory
  }
}

// Launches the transposed-run form when the collapsed copy (counted in
// 16-byte elements) has that shape; *taken says whether it did.
int launch_copy_transpose(void* dst, const void* src, const CopyIndex& ix, int r, int64_t n,
                          cudaStream_t stream, int dev, bool* taken) {
  *taken = false;
  if (r < 3) return TVR_OK;
  const int64_t run = ix.size[r - 1];
  const int A = r - 2;
  if (ix.sd[r - 1] != 1 || ix.ss[r - 1] != 1 || run < 1 || run > 64 || ix.sd[A] != run) {
    return TVR_OK;
  }
  int B = -1;
  for (int d = 0; d < A; ++d) {
    if (ix.ss[d] == run) {
      B = d;
      break;
    }
  }
  if (B < 0) return TVR_OK;
  const int64_t lim = int64_t(1) << 31;
  int64_t max_d = 0, max_s = 0;
  for (int d = 0; d < r; ++d) {
    if (ix.sd[d] < 0 || ix.ss[d] < 0 || ix.sd[d] >= lim || ix.ss[d] >= lim) return TVR_OK;
    max_d += (ix.size[d] - 1) * ix.sd[d];
    max_s += (ix.size[d] - 1) * ix.ss[d];
  }
  if (n >= lim || max_d >= lim || max_s >= lim) return TVR_OK;
  TransposeIndex t{};
  t.run = static_cast<uint32_t>(run);
  t.na = static_cast<uint32_t>(ix.size[A]);
  t.nb = static_cast<uint32_t>(ix.size[B]);
  t.a_ss = static_cast<uint32_t>(ix.ss[A]);
  t.b_sd = static_cast<uint32_t>(ix.sd[B]);
  t.tb = std::min<uint32_t>(t.nb, 16);
  t.ta = std::min<uint32_t>(t.na, std::max<uint32_t>(1, kTransposeTileUnits / (t.tb * t.run)));
  t.tiles_a = static_cast<uint32_t>(ceil_div(int64_t(t.na), int64_t(t.ta)));
  t.tiles_b = static_cast<uint32_t>(ceil_div(int64_t(t.nb), int64_t(t.tb)));
  int64_t outer_count = 1;
  t.n_outer = 0;
  for (int d = 0; d < A; ++d) {
    if (d == B) continue;
    t.outer[t.n_outer] = make_fastdiv(static_cast<uint32_t>(ix.size[d]));
    t.outer_sd[t.n_outer] = static_cast<uint32_t>(ix.sd[d]);
    t.outer_ss[t.n_outer] = static_cast<uint32_t>(ix.ss[d]);
    ++t.n_outer;
    outer_count *= ix.size[d];
  }
  const int64_t tiles = outer_count * t.tiles_a * t.tiles_b;
  if (tiles >= lim) return TVR_OK;
  t.tiles = static_cast<uint32_t>(tiles);
  t.div_run = make_fastdiv(t.run);
  t.div_tb_run = make_fastdiv(t.tb * t.run);
  t.div_ta_run = make_fastdiv(t.ta * t.run);
  t.div_tiles_a = make_fastdiv(t.tiles_a);
  t.div_tiles_b = make_fastdiv(t.tiles_b);
  const size_t smem = static_cast<size_t>(t.ta) * t.tb * t.run * sizeof(uint4);
  // persistent: only as many blocks as are resident at once (with the largest
  // tile), so no block starts its share of the tiles after the others ended
  static const int per_sm = [] {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, copy_transpose_kernel, kThreads,
                                                      kTransposeTileUnits * sizeof(uint4)) !=
            cudaSuccess ||
        b < 1) {
      b = 1;
    }
    return b;
  }();
  const int64_t grid = std::min<int64_t>(tiles, static_cast<int64_t>(sm_count(dev)) * per_sm);
  copy_transpose_kernel<<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(
      static_cast<uint4*>(dst), static_cast<const uint4*>(src), t);
  TVR_LAUNCH_CHECK();
  *taken = true;
  return TVR_OK;
}

// Sort dimensions so the destination is traversed in memory order, then
// merge dimensions contiguous in both tensors.
int collapse_copy(int ndim, const int64_t* sizes, const int64_t* sd, const int64_t* ss,
                  CopyIndex* ix) {
  int order[TVR_MAX_DIMS];
  int m = 0;
  for (int d = 0; d < ndim; ++d) {
    if (sizes[d] != 1) order[m++] = d;
  }
  // insertion sort by destination stride, descending (outermost first)
  for (int i = 1; i < m; ++i) {
    int v = order[i];
    int j = i - 1;
    while (j >= 0 && sd[order[j]] < sd[v]) {
      order[j + 1] = order[j];
      --j;
    }
    order[j + 1] = v;
  }
  int r = 0;
  for (int t = 0; t < m; ++t) {
    const int d = order[t];
    if (r > 0) {
      const int p = r - 1;
      if (ix->sd[p] == sd[d] * sizes[d] && ix->ss[p] == ss[d] * sizes[d]) {
        ix->size[p] *= sizes[d];
        ix->sd[p] = sd[d];
        ix->ss[p] = ss[d];
        continue;
      }
    }
    ix->size[r] = sizes[d];
    ix->sd[r] = sd[d];
    ix->ss[r] = ss[d];
    ++r;
  }
  if (r == 0) {
    ix->size[0] = 1;
    ix->sd[0] = 1;
    ix->ss[0] = 1;
    r = 1;
  }
  return r;
}

template <typename T>
int launch_copy(void* dst, const void* src, const CopyIndex& ix, int r, int64_t n,
                cudaStream_t stream, int dev) {
  bool fits = n < (int64_t(1) << 31);
  int64_t max_d = 0, max_s = 0;  // largest element offset of each tensor
  for (int d = 0; fits && d < r; ++d) {
    fits = ix.sd[d] >= 0 && ix.ss[d] >= 0 && ix.size[d] < (int64_t(1) << 31) &&
           ix.sd[d] < (int64_t(1) << 31) && ix.ss[d] < (int64_t(1) << 31);
    max_d += (ix.size[d] - 1) * ix.sd[d];
    max_s += (ix.size[d] - 1) * ix.ss[d];
  }
  fits = fits && max_d < (int64_t(1) << 31) && max_s < (int64_t(1) << 31);
  if (fits) {
    CopyIndexFast fx;
    for (int d = 0; d < r; ++d) {
      fx.div[d] = make_fastdiv(static_cast<uint32_t>(ix.size[d]));
      fx.sd[d] = static_cast<uint32_t>(ix.sd[d]);
      fx.ss[d] = static_cast<uint32_t>(ix.ss[d]);
    }
    strided_copy_fast_kernel<T><<<elementwise_grid(n, kThreads, dev), kThreads, 0, stream>>>(
        static_cast<T*>(dst), static_cast<const T*>(src), fx, r, static_cast<uint32_t>(n));
  } else {
    strided_copy_kernel<T><<<elementwise_grid(n, kThreads, dev), kThreads, 0, stream>>>(
        static_cast<T*>(dst), static_cast<const T*>(src), ix, r, n);
  }
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

// ---- conversion ----------------------------------------------------------------

template <typename D, typename S>
__global__ void __launch_bounds__(kThreads) convert_kernel(D* __restrict__ dst,
                                                           const S* __restrict__ src, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    if constexpr (sizeof(D) == 1) {
      dst[i] = static_cast<D>(src[i] != S(0));
    } else {
      dst[i] = static_cast<D>(src[i]);
    }
  }
}

template <typename D>
int convert_from(void* dst, const void* src, int src_type, int64_t n, cudaStream_t s,
                 int dev) {
  const unsigned g = elementwise_grid(n, kThreads, dev);
  D* d = static_cast<D*>(dst);
  switch (src_type) {
    case 0: convert_kernel<D, float><<<g, kThreads, 0, s>>>(d, static_cast<const float*>(src), n); break;
    case 1: convert_kernel<D, double><<<g, kThreads, 0, s>>>(d, static_cast<const double*>(src), n); break;
    case 2: convert_kernel<D, int32_t><<<g, kThreads, 0, s>>>(d, static_cast<const int32_t*>(src), n); break;
    case 3: convert_kernel<D, int64_t><<<g, kThreads, 0, s>>>(d, static_cast<const int64_t*>(src), n); break;
    case 4: convert_kernel<D, uint8_t><<<g, kThreads, 0, s>>>(d, static_cast<const uint8_t*>(src), n); break;
    default: return fail(TVR_ERR_INVALID, "tvr_convert: unknown source type %d", src_type);
  }
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

}  // namespace
}  // namespace tvr

using namespace tvr;

extern "C" {

int tvr_unary(int op, const float* x, float* y, int64_t n, float scalar, void* stream) {
  TVR_CHECK(n >= 0, "tvr_unary: negative size");
  if (n == 0) return TVR_OK;
  TVR_CHECK(x != nullptr && y != nullptr, "tvr_unary: null pointer");
  const int dev = current_device();
  cudaStream_t s = as_stream(stream);
  switch (op) {
    case TVR_UNARY_RELU: return launch_unary<TVR_UNARY_RELU>(x, y, n, scalar, s, dev);
    case TVR_UNARY_SILU: return launch_unary<TVR_UNARY_SILU>(x, y, n, scalar, s, dev);
    case TVR_UNARY_NEG: return launch_unary<TVR_UNARY_NEG>(x, y, n, scalar, s, dev);
    case TVR_UNARY_ABS: return launch_unary<TVR_UNARY_ABS>(x, y, n, scalar, s, dev);
    case TVR_UNARY_EXP: return launch_unary<TVR_UNARY_EXP>(x, y, n, scalar, s, dev);
    case TVR_UNARY_EXP2: return launch_unary<TVR_UNARY_EXP2>(x, y, n, scalar, s, dev);
    case TVR_UNARY_SQRT: return launch_unary<TVR_UNARY_SQRT>(x, y, n, scalar, s, dev);
    case TVR_UNARY_RSQRT: return launch_unary<TVR_UNARY_RSQRT>(x, y, n, scalar, s, dev);
    case TVR_UNARY_SCALE: return launch_unary<TVR_UNARY_SCALE>(x, y, n, scalar, s, dev);
    case TVR_UNARY_ADD_SCALAR: return launch_unary<TVR_UNARY_ADD_SCALAR>(x, y, n, scalar, s, dev);
    case TVR_UNARY_SIGMOID: return launch_unary<TVR_UNARY_SIGMOID>(x, y, n, scalar, s, dev);
    case TVR_UNARY_COPY:
      if (x == y) return TVR_OK;
      TVR_CUDA_TRY(cudaMemcpyAsync(y, x, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToDevice, s));
      return TVR_OK;
    default:
      return fail(TVR_ERR_INVALID, "tvr_unary: unknown op %d", op);
  }
}

int tvr_fill(void* dst, const void* value, int elem_size, int64_t n, void* stream) {
  TVR_CHECK(n >= 0, "tvr_fill: negative size");
  if (n == 0) return TVR_OK;
  TVR_CHECK(dst != nullptr && value != nullptr, "tvr_fill: null pointer");
  const int dev = current_device();
  cudaStream_t s = as_stream(stream);
  switch (elem_size) {
    case 1: {
      uint8_t v;
      memcpy(&v, value, 1);
      TVR_CUDA_TRY(cudaMemsetAsync(dst, v, static_cast<size_t>(n), s));
      return TVR_OK;
    }
    case 2: {
      uint16_t v;
      memcpy(&v, value, 2);
      fill_kernel<uint16_t><<<elementwise_grid(n, kThreads, dev), kThreads, 0, s>>>(
          static_cast<uint16_t*>(dst), v, n);
      break;
    }
    case 4: {
      uint32_t v;
      memcpy(&v, value, 4);
      if (v == 0) {
        TVR_CUDA_TRY(cudaMemsetAsync(dst, 0, static_cast<size_t>(n) * 4, s));
        return TVR_OK;
      }
      if ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0 && n % 4 == 0) {
        fill_kernel<uint4><<<elementwise_grid(n / 4, kThreads, dev), kThreads, 0, s>>>(
            static_cast<uint4*>(dst), make_uint4(v, v, v, v), n / 4);
      } else {
        fill_kernel<uint32_t><<<elementwise_grid(n, kThreads, dev), kThreads, 0, s>>>(
            static_cast<uint32_t*>(dst), v, n);
      }
      break;
    }
    case 8: {
      unsigned long long v;
      memcpy(&v, value, 8);
      fill_kernel<unsigned long long><<<elementwise_grid(n, kThreads, dev), kThreads, 0, s>>>(
          static_cast<unsigned long long*>(dst), v, n);
      break;
    }
    default:
      return fail(TVR_ERR_INVALID, "tvr_fill: unsupported element size %d", elem_size);
  }
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

int tvr_binary(int op, const float* a, const float* b, float* out, int ndim,
               const int64_t* sizes, const int64_t* a_strides, const int64_t* b_strides,
               float alpha, void* stream) {
  TVR_CHECK(ndim >= 0 && ndim <= TVR_MAX_DIMS, "tvr_binary: rank %d out of range", ndim);
  TVR_CHECK(ndim == 0 || (sizes && a_strides && b_strides), "tvr_binary: null shape");
  int64_t one = 1, zero = 0;
  if (ndim == 0) {
    sizes = &one;
    a_strides = &zero;
    b_strides = &zero;
    ndim = 1;
  }
  int64_t numel = 1;
  for (int d = 0; d < ndim; ++d) {
    TVR_CHECK(sizes[d] >= 0, "tvr_binary: negative size");
    numel *= sizes[d];
  }
  if (numel == 0) return TVR_OK;
  TVR_CHECK(a && b && out, "tvr_binary: null pointer");
  const int dev = current_device();
  cudaStream_t s = as_stream(stream);
  switch (op) {
    case TVR_BINARY_ADD:
      return launch_binary<TVR_BINARY_ADD>(a, b, out, ndim, sizes, a_strides, b_strides, alpha, s, dev);
    case TVR_BINARY_MUL:
      return launch_binary<TVR_BINARY_MUL>(a, b, out, ndim, sizes, a_strides, b_strides, alpha, s, dev);
    default:
      return fail(TVR_ERR_INVALID, "tvr_binary: unknown op %d", op);
  }
}

int tvr_strided_copy(void* dst, const void* src, int64_t elem_size, int ndim,
                     const int64_t* sizes, const int64_t* dst_strides,
                     const int64_t* src_strides, void* stream) {
  TVR_CHECK(ndim >= 0 && ndim <= TVR_MAX_DIMS, "tvr_strided_copy: rank %d out of range", ndim);
  int64_t numel = 1;
  for (int d = 0; d < ndim; ++d) {
    TVR_CHECK(sizes[d] >= 0, "tvr_strided_copy: negative size");
    numel *= sizes[d];
  }
  if (numel == 0) return TVR_OK;
  TVR_CHECK(dst && src, "tvr_strided_copy: null pointer");
  TVR_CHECK(elem_size == 1 || elem_size == 2 || elem_size == 4 || elem_size == 8 ||
                elem_size == 16,
            "tvr_strided_copy: unsupported element size %lld", (long long)elem_size);
  const int dev = current_device();
  cudaStream_t s = as_stream(stream);
  CopyIndex ix;
  int r = 1;
  if (ndim == 0) {
    ix.size[0] = 1;
    ix.sd[0] = 1;
    ix.ss[0] = 1;
  } else {
    r = collapse_copy(ndim, sizes, dst_strides, src_strides, &ix);
  }
  if (r == 1 && ix.sd[0] == 1 && ix.ss[0] == 1) {
    TVR_CUDA_TRY(cudaMemcpyAsync(dst, src, static_cast<size_t>(numel * elem_size),
                                 cudaMemcpyDeviceToDevice, s));
    return TVR_OK;
  }
  // Widen the element to 16 bytes when the innermost run is contiguous in
  // both tensors and everything stays aligned.
  int64_t es = elem_size;
  while (es < 16) {
    const int64_t f = 2;
    const int64_t inner = ix.size[r - 1];
    bool ok = ix.sd[r - 1] == 1 && ix.ss[r - 1] == 1 && inner % f == 0 &&
              (reinterpret_cast<uintptr_t>(dst) % (es * f)) == 0 &&
              (reinterpret_cast<uintptr_t>(src) % (es * f)) == 0;
    for (int d = 0; ok && d < r - 1; ++d) ok = ix.sd[d] % f == 0 && ix.ss[d] % f == 0;
    if (!ok) break;
    ix.size[r - 1] /= f;
    for (int d = 0; d < r - 1; ++d) {
      ix.sd[d] /= f;
      ix.ss[d] /= f;
    }
    numel /= f;
    es *= f;
  }
  if (es == 16) {
    bool taken = false;
    const int rc = launch_copy_transpose(dst, src, ix, r, numel, s, dev, &taken);
    if (rc != TVR_OK || taken) return rc;
  }
  switch (es) {
    case 1: return launch_copy<uint8_t>(dst, src, ix, r, numel, s, dev);
    case 2: return launch_copy<uint16_t>(dst, src, ix, r, numel, s, dev);
    case 4: return launch_copy<uint32_t>(dst, src, ix, r, numel, s, dev);
    case 8: return launch_copy<unsigned long long>(dst, src, ix, r, numel, s, dev);
    default: return launch_copy<uint4>(dst, src, ix, r, numel, s, dev);
  }
}

int tvr_convert(void* dst, int dst_type, const void* src, int src_type, int64_t n,
                void* stream) {
  TVR_CHECK(n >= 0, "tvr_convert: negative size");
  if (n == 0) return TVR_OK;
  TVR_CHECK(dst && src, "tvr_convert: null pointer");
  const int dev = current_device();
  cudaStream_t s = as_stream(stream);
  switch (dst_type) {
    case 0: return convert_from<float>(dst, src, src_type, n, s, dev);
    case 1: return convert_from<double>(dst, src, src_type, n, s, dev);
    case 2: return convert_from<int32_t>(dst, src, src_type, n, s, dev);
    case 3: return convert_from<int64_t>(dst, src, src_type, n, s, dev);
    case 4: return convert_from<uint8_t>(dst, src, src_type, n, s, dev);
    default: return fail(TVR_ERR_INVALID, "tvr_convert: unknown destination type %d", dst_type);
  }
}

}  // extern "C"

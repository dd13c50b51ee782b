// Selection kernels: where / masked_fill, the triangular masks tril / triu,
// and row argmax (greedy token choice).
//
// The reference runs these on the CPU through its boxed fallback
// (csrc/aten/Ops.cpp:499-501); here they are native so that attention masks
// (is_causal, boolean attn_mask) and model code that builds them stay on the
// device.  Both kernels are HBM-bound with 32-bit index arithmetic
// (fastdiv.cuh) for every tensor whose offsets fit in 31 bits, and a 64-bit
// path otherwise.
#include "internal.h"

#include "cluster.cuh"
#include "fastdiv.cuh"

#include <cfloat>
#include <climits>
#include <cmath>
#include <cstring>

namespace tvr {
namespace {

constexpr int kThreads = 256;

struct Where8 {
  int64_t size[TVR_MAX_DIMS];
  int64_t sc[TVR_MAX_DIMS];
  int64_t sa[TVR_MAX_DIMS];
  int64_t sb[TVR_MAX_DIMS];
};

struct Where8Fast {
  FastDiv div[TVR_MAX_DIMS];
  uint32_t sc[TVR_MAX_DIMS];
  uint32_t sa[TVR_MAX_DIMS];
  uint32_t sb[TVR_MAX_DIMS];
};

// out[i] = cond[i] ? a[i] : b[i] over a dense output; each operand is read
// through its own (possibly zero, i.e. broadcast) strides.
template <typename T>
__global__ void __launch_bounds__(kThreads) where_fast_kernel(const uint8_t* __restrict__ c,
                                                              const T* __restrict__ a,
                                                              const T* __restrict__ b,
                                                              T* __restrict__ out, Where8Fast ix,
                                                              int ndim, uint32_t n) {
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    uint32_t rem = i, oc = 0, oa = 0, ob = 0;
    for (int d = ndim - 1; d >= 0; --d) {
      const uint32_t q = fast_div(rem, ix.div[d]);
      const uint32_t k = rem - q * ix.div[d].d;
      rem = q;
      oc += k * ix.sc[d];
      oa += k * ix.sa[d];
      ob += k * ix.sb[d];
    }
    out[i] = c[oc] ? a[oa] : b[ob];
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) where_kernel(const uint8_t* __restrict__ c,
                                                         const T* __restrict__ a,
                                                         const T* __restrict__ b,
                                                         T* __restrict__ out, Where8 ix, int ndim,
                                                         int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    int64_t rem = i, oc = 0, oa = 0, ob = 0;
    for (int d = ndim - 1; d >= 0; --d) {
      const int64_t k = rem % ix.size[d];
      rem /= ix.size[d];
      oc += k * ix.sc[d];
      oa += k * ix.sa[d];
      ob += k * ix.sb[d];
    }
    out[i] = c[oc] ? a[oa] : b[ob];
  }
}

// Merges adjacent dimensions contiguous for the output and all three
// operands; drops size-1 dimensions.
int collapse_where(int ndim, const int64_t* sizes, const int64_t* sc, const int64_t* sa,
                   const int64_t* sb, Where8* ix) {
  int r = 0;
  for (int d = 0; d < ndim; ++d) {
    if (sizes[d] == 1) continue;
    if (r > 0) {
      const int p = r - 1;
      if (ix->sc[p] == sc[d] * sizes[d] && ix->sa[p] == sa[d] * sizes[d] &&
          ix->sb[p] == sb[d] * sizes[d]) {
        ix->size[p] *= sizes[d];
        ix->sc[p] = sc[d];
        ix->sa[p] = sa[d];
        ix->sb[p] = sb[d];
        continue;
      }
    }
    ix->size[r] = sizes[d];
    ix->sc[r] = sc[d];
    ix->sa[r] = sa[d];
    ix->sb[r] = sb[d];
    ++r;
  }
  if (r == 0) {
    ix->size[0] = 1;
    ix->sc[0] = ix->sa[0] = ix->sb[0] = 0;
    r = 1;
  }
  return r;
}

template <typename T>
int launch_where(const uint8_t* c, const void* a, const void* b, void* out, const Where8& ix,
                 int r, int64_t n, cudaStream_t s, int dev) {
  bool fits = n < (int64_t(1) << 31);
  int64_t mc = 0, ma = 0, mb = 0;
  for (int d = 0; fits && d < r; ++d) {
    fits = ix.sc[d] >= 0 && ix.sa[d] >= 0 && ix.sb[d] >= 0 && ix.size[d] < (int64_t(1) << 31) &&
           ix.sc[d] < (int64_t(1) << 31) && ix.sa[d] < (int64_t(1) << 31) &&
           ix.sb[d] < (int64_t(1) << 31);
    mc += (ix.size[d] - 1) * ix.sc[d];
    ma += (ix.size[d] - 1) * ix.sa[d];
    mb += (ix.size[d] - 1) * ix.sb[d];
  }
  fits = fits && mc < (int64_t(1) << 31) && ma < (int64_t(1) << 31) && mb < (int64_t(1) << 31);
  const unsigned grid = elementwise_grid(n, kThreads, dev);
  if (fits) {
    Where8Fast fx;
    for (int d = 0; d < r; ++d) {
      fx.div[d] = make_fastdiv(static_cast<uint32_t>(ix.size[d]));
      fx.sc[d] = static_cast<uint32_t>(ix.sc[d]);
      fx.sa[d] = static_cast<uint32_t>(ix.sa[d]);
      fx.sb[d] = static_cast<uint32_t>(ix.sb[d]);
    }
    where_fast_kernel<T><<<grid, kThreads, 0, s>>>(c, static_cast<const T*>(a),
                                                   static_cast<const T*>(b), static_cast<T*>(out),
                                                   fx, r, static_cast<uint32_t>(n));
  } else {
    where_kernel<T><<<grid, kThreads, 0, s>>>(c, static_cast<const T*>(a),
                                              static_cast<const T*>(b), static_cast<T*>(out), ix,
                                              r, n);
  }
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

// out[b, i, j] = keep(i, j) ? x[b, i, j] : 0 for dense [batch, rows, cols];
// keep = j - i >= diagonal (upper) or j - i <= diagonal (lower).
template <typename T>
__global__ void __launch_bounds__(kThreads) tri_kernel(const T* __restrict__ x, T* __restrict__ out,
                                                       int64_t n, int64_t rows, int64_t cols,
                                                       int64_t diagonal, int upper) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < n;
       e += stride) {
    const int64_t j = e % cols;
    const int64_t i = (e / cols) % rows;
    const bool keep = upper ? (j - i >= diagonal) : (j - i <= diagonal);
    out[e] = keep ? x[e] : T(0);
  }
}

// Row argmax: index of the largest value of each row of n contiguous values,
// the first one on ties, NaN counting as larger than any number (PyTorch's
// rule).  A row is split over the CL CTAs of a cluster (CL > 1 when there are
// too few rows to fill the GPU, e.g. a decode step's [batch, vocab] logits):
// each thread scans a strided slice of its CTA's part with sixteen loads in
// flight, then a (value, index) reduction across the block and, through
// distributed shared memory, across the cluster.  The comparison orders
// candidates totally (value, then index), so the result does not depend on
// how the row is split.
__device__ __forceinline__ bool argmax_better(float v, int64_t i, float bv, int64_t bi) {
  const bool vn = v != v, bn = bv != bv;
  if (vn != bn) return vn;                    // a NaN beats a number
  if (!vn && v != bv) return v > bv;          // larger number
  return i < bi;                              // equal (or both NaN): first index
}

constexpr int kArgmaxThreads = 256;
constexpr int kArgmaxCluster = 8;

template <int CL>
__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows_kernel(const float* __restrict__ x,
                                                                     int64_t* __restrict__ out,
                                                                     int64_t n) {
  __shared__ float sv[kArgmaxThreads / 32];
  __shared__ int64_t si[kArgmaxThreads / 32];
  const int64_t row = CL == 1 ? blockIdx.x : blockIdx.y;
  const int64_t part = CL == 1 ? 0 : static_cast<int64_t>(cluster_rank());
  const int64_t chunk = (n + CL - 1) / CL;
  const int64_t begin = part * chunk;
  const int64_t end = min(n, begin + chunk);
  const float* xr = x + row * n;
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
  constexpr int U = 16;
  for (int64_t i = begin + threadIdx.x; i < end; i += U * kArgmaxThreads) {
    float v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t j = i + u * kArgmaxThreads;
      v[u] = j < end ? __ldg(xr + j) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t j = i + u * kArgmaxThreads;
      if (j < end && argmax_better(v[u], j, bv, bi)) {
        bv = v[u];
        bi = j;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (argmax_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kArgmaxThreads / 32; ++w) {
      if (argmax_better(sv[w], si[w], bv, bi)) {
        bv = sv[w];
        bi = si[w];
      }
    }
    sv[0] = bv;
    si[0] = bi;
  }
  if (CL == 1) {
    if (threadIdx.x == 0) out[row] = bi;
    return;
  }
  cluster_sync();  // every CTA's candidate is in its shared memory
  if (part == 0 && threadIdx.x == 0) {
    const uint32_t av = smem_addr_u32(&sv[0]), ai = smem_addr_u32(&si[0]);
    for (int r = 1; r < CL; ++r) {
      const float ov = ld_dsmem(dsmem_addr(av, static_cast<uint32_t>(r)));
      const int64_t oi = ld_dsmem_s64(dsmem_addr(ai, static_cast<uint32_t>(r)));
      if (argmax_better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    out[row] = bi;
  }
  cluster_sync();  // no CTA leaves while CTA 0 still reads its shared memory
}

}  // namespace
}  // namespace tvr

using namespace tvr;

extern "C" {

int tvr_where(const void* cond, const void* a, const void* b, void* out, int elem_size, int ndim,
              const int64_t* sizes, const int64_t* cond_strides, const int64_t* a_strides,
              const int64_t* b_strides, void* stream) {
  TVR_CHECK(ndim >= 0 && ndim <= TVR_MAX_DIMS, "tvr_where: rank %d out of range", ndim);
  TVR_CHECK(elem_size == 1 || elem_size == 4 || elem_size == 8,
            "tvr_where: unsupported element size %d", elem_size);
  int64_t one = 1, zero = 0;
  if (ndim == 0) {
    sizes = &one;
    cond_strides = a_strides = b_strides = &zero;
    ndim = 1;
  }
  TVR_CHECK(sizes && cond_strides && a_strides && b_strides, "tvr_where: null shape");
  int64_t n = 1;
  for (int d = 0; d < ndim; ++d) {
    TVR_CHECK(sizes[d] >= 0, "tvr_where: negative size");
    n *= sizes[d];
  }
  if (n == 0) return TVR_OK;
  TVR_CHECK(cond && a && b && out, "tvr_where: null pointer");
  Where8 ix;
  const int r = collapse_where(ndim, sizes, cond_strides, a_strides, b_strides, &ix);
  const int dev = current_device();
  const auto* c = static_cast<const uint8_t*>(cond);
  cudaStream_t s = as_stream(stream);
  switch (elem_size) {
    case 1: return launch_where<uint8_t>(c, a, b, out, ix, r, n, s, dev);
    case 4: return launch_where<uint32_t>(c, a, b, out, ix, r, n, s, dev);
    default: return launch_where<unsigned long long>(c, a, b, out, ix, r, n, s, dev);
  }
}

int tvr_argmax_rows(const float* x, int64_t* out, int64_t rows, int64_t n, void* stream) {
  TVR_CHECK(rows >= 0 && n >= 1, "tvr_argmax_rows: invalid shape rows=%lld n=%lld",
            (long long)rows, (long long)n);
  TVR_CHECK(rows <= 0x7fffffff, "tvr_argmax_rows: too many rows");
  if (rows == 0) return TVR_OK;
  TVR_CHECK(x && out, "tvr_argmax_rows: null pointer");
  const int dev = current_device();
  cudaStream_t s = as_stream(stream);
  // Fewer rows than two per SM and long rows: each row over a cluster of
  // CTAs (a single CTA streaming a 50257-float row took ~80 us).
  if (rows < 2 * static_cast<int64_t>(sm_count(dev)) && n >= kArgmaxCluster * 2048) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(kArgmaxCluster, static_cast<unsigned>(rows), 1);
    cfg.blockDim = dim3(kArgmaxThreads, 1, 1);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    memset(attr, 0, sizeof(attr));
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kArgmaxCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    TVR_CUDA_TRY(cudaLaunchKernelEx(&cfg, argmax_rows_kernel<kArgmaxCluster>, x, out, n));
    return TVR_OK;
  }
  argmax_rows_kernel<1><<<static_cast<unsigned>(rows), kArgmaxThreads, 0, s>>>(x, out, n);
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

int tvr_triangle(const void* x, void* out, int elem_size, int64_t batch, int64_t rows,
                 int64_t cols, int64_t diagonal, int upper, void* stream) {
  TVR_CHECK(batch >= 0 && rows >= 0 && cols >= 0, "tvr_triangle: negative size");
  TVR_CHECK(elem_size == 1 || elem_size == 4 || elem_size == 8,
            "tvr_triangle: unsupported element size %d", elem_size);
  const int64_t n = batch * rows * cols;
  if (n == 0) return TVR_OK;
  TVR_CHECK(x && out, "tvr_triangle: null pointer");
  const int dev = current_device();
  const unsigned grid = elementwise_grid(n, kThreads, dev);
  cudaStream_t s = as_stream(stream);
  switch (elem_size) {
    case 1:
      tri_kernel<uint8_t><<<grid, kThreads, 0, s>>>(static_cast<const uint8_t*>(x),
                                                    static_cast<uint8_t*>(out), n, rows, cols,
                                                    diagonal, upper);
      break;
    case 4:
      tri_kernel<uint32_t><<<grid, kThreads, 0, s>>>(static_cast<const uint32_t*>(x),
                                                     static_cast<uint32_t*>(out), n, rows, cols,
                                                     diagonal, upper);
      break;
    default:
      tri_kernel<unsigned long long><<<grid, kThreads, 0, s>>>(
          static_cast<const unsigned long long*>(x), static_cast<unsigned long long*>(out), n,
          rows, cols, diagonal, upper);
      break;
  }
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

}  // extern "C"

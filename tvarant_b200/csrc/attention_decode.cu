// Attention of a few query rows (decode steps: one new token per sequence)
// over many keys, for head dimension 64:
//   out[b, h, i] = softmax_j(scale * q[b, h, i] . k[b, h, j]) v[b, h, j]
// for the first n keys (n = seq_k, or clamp(*key_len + key_len_add, 1, seq_k)
// read on the device), PyTorch's is_causal mask (key j <= query i) when asked.
//
// With one query row per (sequence, head) the tensor-core kernel would spend a
// 128-row MMA tile on one row and pay two tensor-core round trips per 64-key
// block (~2 us a block, 20 us for a 520-key decode layer), while the work is a
// stream of the cached keys and values.  This kernel streams them on the CUDA
// cores in fp32 (at least as accurate as the TF32 tensor-core path it stands
// in for):
//   * a cluster of CL = 8 CTAs per (sequence, head); CTA r takes keys
//     [r c, (r+1) c), c = ceil(n / CL), so the split depends on n alone and a
//     step gives the same result whether the cache is passed trimmed to n keys
//     or whole with n on the device;
//   * in a CTA four lanes share a key, each holding 16 of its 64 dimensions
//     (the four lanes read 64 contiguous bytes per load instruction, eight keys
//     of a warp 2 KB), so a score is 16 FMAs and two shuffles; every four-lane
//     group keeps its own running maximum, sum and output (online softmax in
//     the exp2 domain) over the keys it is dealt;
//   * the 32 groups of a CTA merge by shuffles, then across warps in shared
//     memory, and the CL CTA partials through distributed shared memory into
//     CTA 0, which writes the normalised rows: one launch, no workspace, and
//     a fixed merge order (the result does not depend on scheduling);
//   * the append form (tvr_attention_decode_append) also takes the step's new
//     key and value rows: the group that owns position *pos reads them from
//     the projection's output instead of the cache and writes them into the
//     cache, so the cache append costs no launch of its own; the arithmetic is
//     the same as appending first and then attending.
// Loads are plain coalesced 16-byte loads into registers (a cp.async ring in
// shared memory measured slower, 11.8 against 10.5 us for a decode layer,
// likely because 35 KB per CTA leaves too little room to place 96 eight-CTA
// clusters in one wave); no TMA, no multicast.
#include "internal.h"

#include <cmath>
#include <cstring>

#include "cluster.cuh"

namespace tvr {
namespace attn_decode {

constexpr int D = 64;
constexpr int CL = 8;         // CTAs per (sequence, head)
constexpr int THREADS = 128;  // four warps, 32 four-lane key groups
constexpr int WARPS = THREADS / 32;
constexpr int GROUPS = THREADS / 4;

struct Params {
  const float* q;
  const float* k;
  const float* v;
  float* out;
  float* lse;  // [B, H, Sq] natural-log sum of exponentials, or null
  int64_t q_sb, q_sh, q_ss;
  int64_t k_sb, k_sh, k_ss;
  int64_t v_sb, v_sh, v_ss;
  int64_t o_sb, o_sh, o_ss;
  int heads;
  int seq_q;
  int seq_k;
  int causal;
  float scale_log2;
  const int64_t* key_len;  // non-null: attend to clamp(*key_len + key_len_add, 1, seq_k) keys
  int key_len_add;
  // append form: k_new / v_new [B, H, 1, D] are the keys and values of
  // position *key_len, written into k_cache / v_cache (= k / v) there
  const float* k_new;
  const float* v_new;
  int64_t kn_sb, kn_sh, vn_sb, vn_sh;
  float* k_cache;
  float* v_cache;
  int* status;
};

// The running state of one query row: maximum and sum in the exp2 domain and
// the unnormalised output over this lane's 16 dimensions.
template <int NQ>
struct RowState {
  float m[NQ];
  float l[NQ];
  float o[NQ][16];
};

// Folds (om, ol, oo) into (m, l, o); an empty side (maximum -inf) has weight 0.
__device__ __forceinline__ void merge_into(float& m, float& l, float* o, float om, float ol,
                                           const float* oo) {
  const float M = fmaxf(m, om);
  const float a = m == -INFINITY ? 0.f : exp2f(m - M);
  const float b = om == -INFINITY ? 0.f : exp2f(om - M);
  l = l * a + ol * b;
#pragma unroll
  for (int d = 0; d < 16; ++d) o[d] = o[d] * a + oo[d] * b;
  m = M;
}

__device__ __forceinline__ float4 ldg4(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}

// One step of a four-lane group's online softmax: key row kv, value row vv
// (this lane's 16 dimensions of each), visible or not.  The group's four
// lanes are `mask`.
template <int NQ>
__device__ __forceinline__ void group_step(RowState<NQ>& st, const float (&q)[NQ][16],
                                           const float (&kv)[16], const float (&vv)[16],
                                           bool live, int j, const Params& p, unsigned mask) {
#pragma unroll
  for (int i = 0; i < NQ; ++i) {
    float acc = 0.f;
#pragma unroll
    for (int d = 0; d < 16; ++d) acc = fmaf(q[i][d], kv[d], acc);
    acc += __shfl_xor_sync(mask, acc, 1);
    acc += __shfl_xor_sync(mask, acc, 2);
    const bool vis = live && (!p.causal || j <= i);
    const float sc = vis ? acc * p.scale_log2 : -INFINITY;
    const float mx = fmaxf(st.m[i], sc);
    if (mx == -INFINITY) continue;  // nothing visible yet (uniform over the group)
    const float corr = st.m[i] == -INFINITY ? 0.f : exp2f(st.m[i] - mx);
    const float pr = sc == -INFINITY ? 0.f : exp2f(sc - mx);
    st.l[i] = st.l[i] * corr + pr;
#pragma unroll
    for (int d = 0; d < 16; ++d) st.o[i][d] = fmaf(pr, vv[d], st.o[i][d] * corr);
    st.m[i] = mx;
  }
}

// This lane's 16 dimensions of a row (float4s 4 c + sub, c = 0..3); zeros
// when the row is not live.
__device__ __forceinline__ void load_row16(const float* row, int sub, bool live,
                                           float (&x)[16]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) a = ldg4(row + 4 * (c * 4 + sub));
    x[4 * c] = a.x;
    x[4 * c + 1] = a.y;
    x[4 * c + 2] = a.z;
    x[4 * c + 3] = a.w;
  }
}

// NQ query rows (seq_q <= NQ); APPEND: the append form (NQ = 1).  One query
// row: at most 72 registers, so seven CTAs fit an SM (a GPT-2 decode step's
// 96 clusters of 8 in one wave).
template <int NQ, bool APPEND>
__global__ void __launch_bounds__(THREADS, NQ == 1 ? 7 : 1)
    attn_decode_kernel(const __grid_constant__ Params p) {
  // the warp partials, then the CTA partial that the cluster merges
  __shared__ float s_wm[WARPS][NQ], s_wl[WARPS][NQ];
  __shared__ float s_wo[WARPS][NQ][D];
  __shared__ float s_cm[NQ], s_cl[NQ];
  __shared__ float s_co[NQ][D];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane & 3;  // dimension quarter of the lane's four-lane group
  const int64_t bh = blockIdx.x / CL;
  const int part = static_cast<int>(cluster_rank());
  const int64_t b = bh / p.heads, h = bh % p.heads;
  const int n = p.key_len != nullptr
                    ? max(1, min(p.seq_k, static_cast<int>(*p.key_len) + p.key_len_add))
                    : p.seq_k;
  const int chunk = (n + CL - 1) / CL;
  const int k0 = part * chunk;
  const int k1 = min(n, k0 + chunk);

  // this lane's 16 dimensions: float4 c*4 + sub of the row, c = 0..3
  float q[NQ][16];
#pragma unroll
  for (int i = 0; i < NQ; ++i) {
    const float* qr = p.q + b * p.q_sb + h * p.q_sh + static_cast<int64_t>(i) * p.q_ss;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < p.seq_q) t = ldg4(qr + 4 * (c * 4 + sub));
      q[i][4 * c] = t.x;
      q[i][4 * c + 1] = t.y;
      q[i][4 * c + 2] = t.z;
      q[i][4 * c + 3] = t.w;
    }
  }
  RowState<NQ> st;
#pragma unroll
  for (int i = 0; i < NQ; ++i) {
    st.m[i] = -INFINITY;
    st.l[i] = 0.f;
#pragma unroll
    for (int d = 0; d < 16; ++d) st.o[i][d] = 0.f;
  }

  const float* kbase = p.k + b * p.k_sb + h * p.k_sh;
  const float* vbase = p.v + b * p.v_sb + h * p.v_sh;
  // Append form: position *key_len (the last of the n keys) is the step's
  // own key.  It is left out of the loop and taken last, from k_new / v_new,
  // by the group the loop would have dealt it to, so every group sees its
  // keys in the same order as when the append runs first.
  int fresh = -1;
  if (APPEND) {
    const int64_t at = *p.key_len;
    if (at >= 0 && at < p.seq_k) {
      fresh = static_cast<int>(at);
    } else if (blockIdx.x == 0 && threadIdx.x == 0 && p.status != nullptr) {
      atomicCAS(p.status, TVR_DEV_OK, TVR_DEV_CACHE_FULL);  // dropped, as tvr_kv_append
    }
  }
  const bool mine = APPEND && fresh >= k0 && fresh < k1;
  const int kend = mine ? fresh : k1;
  // Group g of warp w takes keys k0 + 8 w + g + 32 t (t = 0, 1, ...).  The
  // loop bound is warp-uniform (the score shuffles need every lane); a lane
  // past the end loads nothing and scores -inf.
  for (int jw = k0 + 8 * warp; jw < kend; jw += GROUPS) {
    const int j = jw + (lane >> 2);
    const bool live = j < kend;
    float kv[16], vv[16];
    load_row16(kbase + static_cast<int64_t>(j) * p.k_ss, sub, live, kv);
    load_row16(vbase + static_cast<int64_t>(j) * p.v_ss, sub, live, vv);
    group_step<NQ>(st, q, kv, vv, live, j, p, 0xffffffffu);
  }
  if (APPEND && mine) {
    const int off = fresh - k0;
    if (warp == (off % GROUPS) / 8 && (lane >> 2) == off % 8) {
      float kv[16], vv[16];
      load_row16(p.k_new + b * p.kn_sb + h * p.kn_sh, sub, true, kv);
      load_row16(p.v_new + b * p.vn_sb + h * p.vn_sh, sub, true, vv);
      float* kc = p.k_cache + b * p.k_sb + h * p.k_sh + static_cast<int64_t>(fresh) * p.k_ss;
      float* vc = p.v_cache + b * p.v_sb + h * p.v_sh + static_cast<int64_t>(fresh) * p.v_ss;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int f = 4 * (c * 4 + sub);
        *reinterpret_cast<float4*>(kc + f) =
            make_float4(kv[4 * c], kv[4 * c + 1], kv[4 * c + 2], kv[4 * c + 3]);
        *reinterpret_cast<float4*>(vc + f) =
            make_float4(vv[4 * c], vv[4 * c + 1], vv[4 * c + 2], vv[4 * c + 3]);
      }
      group_step<NQ>(st, q, kv, vv, true, fresh, p, 0xfu << (lane & ~3));
    }
  }

  // the eight groups of a warp (lanes differing in bits 2..4), fixed order
#pragma unroll
  for (int x = 4; x < 32; x <<= 1) {
#pragma unroll
    for (int i = 0; i < NQ; ++i) {
      const float om = __shfl_xor_sync(0xffffffffu, st.m[i], x);
      const float ol = __shfl_xor_sync(0xffffffffu, st.l[i], x);
      float oo[16];
#pragma unroll
      for (int d = 0; d < 16; ++d) oo[d] = __shfl_xor_sync(0xffffffffu, st.o[i][d], x);
      merge_into(st.m[i], st.l[i], st.o[i], om, ol, oo);
    }
  }
  if (lane < 4) {
#pragma unroll
    for (int i = 0; i < NQ; ++i) {
      if (lane == 0) {
        s_wm[warp][i] = st.m[i];
        s_wl[warp][i] = st.l[i];
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int e = 0; e < 4; ++e) s_wo[warp][i][4 * (c * 4 + sub) + e] = st.o[i][4 * c + e];
      }
    }
  }
  __syncthreads();
  // the CTA's partial: thread t merges dimension t % 64 of query row t / 64
  for (int t = threadIdx.x; t < NQ * D; t += THREADS) {
    const int i = t / D, d = t % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, s_wm[w][i]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      const float wm = s_wm[w][i];
      const float a = wm == -INFINITY ? 0.f : exp2f(wm - M);
      L = L + s_wl[w][i] * a;
      O = O + s_wo[w][i][d] * a;
    }
    s_co[i][d] = O;
    if (d == 0) {
      s_cm[i] = M;
      s_cl[i] = L;
    }
  }
  cluster_sync();  // every CTA's partial is in its shared memory
  if (part == 0) {
    const uint32_t am = smem_addr_u32(&s_cm[0]), al = smem_addr_u32(&s_cl[0]);
    const uint32_t ao = smem_addr_u32(&s_co[0][0]);
    for (int t = threadIdx.x; t < NQ * D; t += THREADS) {
      const int i = t / D, d = t % D;
      if (i >= p.seq_q) continue;
      float pm[CL], pl[CL], po[CL];
#pragma unroll
      for (int r = 0; r < CL; ++r) {
        pm[r] = ld_dsmem(dsmem_addr(am + 4u * i, static_cast<uint32_t>(r)));
        pl[r] = ld_dsmem(dsmem_addr(al + 4u * i, static_cast<uint32_t>(r)));
        po[r] = ld_dsmem(dsmem_addr(ao + 4u * (i * D + d), static_cast<uint32_t>(r)));
      }
      float M = -INFINITY;
#pragma unroll
      for (int r = 0; r < CL; ++r) M = fmaxf(M, pm[r]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int r = 0; r < CL; ++r) {
        const float a = pm[r] == -INFINITY ? 0.f : exp2f(pm[r] - M);
        L = L + pl[r] * a;
        O = O + po[r] * a;
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      p.out[b * p.o_sb + h * p.o_sh + static_cast<int64_t>(i) * p.o_ss + d] = O * inv;
      if (d == 0 && p.lse != nullptr) {
        p.lse[bh * p.seq_q + i] = M * 0.69314718055994531f + logf(L);
      }
    }
  }
  cluster_sync();  // no CTA leaves while CTA 0 still reads its shared memory
}

template <int NQ, bool APPEND>
int launch(const Params& p, int64_t bh, cudaStream_t stream) {
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(static_cast<unsigned>(bh * CL), 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  memset(attr, 0, sizeof(attr));
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TVR_CUDA_TRY(cudaLaunchKernelEx(&cfg, attn_decode_kernel<NQ, APPEND>, p));
  return TVR_OK;
}

}  // namespace attn_decode

bool attention_decode_applies(int64_t seq_q, int64_t head_dim) {
  return seq_q >= 1 && seq_q <= 4 && head_dim == attn_decode::D;
}

namespace {

attn_decode::Params decode_params(const float* q, const float* k, const float* v, float* out,
                                  float* lse, int64_t heads, int64_t seq_q, int64_t seq_k,
                                  const int64_t* q_strides, const int64_t* k_strides,
                                  const int64_t* v_strides, const int64_t* o_strides, float scale,
                                  int causal, const int64_t* key_len, int key_len_add) {
  attn_decode::Params p;
  memset(&p, 0, sizeof(p));
  p.q = q;
  p.k = k;
  p.v = v;
  p.out = out;
  p.lse = lse;
  p.q_sb = q_strides[0];
  p.q_sh = q_strides[1];
  p.q_ss = q_strides[2];
  p.k_sb = k_strides[0];
  p.k_sh = k_strides[1];
  p.k_ss = k_strides[2];
  p.v_sb = v_strides[0];
  p.v_sh = v_strides[1];
  p.v_ss = v_strides[2];
  p.o_sb = o_strides[0];
  p.o_sh = o_strides[1];
  p.o_ss = o_strides[2];
  p.heads = static_cast<int>(heads);
  p.seq_q = static_cast<int>(seq_q);
  p.seq_k = static_cast<int>(seq_k);
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.key_len = key_len;
  p.key_len_add = key_len_add;
  return p;
}

int decode_launch(const attn_decode::Params& p, int64_t bh, int64_t seq_q, cudaStream_t stream) {
  using namespace attn_decode;
  TVR_CHECK(bh <= 0x7fffffff / CL, "attention: too many (sequence, head) pairs");
  if (p.k_new != nullptr) return launch<1, true>(p, bh, stream);
  switch (seq_q) {
    case 1: return launch<1, false>(p, bh, stream);
    case 2: return launch<2, false>(p, bh, stream);
    default: return launch<4, false>(p, bh, stream);
  }
}

}  // namespace

int attention_decode(const float* q, const float* k, const float* v, float* out, float* lse,
                     int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_k,
                     const int64_t* q_strides, const int64_t* k_strides,
                     const int64_t* v_strides, const int64_t* o_strides, float scale, int causal,
                     const int64_t* key_len, int key_len_add, cudaStream_t stream) {
  const attn_decode::Params p =
      decode_params(q, k, v, out, lse, heads, seq_q, seq_k, q_strides, k_strides, v_strides,
                    o_strides, scale, causal, key_len, key_len_add);
  return decode_launch(p, batch * heads, seq_q, stream);
}

}  // namespace tvr

using namespace tvr;

extern "C" int tvr_attention_decode_append(
    const float* q, const float* k_new, const float* v_new, float* k_cache, float* v_cache,
    float* out, int64_t batch, int64_t heads, int64_t max_len, int64_t head_dim,
    const int64_t* q_strides, const int64_t* kn_strides, const int64_t* vn_strides,
    const int64_t* kc_strides, const int64_t* vc_strides, const int64_t* o_strides, float scale,
    const int64_t* pos, int mode, void* stream) {
  TVR_CHECK(batch >= 0 && heads >= 0 && max_len >= 0, "attention_decode_append: negative size");
  if (batch == 0 || heads == 0) return TVR_OK;
  TVR_CHECK(max_len >= 1, "attention_decode_append: the cache has no positions");
  TVR_CHECK(q && k_new && v_new && k_cache && v_cache && out && q_strides && kn_strides &&
                vn_strides && kc_strides && vc_strides && o_strides,
            "attention_decode_append: null pointer");
  TVR_CHECK(pos != nullptr && reinterpret_cast<uintptr_t>(pos) % 8 == 0,
            "attention_decode_append: null or unaligned position");
  TVR_CHECK(max_len <= 0x7fffff00, "attention_decode_append: too many positions");
  if (head_dim != attn_decode::D) {
    return fail(TVR_ERR_UNSUPPORTED, "attention_decode_append: head dimension %lld (the kernel "
                "takes %d)", (long long)head_dim, attn_decode::D);
  }
  if (mode != TVR_GEMM_AUTO && mode != TVR_GEMM_TF32 && mode != TVR_GEMM_3XTF32 &&
      mode != TVR_GEMM_FP32) {
    return fail(TVR_ERR_INVALID, "attention_decode_append: unknown precision mode %d", mode);
  }
  if (mode == TVR_GEMM_FP32) {
    return fail(TVR_ERR_UNSUPPORTED,
                "attention_decode_append: FP32 mode keeps the composed attention");
  }
  if (!(scale > 0.f) || !std::isfinite(scale)) {
    return fail(TVR_ERR_UNSUPPORTED, "attention_decode_append: the kernel takes a positive "
                "finite scale");
  }
  auto vec_ok = [](const void* ptr, const int64_t* st) {
    return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0 && st[0] % 4 == 0 && st[1] % 4 == 0 &&
           st[2] % 4 == 0;
  };
  if (!vec_ok(q, q_strides) || !vec_ok(k_new, kn_strides) || !vec_ok(v_new, vn_strides) ||
      !vec_ok(k_cache, kc_strides) || !vec_ok(v_cache, vc_strides)) {
    return fail(TVR_ERR_UNSUPPORTED, "attention_decode_append: operands need 16-byte aligned "
                "bases and strides that are multiples of 4 elements");
  }
  const int dev = current_device();
  attn_decode::Params p =
      decode_params(q, k_cache, v_cache, out, nullptr, heads, 1, max_len, q_strides, kc_strides,
                    vc_strides, o_strides, scale, 0, pos, 1);
  p.k_new = k_new;
  p.v_new = v_new;
  p.kn_sb = kn_strides[0];
  p.kn_sh = kn_strides[1];
  p.vn_sb = vn_strides[0];
  p.vn_sh = vn_strides[1];
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.status = device_status_ptr(dev);
  return decode_launch(p, batch * heads, 1, as_stream(stream));
}

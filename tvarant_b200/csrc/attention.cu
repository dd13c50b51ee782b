// Fused causal / full attention forward for sm_100a (tcgen05 kind::tf32):
// out = softmax(scale * Q K^T [+ causal mask]) V without materialising the
// [seq_q, seq_k] scores.  The reference has no fused attention — its models
// run bmm -> add(mask) -> softmax -> bmm (csrc/aten/LlmOps.cpp:68-148) and
// the fused kernel is a roadmap item — so this kernel serves
// F.scaled_dot_product_attention on the tvarant device (TF32 mode).
//
// One CTA per (128-query tile, batch x head).  Head dimension 64.
//   warp 0     TMA producer: the Q tile once, then K and V tiles of 128 keys
//              into a 2-deep ring, straight from strided [B, H, S, 64]
//              views (no head-split copies);
//   warp 1     TMEM owner and MMA issuer: S_j = Q K_j^T (M=128, N=128,
//              K=64) into one of two TMEM score buffers, issued one block
//              ahead of the softmax; PV_j = P_j V_j (M=128, N=64, K=128)
//              with V read as an N-major operand;
//   warps 2-5  one thread per query row: online softmax in the log2 domain
//              over the row's 128 scores (read twice from TMEM: maximum,
//              then exp2 and the row sum), P written to shared memory in the
//              128-byte-swizzled K-major layout the MMA reads, and the
//              output row kept in 64 registers: O = O * exp2(m_old - m_new)
//              + PV_j.  At the end O / l is stored and the log-sum-exp
//              (natural log) is written.
// Causal masking follows PyTorch's is_causal (key index <= query index,
// aligned at the top-left); keys at or beyond seq_k are masked.  Every
// mbarrier wait is bounded (status word + abort flag), as in gemm_tc.  No TMA
// load uses cluster multicast.
#include "internal.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>

#include "tc_ptx.cuh"

namespace tvr {
namespace attn {

using namespace tc;

constexpr int D = 64;                    // head dimension
constexpr int BM = 128;                  // queries per CTA (MMA M)
constexpr int BN = 128;                  // keys per block
constexpr int ATOM = 128 * 128;          // one [128 rows x 128 B] swizzle block
constexpr int Q_BYTES = BM * D * 4;      // D/32 atoms
constexpr int K_BYTES = BN * D * 4;      // D/32 atoms
constexpr int V_KB_BYTES = 32 * D * 4;   // one 32-key k-block of V: D/32 atoms of [32 x 128 B]
constexpr int V_BYTES = BN * D * 4;      // BN/32 k-blocks
constexpr int P_BYTES = BM * BN * 4;     // BN/32 atoms
constexpr int STAGES = 2;
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;      // S buffers at 0 and 128, PV at 256
constexpr uint32_t PV_COL = 256;
constexpr int BAR_BYTES = 8 * 16;
constexpr int SMEM_BYTES = 1024 + Q_BYTES + STAGES * (K_BYTES + V_BYTES) + P_BYTES + BAR_BYTES;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

struct Params {
  CUtensorMap tma_q;  // {D, seq_q, heads, batch}, box {32, 128}
  CUtensorMap tma_k;  // {D, seq_k, heads, batch}, box {32, 128}
  CUtensorMap tma_v;  // {D, seq_k, heads, batch}, box {32, 32}, 32-byte-atom swizzle
  float* out;
  int64_t o_sb, o_sh, o_ss;  // output element strides (last dimension contiguous)
  float* lse;                // [batch, heads, seq_q] or null
  int heads, seq_q, seq_k;
  float scale_log2;          // softmax scale * log2(e)
  int causal;
  int* status;
};

// N-major V operand: 32-wide atoms (of the head dimension) [32 keys x 128 B]
// placed V_KB/2 bytes apart within a k-block; 32-byte chunks swizzled over
// 4 rows, so K groups of 4 keys are 512 B apart.
__device__ __forceinline__ uint64_t desc_v(uint32_t saddr) {
  return make_desc(saddr, 32 * 128, 512, 1);
}

// 2^x with the MUFU approximation (ex2.approx.ftz: about 2 ulp, flushes
// subnormal results to 0, ex2(-inf) = 0), well inside the TF32 tolerance
// of the attention output.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void st_shared4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

__global__ void __launch_bounds__(THREADS, 1) attn_fwd_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_abort;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t sq = base;
  const uint32_t sk = sq + Q_BYTES;                  // [STAGES][K_BYTES]
  const uint32_t sv = sk + STAGES * K_BYTES;         // [STAGES][V_BYTES]
  const uint32_t sp = sv + STAGES * V_BYTES;         // P tile
  // mbarriers, one 8-byte slot each
  const uint32_t bar = sp + P_BYTES;
  const uint32_t q_full = bar;              // slot 0
  const uint32_t k_full = bar + 8;          // slots 1-2, one per stage
  const uint32_t k_empty = bar + 24;        // slots 3-4
  const uint32_t v_full = bar + 40;         // slots 5-6
  const uint32_t v_empty = bar + 56;        // slots 7-8
  const uint32_t s_full = bar + 72;         // slots 9-10, one per score buffer
  const uint32_t s_empty = bar + 88;        // slots 11-12
  const uint32_t p_full = bar + 104;        // slot 13
  const uint32_t pv_full = bar + 112;       // slot 14
  const uint32_t pv_empty = bar + 120;      // slot 15
  __shared__ uint64_t s_drain;
  __shared__ uint32_t s_tmem;
  const uint32_t drain = smem_u32(&s_drain);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const volatile int* abort_flag = &s_abort;
  const int bh = blockIdx.y;
  const int b = bh / p.heads;
  const int h = bh - b * p.heads;
  const int qt = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);  // heavy tiles first
  const int q0 = qt * BM;
  const int kblocks = (p.seq_k + BN - 1) / BN;
  const int nkb = p.causal ? min(kblocks, (min(q0 + BM, p.seq_q) - 1) / BN + 1) : kblocks;

  if (threadIdx.x == 0) {
    s_abort = 0;
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(k_full + 8 * s, 1);
      mbar_init(k_empty + 8 * s, 1);
      mbar_init(v_full + 8 * s, 1);
      mbar_init(v_empty + 8 * s, 1);
      mbar_init(s_full + 8 * s, 1);
      mbar_init(s_empty + 8 * s, 4);
    }
    mbar_init(p_full, 4);
    mbar_init(pv_full, 1);
    mbar_init(pv_empty, 4);
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s_tmem)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(&s_tmem);

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      bool ok = true;
      uint32_t k_issued = 0, v_issued = 0, k_par = 0, v_par = 0;
      mbar_expect_tx(q_full, Q_BYTES);
      for (int a = 0; a < D / 32; ++a) tma_load_4d(sq + a * ATOM, &p.tma_q, q_full, 32 * a, q0, h, b);
      for (int j = 0; ok && j < nkb; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(k_empty + 8 * st, ph ^ 1u, abort_flag)) { ok = false; break; }
        mbar_expect_tx(k_full + 8 * st, K_BYTES);
        for (int a = 0; a < D / 32; ++a)
          tma_load_4d(sk + st * K_BYTES + a * ATOM, &p.tma_k, k_full + 8 * st, 32 * a, j * BN, h, b);
        k_issued |= 1u << st;
        k_par = (k_par & ~(1u << st)) | (ph << st);
        if (!mbar_wait(v_empty + 8 * st, ph ^ 1u, abort_flag)) { ok = false; break; }
        mbar_expect_tx(v_full + 8 * st, V_BYTES);
        for (int kb = 0; kb < BN / 32; ++kb)
          for (int a = 0; a < D / 32; ++a)
            tma_load_4d(sv + st * V_BYTES + kb * V_KB_BYTES + a * (32 * 128), &p.tma_v,
                        v_full + 8 * st, 32 * a, j * BN + 32 * kb, h, b);
        v_issued |= 1u << st;
        v_par = (v_par & ~(1u << st)) | (ph << st);
      }
      if (!ok) {
        record_status(p.status, TVR_DEV_TIMEOUT_PRODUCER);
        *const_cast<volatile int*>(abort_flag) = 1;
      }
      // every issued load lands before the CTA may exit
      if (!mbar_wait(q_full, 0, nullptr)) record_status(p.status, TVR_DEV_TIMEOUT_DRAIN);
      for (int st = 0; st < 2; ++st) {
        if ((k_issued >> st) & 1u)
          if (!mbar_wait(k_full + 8 * st, (k_par >> st) & 1u, nullptr)) record_status(p.status, TVR_DEV_TIMEOUT_DRAIN);
        if ((v_issued >> st) & 1u)
          if (!mbar_wait(v_full + 8 * st, (v_par >> st) & 1u, nullptr)) record_status(p.status, TVR_DEV_TIMEOUT_DRAIN);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_tf32(BM, BN, false);
      constexpr uint32_t idesc_pv = idesc_tf32(BM, D, true);
      bool ok = mbar_wait(q_full, 0, abort_flag);
      bool issued = false;
      // S_i = Q K_i^T into score buffer i & 1
      auto issue_s = [&](int i) -> bool {
        const int st = i & 1;
        if (!mbar_wait(k_full + 8 * st, (i >> 1) & 1, abort_flag)) return false;
        if (i >= 2 && !mbar_wait(s_empty + 8 * st, ((i >> 1) - 1) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(st * BN);
#pragma unroll
        for (int x = 0; x < D / 8; ++x) {
          const uint32_t off = (x >> 2) * ATOM + (x & 3) * 32;
          mma_tf32(d, desc_kmajor(sq + off), desc_kmajor(sk + st * K_BYTES + off), idesc_s,
                   x > 0 ? 1u : 0u);
        }
        mma_commit(k_empty + 8 * st);
        mma_commit(s_full + 8 * st);
        return true;
      };
      if (ok && nkb > 0) {
        ok = issue_s(0);
        issued = ok;
      }
      for (int j = 0; ok && j < nkb; ++j) {
        if (j + 1 < nkb && !(ok = issue_s(j + 1))) break;
        // PV_j = P_j V_j
        const int st = j & 1;
        if (!mbar_wait(p_full, j & 1, abort_flag) ||
            !mbar_wait(v_full + 8 * st, (j >> 1) & 1, abort_flag) ||
            (j >= 1 && !mbar_wait(pv_empty, (j - 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int x = 0; x < BN / 8; ++x) {
          const int kb = x >> 2, kk = x & 3;
          mma_tf32(tmem + PV_COL, desc_kmajor(sp + kb * ATOM + kk * 32),
                   desc_v(sv + st * V_BYTES + kb * V_KB_BYTES + kk * 1024), idesc_pv,
                   x > 0 ? 1u : 0u);
        }
        mma_commit(v_empty + 8 * st);
        mma_commit(pv_full);
      }
      if (!ok) {
        record_status(p.status, TVR_DEV_TIMEOUT_MMA);
        *const_cast<volatile int*>(abort_flag) = 1;
      }
      if (issued) {
        mma_commit(drain);
        if (!mbar_wait(drain, 0, nullptr)) record_status(p.status, TVR_DEV_TIMEOUT_DRAIN);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------ softmax rows ------------------------------
    const int q = warp & 3;
    const int t = 32 * q + lane;  // TMEM lane = query row within the tile
    const int qidx = q0 + t;
    const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
    float o[D];
#pragma unroll
    for (int i = 0; i < D; ++i) o[i] = 0.f;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      const int sb = j & 1;
      const bool got = mbar_wait(s_full + 8 * sb, (j >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t srow = tmem + lane_off + static_cast<uint32_t>(sb * BN);
      const int key0 = j * BN;
      // keys [key0, key_end) are visible to this row
      int key_end = min(p.seq_k, key0 + BN);
      if (p.causal) key_end = min(key_end, qidx + 1);
      const int nvis = key_end - key0;  // may be <= 0 for padding rows
      // the row's 128 scores: four TMEM loads in flight, one wait
      float sc[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_load_32_async(srow + 32 * c, sc + 32 * c);
      tmem_wait_loads();
      // scores consumed: the buffer may take S_{j+2}
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_empty + 8 * sb);
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < BN; ++i) {
        if (i < nvis) mx = fmaxf(mx, sc[i] * p.scale_log2);
      }
      // scores are scaled inside exp2: x * scale_log2 - m in one FMA
      const float m_new = fmaxf(m, mx);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = ex2(m - m_use);
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < BN; ++i) {
        const float e = i < nvis ? ex2(fmaf(sc[i], p.scale_log2, -m_use)) : 0.f;
        sc[i] = e;
        sum += e;
      }
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        const uint32_t row = sp + c * ATOM + t * 128;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          const float* q4 = sc + 32 * c + 4 * cc;
          st_shared4(row + ((cc ^ (t & 7)) << 4), q4[0], q4[1], q4[2], q4[3]);
        }
      }
      // P visible to the tensor core
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      l = l * alpha + sum;
      m = m_new;
      const bool got_pv = mbar_wait(pv_full, j & 1, abort_flag);
      if (!__all_sync(0xffffffffu, got_pv)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float pv[D];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) tmem_load_32_async(tmem + lane_off + PV_COL + 32 * c, pv + 32 * c);
      tmem_wait_loads();
#pragma unroll
      for (int i = 0; i < D; ++i) o[i] = fmaf(o[i], alpha, pv[i]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pv_empty);
    }
    if (!ok) {
      if (lane == 0) {
        record_status(p.status, TVR_DEV_TIMEOUT_EPILOGUE);
        *const_cast<volatile int*>(abort_flag) = 1;
      }
    } else if (qidx < p.seq_q) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      float* dst = p.out + b * p.o_sb + h * p.o_sh + static_cast<int64_t>(qidx) * p.o_ss;
      if ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
#pragma unroll
        for (int i = 0; i < D / 4; ++i) {
          reinterpret_cast<float4*>(dst)[i] =
              make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv, o[4 * i + 3] * inv);
        }
      } else {
#pragma unroll
        for (int i = 0; i < D; ++i) dst[i] = o[i] * inv;
      }
      if (p.lse != nullptr) {
        p.lse[(static_cast<int64_t>(b) * p.heads + h) * p.seq_q + qidx] =
            m * 0.69314718055994531f + logf(l);
      }
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                 : "memory");
  }
}

}  // namespace attn
}  // namespace tvr

using namespace tvr;

extern "C" int tvr_attention_fwd(const float* q, const float* k, const float* v, float* out,
                                 float* lse, int64_t batch, int64_t heads, int64_t seq_q,
                                 int64_t seq_k, int64_t head_dim, const int64_t* q_strides,
                                 const int64_t* k_strides, const int64_t* v_strides,
                                 const int64_t* o_strides, float scale, int causal, int mode,
                                 void* stream) {
  using namespace attn;
  TVR_CHECK(batch >= 0 && heads >= 0 && seq_q >= 0 && seq_k >= 0, "attention: negative size");
  if (batch == 0 || heads == 0 || seq_q == 0) return TVR_OK;
  TVR_CHECK(q && k && v && out && q_strides && k_strides && v_strides && o_strides,
            "attention: null pointer");
  TVR_CHECK(seq_k >= 1, "attention: no keys");
  if (head_dim != D) {
    return fail(TVR_ERR_UNSUPPORTED, "attention: head dimension %lld (the fused kernel takes %d)",
                (long long)head_dim, D);
  }
  if (mode == TVR_GEMM_AUTO) {
    const char* env = std::getenv("TVARANT_GEMM_MODE");
    mode = (env != nullptr && std::strcmp(env, "tf32") == 0) ? TVR_GEMM_TF32 : TVR_GEMM_3XTF32;
  }
  if (mode != TVR_GEMM_TF32) {
    return fail(TVR_ERR_UNSUPPORTED, "attention: the fused kernel computes in TF32 only");
  }
  TVR_CHECK(batch * heads <= 65535 && seq_q <= 0x7fffff00 && seq_k <= 0x7fffff00,
            "attention: too many (batch, head) pairs or positions");
  auto strides_ok = [](const float* ptr, const int64_t* s) {
    return tc::al16(ptr) && s[0] % 4 == 0 && s[1] % 4 == 0 && s[2] % 4 == 0 && s[0] > 0 &&
           s[1] > 0 && s[2] > 0;
  };
  if (!strides_ok(q, q_strides) || !strides_ok(k, k_strides) || !strides_ok(v, v_strides)) {
    return fail(TVR_ERR_UNSUPPORTED,
                "attention: operands need 16-byte aligned bases and strides that are multiples "
                "of 4 elements (TMA)");
  }
  const int dev = current_device();
  Params p;
  memset(&p, 0, sizeof(p));
  int rc;
  auto enc = [&](CUtensorMap* map, const float* ptr, int64_t seq, const int64_t* s, uint32_t box1,
                 CUtensorMapSwizzle sw) {
    const uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(seq),
                              static_cast<uint64_t>(heads), static_cast<uint64_t>(batch)};
    const uint64_t st[3] = {static_cast<uint64_t>(s[2]) * 4, static_cast<uint64_t>(s[1]) * 4,
                            static_cast<uint64_t>(s[0]) * 4};
    return tc::encode_4d(map, ptr, dims, st, 32, box1, sw);
  };
  if ((rc = enc(&p.tma_q, q, seq_q, q_strides, BM, CU_TENSOR_MAP_SWIZZLE_128B)) != TVR_OK) return rc;
  if ((rc = enc(&p.tma_k, k, seq_k, k_strides, BN, CU_TENSOR_MAP_SWIZZLE_128B)) != TVR_OK) return rc;
  if ((rc = enc(&p.tma_v, v, seq_k, v_strides, 32, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)) != TVR_OK)
    return rc;
  p.out = out;
  p.o_sb = o_strides[0];
  p.o_sh = o_strides[1];
  p.o_ss = o_strides[2];
  p.lse = lse;
  p.heads = static_cast<int>(heads);
  p.seq_q = static_cast<int>(seq_q);
  p.seq_k = static_cast<int>(seq_k);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal ? 1 : 0;
  p.status = device_status_ptr(dev);
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  std::call_once(once[dev & 63], [&]() {
    attr_err[dev & 63] = cudaFuncSetAttribute(attn_fwd_kernel,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              SMEM_BYTES);
  });
  TVR_CUDA_TRY(attr_err[dev & 63]);
  const dim3 grid(static_cast<unsigned>(ceil_div(seq_q, BM)), static_cast<unsigned>(batch * heads));
  attn_fwd_kernel<<<grid, THREADS, SMEM_BYTES, as_stream(stream)>>>(p);
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

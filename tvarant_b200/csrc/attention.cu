// Fused causal / full attention forward for sm_100a (tcgen05 kind::tf32):
// out = softmax(scale * Q K^T [+ causal mask]) V without materialising the
// [seq_q, seq_k] scores.  The reference has no fused attention — its models
// run bmm -> add(mask) -> softmax -> bmm (csrc/aten/LlmOps.cpp:68-148) and
// the fused kernel is a roadmap item — so this kernel serves
// F.scaled_dot_product_attention on the tvarant device (TF32 mode).
//
// Persistent: two CTAs per SM, each working through its share of the units
// (a unit is one 128-query tile of one (batch, head)), heaviest first in a
// snake order over the CTAs.  Tensor memory, barriers and their phases carry
// over from one unit to the next.  (With one CTA per unit the block
// scheduler refilled an SM only once both of its CTAs had exited, so under
// the causal mask, where tiles differ in length up to 16x, an SM ran one CTA
// for much of the time.)  Head dimension 64.
//   warp 0     TMA producer: lane 0 loads each unit's Q tile and the K and V
//              tiles of each block of 64 keys (two buffers each), straight
//              from strided [B, H, S, 64] views (no head-split copies), with
//              an L2 prefetch two blocks ahead;
//   warp 1     TMEM owner; lane 0 issues every MMA in a fixed order:
//              PV_j = P_j V_j (M=128, N=64, K=64) as soon as P_j is written,
//              then S_{j+3} = Q K_{j+3}^T (M=128, N=64, K=64) into the TMEM
//              score buffer PV_j has just read, so the scores run three
//              blocks ahead of the softmax; P_j is read from tensor memory,
//              V as an N-major operand, and O accumulates in tensor memory;
//   warps 2-5  one thread per query row: online softmax in the log2 domain
//              over the row's 64 scores of a block (two TMEM loads in flight,
//              one wait), P_j written back over S_j in tensor memory.  The
//              running maximum is raised lazily (only when a block's maximum
//              exceeds it by more than 2^8), and only then are the warp's rows
//              of O rescaled in tensor memory; O / l does not depend on which
//              maximum was used.  At the end of a unit O / l is stored
//              and the log-sum-exp (natural log) is written.
// Without P tiles in shared memory a CTA needs 97 KB, so two CTAs share an SM
// and each SM scheduler holds two softmax warps.
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
constexpr int BN = 64;                   // keys per block
constexpr int Q_ATOM = BM * 128;         // [128 query rows x 128 B] swizzle block
constexpr int K_ATOM = BN * 128;         // [64 key rows x 128 B]
constexpr int Q_BYTES = BM * D * 4;      // D/32 atoms
constexpr int K_BYTES = BN * D * 4;      // D/32 atoms
constexpr int V_ATOM = BN * 128;         // one 32-wide slice of the head dimension: [64 keys x 128 B]
constexpr int V_BYTES = BN * D * 4;      // D/32 atoms
constexpr int STAGES = 2;                // K and V tiles are double-buffered
constexpr int SBUF = 3;                  // TMEM score / P buffers: S runs this many blocks ahead of PV
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 256;      // S / P buffers at 0, 64 and 128, O at 192
constexpr uint32_t PV_COL = SBUF * BN;
constexpr float kLazyLog2 = 8.f;         // raise the running maximum past 2^8 growth
constexpr int BAR_BYTES = 8 * 24;
constexpr int SMEM_BYTES = 1024 + Q_BYTES + STAGES * (K_BYTES + V_BYTES) + BAR_BYTES;
static_assert(2 * (SMEM_BYTES + 1024 + 64) <= 233472, "two CTAs per SM");

struct Params {
  CUtensorMap tma_q;  // {D, seq_q, heads, batch}, box {32, 128}
  CUtensorMap tma_k;  // {D, seq_k, heads, batch}, box {32, 64}
  CUtensorMap tma_v;  // {D, seq_k, heads, batch}, box {32, 64}, 32-byte-atom swizzle
  float* out;
  int64_t o_sb, o_sh, o_ss;  // output element strides (last dimension contiguous)
  float* lse;                // [batch, heads, seq_q] or null
  int heads, seq_q, seq_k;
  float scale_log2;          // softmax scale * log2(e)
  int causal;
  int* status;
  const int64_t* key_len;    // non-null: attend to clamp(*key_len + key_len_add, 1, seq_k) keys
  int key_len_add;
  int batch_heads;           // batch * heads
  int nqt;                   // query tiles per (batch, head)
  int units;                 // nqt * batch_heads
};

// One unit of work: a 128-query tile of one (batch, head).
struct Tile {
  int b, h, q0, nkb;
};

// The n-th unit of this CTA, or -1.  Units are numbered heaviest first (under
// the causal mask the last query tiles see the most keys); CTA c takes unit c
// of the first round of gridDim.x units, unit gridDim.x - 1 - c of the
// second, and so on (a snake order), which evens out the CTAs' total work.
__device__ __forceinline__ int cta_unit(int n, int units) {
  const long long ctas = gridDim.x;
  const long long c = blockIdx.x;
  const long long idx = n * ctas + ((n & 1) ? ctas - 1 - c : c);
  return idx < units ? static_cast<int>(idx) : -1;
}

__device__ __forceinline__ Tile tile_of(const Params& p, int idx, int kblocks) {
  const int rank = idx / p.batch_heads;
  const int bh = idx - rank * p.batch_heads;
  Tile t;
  t.b = bh / p.heads;
  t.h = bh - t.b * p.heads;
  t.q0 = (p.nqt - 1 - rank) * BM;
  t.nkb = p.causal ? min(kblocks, (min(t.q0 + BM, p.seq_q) - 1) / BN + 1) : kblocks;
  return t;
}

// Walks this CTA's key blocks in order: block j of its unit n.  Every role
// keeps one, so the barrier phases run on across units.
struct BlockCursor {
  int n, idx, j;
  Tile t;
  __device__ __forceinline__ void start(const Params& p, int kblocks) {
    n = 0;
    j = 0;
    idx = cta_unit(0, p.units);
    if (idx >= 0) t = tile_of(p, idx, kblocks);
  }
  __device__ __forceinline__ bool valid() const { return idx >= 0; }
  __device__ __forceinline__ bool last_of_unit() const { return j == t.nkb - 1; }
  __device__ __forceinline__ void advance(const Params& p, int kblocks) {
    if (++j == t.nkb) {
      j = 0;
      idx = cta_unit(++n, p.units);
      if (idx >= 0) t = tile_of(p, idx, kblocks);
    }
  }
};

// N-major V operand: 32-wide atoms of the head dimension, each [64 keys x
// 128 B] and V_ATOM bytes apart (leading offset); 32-byte chunks swizzled
// over 4 rows, so K groups of 4 keys are 512 B apart (stride offset).
__device__ __forceinline__ uint64_t desc_v(uint32_t saddr) {
  return make_desc(saddr, V_ATOM, 512, 1);
}

// 2^x with the MUFU approximation (ex2.approx.ftz: about 2 ulp, flushes
// subnormal results to 0, ex2(-inf) = 0), well inside the TF32 tolerance
// of the attention output.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Row qidx of the output (O / l) and its log-sum-exp (natural log), from the
// unnormalised O and the log2-domain running maximum m and sum l.
__device__ __forceinline__ void store_row(const Params& p, int b, int h, int qidx, const float* o,
                                          float m, float l) {
  const float inv = l > 0.f ? 1.f / l : 0.f;
  float* dst = p.out + b * p.o_sb + h * p.o_sh + static_cast<int64_t>(qidx) * p.o_ss;
  if ((reinterpret_cast<uintptr_t>(dst) & 31u) == 0) {
    // 32-byte stores: every lane of a warp writes a different row, so each
    // store instruction touches 32 rows; whole sectors halve the instructions
    // and leave no partly written sector
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const float* v = o + 8 * i;
      asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst + 8 * i),
                   "f"(v[0] * inv), "f"(v[1] * inv), "f"(v[2] * inv), "f"(v[3] * inv),
                   "f"(v[4] * inv), "f"(v[5] * inv), "f"(v[6] * inv), "f"(v[7] * inv)
                   : "memory");
    }
  } else if ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
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

__global__ void __launch_bounds__(THREADS, 2) attn_fwd_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_abort;
  __shared__ uint64_t s_drain;
  __shared__ uint32_t s_tmem;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t sq = base;
  const uint32_t sk = sq + Q_BYTES;                 // [2] K tiles
  const uint32_t sv = sk + STAGES * K_BYTES;        // [2] V tiles
  // mbarriers, one 8-byte slot each; [2] = one per buffer
  const uint32_t bar = sv + STAGES * V_BYTES;
  // One commit per MMA block: s_done (the scores of block g are in buffer
  // g % 3 and K buffer g & 1 is free) and pv_done (the P of block g has been
  // read, so its score buffer and V buffer g & 1 are free, and O holds it).
  const uint32_t q_full = bar;
  const uint32_t k_full = bar + 8;       // [2]
  const uint32_t v_full = bar + 24;      // [2]
  const uint32_t s_done = bar + 40;      // [3] one per score buffer
  const uint32_t p_full = bar + 64;      // [3]
  const uint32_t pv_done = bar + 88;     // [3]
  const uint32_t q_empty = bar + 112;    // every S of a unit read its Q tile
  const uint32_t drain = smem_u32(&s_drain);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const volatile int* abort_flag = &s_abort;
  // the key count: the buffers' extent, or a length held in device memory
  // (written by earlier work on the stream, e.g. a KV cache's fill level)
  const int seq_k = p.key_len != nullptr
                        ? max(1, min(p.seq_k, static_cast<int>(*p.key_len) + p.key_len_add))
                        : p.seq_k;
  const int kblocks = (seq_k + BN - 1) / BN;

  if (threadIdx.x == 0) {
    s_abort = 0;
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(k_full + 8 * i, 1);
      mbar_init(v_full + 8 * i, 1);
    }
    for (int i = 0; i < SBUF; ++i) {
      mbar_init(s_done + 8 * i, 1);
      mbar_init(p_full + 8 * i, 4);
      mbar_init(pv_done + 8 * i, 1);
    }
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
  // a few-row GEMM launched as a programmatic dependent (the projection after
  // a decode step's attention) may start streaming its weights now
  if (threadIdx.x == 0) grid_launch_dependents();

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    // One thread.  It replays the MMA thread's order (S of this CTA's blocks
    // 0, 1 and 2, then per block g: PV_g, S_{g+3}) and after each MMA loads what
    // that MMA frees: after S_g the K tile of block g + 2 (preceded by the
    // next unit's Q tile when block g ends a unit), after PV_g the V tile of
    // block g + 2.  The loads go out in the order in which their buffers
    // free up; two producer lanes of one warp took turns in their barrier
    // waits.  Every K and V tile is also prefetched into L2 two blocks before
    // its load: the query tiles of a head read each tile at about the same
    // time, so its first reads come from HBM.
    if (lane == 0) {
      bool ok = true;
      int gk = 0, gv = 0, nq = 0;  // K, V and Q tiles loaded
      BlockCursor sc, pc, kc, vc;  // S and PV replay, next K and V tile
      sc.start(p, kblocks);
      pc = sc;
      kc = sc;
      vc = sc;
      // Q of unit nq once every S of unit nq - 1 has read the buffer
      auto load_q = [&](const Tile& t) -> bool {
        if (nq >= 1 && !mbar_wait(q_empty, (nq - 1) & 1, abort_flag)) return false;
        mbar_expect_tx(q_full, Q_BYTES);
        for (int a = 0; a < D / 32; ++a) tma_load_4d(sq + a * Q_ATOM, &p.tma_q, q_full, 32 * a, t.q0, t.h, t.b);
        ++nq;
        return true;
      };
      // kc's K tile into K buffer gk & 1 once S of block gk - 2 has read it
      auto load_k = [&]() -> bool {
        const int st = gk & 1;
        if (gk >= STAGES && !mbar_wait(s_done + 8 * ((gk - 2) % SBUF), ((gk - 2) / SBUF) & 1, abort_flag)) {
          return false;
        }
        const uint32_t fb = k_full + 8 * st;
        mbar_expect_tx(fb, K_BYTES);
        for (int a = 0; a < D / 32; ++a)
          tma_load_4d(sk + st * K_BYTES + a * K_ATOM, &p.tma_k, fb, 32 * a, kc.j * BN, kc.t.h, kc.t.b);
        ++gk;
        BlockCursor ahead = kc;
        ahead.advance(p, kblocks);
        ahead.advance(p, kblocks);
        if (ahead.valid()) {
          for (int a = 0; a < D / 32; ++a) {
            tma_prefetch_l2_4d(&p.tma_k, 32 * a, ahead.j * BN, ahead.t.h, ahead.t.b);
            tma_prefetch_l2_4d(&p.tma_v, 32 * a, ahead.j * BN, ahead.t.h, ahead.t.b);
          }
        }
        kc.advance(p, kblocks);
        return true;
      };
      // vc's V tile into V buffer gv & 1 once PV of block gv - 2 has read it
      auto load_v = [&]() -> bool {
        const int st = gv & 1;
        if (gv >= STAGES && !mbar_wait(pv_done + 8 * ((gv - 2) % SBUF), ((gv - 2) / SBUF) & 1, abort_flag)) {
          return false;
        }
        const uint32_t fb = v_full + 8 * st;
        mbar_expect_tx(fb, V_BYTES);
        for (int a = 0; a < D / 32; ++a)
          tma_load_4d(sv + st * V_BYTES + a * V_ATOM, &p.tma_v, fb, 32 * a, vc.j * BN, vc.t.h, vc.t.b);
        ++gv;
        vc.advance(p, kblocks);
        return true;
      };
      // S of sc's block issued: the next unit's Q after a unit's last block,
      // then the K tile two blocks on
      auto after_s = [&]() -> bool {
        if (sc.last_of_unit()) {
          BlockCursor next = sc;
          next.advance(p, kblocks);
          if (next.valid() && !load_q(next.t)) return false;
        }
        if (kc.valid() && !load_k()) return false;
        sc.advance(p, kblocks);
        return true;
      };
      if (sc.valid()) {
        ok = load_q(sc.t);
        for (int i = 0; ok && i < STAGES && kc.valid(); ++i) ok = load_k();
        for (int i = 0; ok && i < STAGES && vc.valid(); ++i) ok = load_v();
        for (int i = 0; ok && i < SBUF && sc.valid(); ++i) ok = after_s();
        while (ok && pc.valid()) {
          if (vc.valid()) ok = load_v();
          pc.advance(p, kblocks);
          if (ok && sc.valid()) ok = after_s();
        }
      }
      if (!ok) {
        record_status(p.status, TVR_DEV_TIMEOUT_PRODUCER);
        *const_cast<volatile int*>(abort_flag) = 1;
      }
      // every issued load lands before the CTA may exit
      if (nq > 0 && !mbar_wait(q_full, (nq - 1) & 1, nullptr)) record_status(p.status, TVR_DEV_TIMEOUT_DRAIN);
      for (int g = max(0, gk - STAGES); g < gk; ++g) {
        if (!mbar_wait(k_full + 8 * (g & 1), (g >> 1) & 1, nullptr)) record_status(p.status, TVR_DEV_TIMEOUT_DRAIN);
      }
      for (int g = max(0, gv - STAGES); g < gv; ++g) {
        if (!mbar_wait(v_full + 8 * (g & 1), (g >> 1) & 1, nullptr)) record_status(p.status, TVR_DEV_TIMEOUT_DRAIN);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    // One thread, one fixed order over this CTA's key blocks (all its units
    // in turn): S of blocks 0, 1 and 2, then for each block g the product
    // PV_g (once P_g and V_g are in place) followed by S_{g+3} into score
    // buffer g % 3 as soon as PV_g has read the P there.  The scores run
    // three blocks ahead of the softmax, across units too, so a softmax warp
    // finds the next block's scores done when it finishes one: the thread is
    // held to the tensor core's pace while it issues (the MMA queue is
    // shallow), and scores issued only two blocks ahead, behind PV_g, came
    // ~0.6 us late per block.  (Two issuing lanes of one warp took turns in
    // their barrier waits and delayed each PV by ~0.7 us.)  The drain commit
    // at the end arrives once every MMA retired.
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_tf32(BM, BN, false);
      constexpr uint32_t idesc_pv = idesc_tf32(BM, D, true);
      BlockCursor sc, pc;
      sc.start(p, kblocks);
      pc = sc;
      int gs = 0, gp = 0;  // S and PV issued
      auto issue_s = [&]() -> bool {
        const int sb = gs % SBUF;
        const int kb = gs & 1;
        if ((sc.j == 0 && !mbar_wait(q_full, sc.n & 1, abort_flag)) ||
            !mbar_wait(k_full + 8 * kb, (gs >> 1) & 1, abort_flag) ||
            (gs >= SBUF && !mbar_wait(pv_done + 8 * sb, (gs / SBUF - 1) & 1, abort_flag))) {
          return false;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(sb * BN);
#pragma unroll
        for (int x = 0; x < D / 8; ++x) {
          const uint32_t k32 = (x & 3) * 32;
          mma_tf32(d, desc_kmajor(sq + (x >> 2) * Q_ATOM + k32),
                   desc_kmajor(sk + kb * K_BYTES + (x >> 2) * K_ATOM + k32), idesc_s,
                   x > 0 ? 1u : 0u);
        }
        mma_commit(s_done + 8 * sb);
        if (sc.last_of_unit()) mma_commit(q_empty);  // the unit's scores have read Q
        ++gs;
        sc.advance(p, kblocks);
        return true;
      };
      bool ok = true;
      for (int i = 0; ok && i < SBUF && sc.valid(); ++i) ok = issue_s();
      while (ok && pc.valid()) {
        const int pb = gp % SBUF;
        const int vb = gp & 1;
        if (!mbar_wait(p_full + 8 * pb, (gp / SBUF) & 1, abort_flag) ||
            !mbar_wait(v_full + 8 * vb, (gp >> 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // P sits in score buffer gp % 3 (K step x: its columns 8x .. 8x+7);
        // O accumulates in place over the unit's blocks (its first block
        // overwrites it)
        const uint32_t pa = tmem + static_cast<uint32_t>(pb * BN);
#pragma unroll
        for (int x = 0; x < BN / 8; ++x) {
          mma_tf32_tmem_a(tmem + PV_COL, pa + 8u * x, desc_v(sv + vb * V_BYTES + x * 1024),
                          idesc_pv, (pc.j > 0 || x > 0) ? 1u : 0u);
        }
        mma_commit(pv_done + 8 * pb);  // P read: the buffer may take the scores of block gp + 3
        ++gp;
        pc.advance(p, kblocks);
        if (sc.valid()) ok = issue_s();
      }
      if (!ok) {
        record_status(p.status, TVR_DEV_TIMEOUT_MMA);
        *const_cast<volatile int*>(abort_flag) = 1;
      }
      // arrives once every MMA this thread issued has retired (at once if none)
      mma_commit(drain);
    }
    __syncwarp();
    if (lane == 0 && !mbar_wait(drain, 0, nullptr)) record_status(p.status, TVR_DEV_TIMEOUT_DRAIN);
    __syncwarp();
  } else {
    // ------------------- softmax rows, P and O in tensor memory -------------------
    // O accumulates in TMEM (PV adds P V to it).  O and l are kept relative
    // to a running maximum m that is raised only when a block's maximum
    // exceeds it by more than 2^kLazyLog2, or at the first visible scores;
    // then the warp rescales its rows of O (a TMEM round trip after the
    // previous block's PV has landed).  Between raises P = 2^(x - m) <=
    // 2^kLazyLog2, far from the fp32 range, and O / l is unchanged by the
    // choice of m.  At the end of a unit O / l is stored; the unit's first PV
    // is issued only after these threads have written the next unit's first
    // P, so it cannot overwrite O before it is read.
    const int q = warp & 3;
    const int tr = 32 * q + lane;  // TMEM lane = query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
    const uint32_t orow = tmem + lane_off + PV_COL;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    // PV of block g done: completion g / 3 of pv_done[g % 3]
    auto wait_pv = [&](int g) -> bool {
      const bool got = mbar_wait(pv_done + 8 * (g % SBUF), (g / SBUF) & 1, abort_flag);
      return __all_sync(0xffffffffu, got);
    };
    // One block of this row: raise m if needed (rescaling O), write P over S
    // and add its sum to l.  Columns the row does not see hold -inf (set by
    // the caller), so one body serves every block: exp2 maps them to 0 and the
    // maximum passes over them.  (Two unrolled copies, for whole and partly
    // masked blocks, left the softmax warps waiting on instruction fetch.)
    auto row_block = [&](float* sc, bool first, int g, uint32_t srow) -> bool {
      // the block maximum of the scaled scores from the raw ones (scaling by
      // s > 0 keeps their order, and rounding is monotone), in eight
      // independent partial maxima (and sums below): a single chain of 64
      // dependent operations would be the row's critical path
      float mp[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) mp[r] = -INFINITY;
#pragma unroll
      for (int i = 0; i < BN; ++i) mp[i & 7] = fmaxf(mp[i & 7], sc[i]);
      const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7]))) *
                       p.scale_log2;
      const float m_new = fmaxf(m, mx);
      if (__any_sync(0xffffffffu, m_new > m + kLazyLog2)) {
        const float alpha = ex2(m - (m_new == -INFINITY ? 0.f : m_new));  // 0 while m = -inf
        if (!first) {
          if (!wait_pv(g - 1)) return false;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            float ov[32];
            tmem_load_32_async(orow + 32 * c, ov);
            tmem_wait_loads();
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] *= alpha;
            tmem_store_32(orow + 32 * c, ov);
          }
        }
        l *= alpha;
        m = m_new;
      }
      const float m_use = m == -INFINITY ? 0.f : m;
      // P over S in this row's lane, each 32-column half stored as soon as it
      // is computed; PV reads it from there.  The wait also covers the O
      // rescale above.
      float sp[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) sp[r] = 0.f;
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
#pragma unroll
        for (int i = 32 * c; i < 32 * c + 32; ++i) {
          const float e = ex2(fmaf(sc[i], p.scale_log2, -m_use));
          sc[i] = e;
          sp[i & 7] += e;
        }
        tmem_store_32(srow + 32 * c, sc + 32 * c);
      }
      l += ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
      tmem_wait_stores();
      return true;
    };
    int g = 0;  // this CTA's key blocks so far, over all its units
    for (int n = 0; ok; ++n) {
      const int idx = cta_unit(n, p.units);
      if (idx < 0) break;
      const Tile t = tile_of(p, idx, kblocks);
      const int qidx = t.q0 + tr;
      m = -INFINITY;
      l = 0.f;
      for (int j = 0; j < t.nkb; ++j, ++g) {
        const int sb = g % SBUF;
        const bool got = mbar_wait(s_done + 8 * sb, (g / SBUF) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        // S_g was issued after PV_{g-3} had read buffer g % 3, so this
        // returns at once; it keeps the thread's view of each pv_done barrier
        // within one phase of its state, which the parity waits for PV_{g-1}
        // and at the end of a unit rely on
        if (g >= SBUF && !wait_pv(g - SBUF)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t srow = tmem + lane_off + static_cast<uint32_t>(sb * BN);
        const int key0 = j * BN;
        int key_end = min(seq_k, key0 + BN);
        if (p.causal) key_end = min(key_end, qidx + 1);
        const int nvis = key_end - key0;  // may be <= 0 for padding rows
        float sc[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_load_32_async(srow + 32 * c, sc + 32 * c);
        tmem_wait_loads();
        if (!__all_sync(0xffffffffu, nvis >= BN)) {
#pragma unroll
          for (int i = 0; i < BN; ++i) sc[i] = i < nvis ? sc[i] : -INFINITY;
        }
        const bool done = row_block(sc, j == 0, g, srow);
        if (!done) {
          ok = false;
          break;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full + 8 * sb);
      }
      // the unit's last PV (t.nkb >= 1: key 0 is always visible)
      if (!ok || !wait_pv(g - 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float o[D];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) tmem_load_32_async(orow + 32 * c, o + 32 * c);
      tmem_wait_loads();
      if (qidx < p.seq_q) store_row(p, t.b, t.h, qidx, o, m, l);
    }
    if (!ok && lane == 0) {
      record_status(p.status, TVR_DEV_TIMEOUT_EPILOGUE);
      *const_cast<volatile int*>(abort_flag) = 1;
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

namespace {

int attention_impl(const float* q, const float* k, const float* v, float* out, float* lse,
                   int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_k, int64_t head_dim,
                   const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                   const int64_t* o_strides, float scale, int causal, int mode,
                   const int64_t* key_len, int key_len_add, void* stream) {
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
  if (!(scale > 0.f) || !std::isfinite(scale)) {
    return fail(TVR_ERR_UNSUPPORTED, "attention: the fused kernel takes a positive finite scale");
  }
  TVR_CHECK(seq_q <= 0x7fffff00 && seq_k <= 0x7fffff00, "attention: too many positions");
  const int64_t nqt = ceil_div(seq_q, BM);
  TVR_CHECK(batch * heads <= 0x7fffffff / nqt, "attention: too many query tiles");
  auto strides_ok = [](const float* ptr, const int64_t* s) {
    return tc::al16(ptr) && s[0] % 4 == 0 && s[1] % 4 == 0 && s[2] % 4 == 0 && s[0] > 0 &&
           s[1] > 0 && s[2] > 0;
  };
  if (!strides_ok(q, q_strides) || !strides_ok(k, k_strides) || !strides_ok(v, v_strides)) {
    return fail(TVR_ERR_UNSUPPORTED,
                "attention: operands need 16-byte aligned bases and strides that are multiples "
                "of 4 elements (TMA)");
  }
  // a few query rows (a decode step): the keys and values are streamed on
  // the CUDA cores instead of through mostly empty 128-row MMA tiles
  if (attention_decode_applies(seq_q, head_dim)) {
    return attention_decode(q, k, v, out, lse, batch, heads, seq_q, seq_k, q_strides, k_strides,
                            v_strides, o_strides, scale, causal, key_len, key_len_add,
                            as_stream(stream));
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
  if ((rc = enc(&p.tma_v, v, seq_k, v_strides, BN, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)) != TVR_OK)
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
  p.key_len = key_len;
  p.key_len_add = key_len_add;
  p.batch_heads = static_cast<int>(batch * heads);
  p.nqt = static_cast<int>(nqt);
  p.units = static_cast<int>(nqt * batch * heads);
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  std::call_once(once[dev & 63], [&]() {
    attr_err[dev & 63] = cudaFuncSetAttribute(
        attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  });
  TVR_CUDA_TRY(attr_err[dev & 63]);
  // persistent: two CTAs per SM, each working through its share of the units
  const int ctas = static_cast<int>(std::min<int64_t>(p.units, 2 * static_cast<int64_t>(sm_count(dev))));
  attn_fwd_kernel<<<ctas, THREADS, SMEM_BYTES, as_stream(stream)>>>(p);
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

// Writes src [batch, heads, seq_new, dim] into cache positions
// *pos .. *pos + seq_new - 1; positions at or past max_len are dropped and
// reported in the status word.
__global__ void __launch_bounds__(256) kv_append_kernel(float* cache, const float* src,
                                                        int64_t heads, int64_t seq_new,
                                                        int64_t dim, int64_t max_len,
                                                        int64_t cb, int64_t ch, int64_t cs,
                                                        int64_t sb, int64_t sh, int64_t ss,
                                                        const int64_t* pos, int64_t total,
                                                        int* status) {
  const int64_t p0 = *pos;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += stride) {
    const int64_t d = t % dim;
    int64_t r = t / dim;
    const int64_t s = r % seq_new;
    r /= seq_new;
    const int64_t h = r % heads;
    const int64_t b = r / heads;
    const int64_t at = p0 + s;
    if (at < 0 || at >= max_len) {
      if (status != nullptr) atomicCAS(status, TVR_DEV_OK, TVR_DEV_CACHE_FULL);
      continue;
    }
    cache[b * cb + h * ch + at * cs + d] = src[b * sb + h * sh + s * ss + d];
  }
}

__global__ void counter_add_kernel(int64_t* counter, int64_t delta) { *counter += delta; }

}  // namespace

extern "C" int tvr_attention_fwd(const float* q, const float* k, const float* v, float* out,
                                 float* lse, int64_t batch, int64_t heads, int64_t seq_q,
                                 int64_t seq_k, int64_t head_dim, const int64_t* q_strides,
                                 const int64_t* k_strides, const int64_t* v_strides,
                                 const int64_t* o_strides, float scale, int causal, int mode,
                                 void* stream) {
  return attention_impl(q, k, v, out, lse, batch, heads, seq_q, seq_k, head_dim, q_strides,
                        k_strides, v_strides, o_strides, scale, causal, mode, nullptr, 0,
                        stream);
}

extern "C" int tvr_attention_fwd_keylen(const float* q, const float* k, const float* v,
                                        float* out, int64_t batch, int64_t heads, int64_t seq_q,
                                        int64_t seq_k, int64_t head_dim,
                                        const int64_t* q_strides, const int64_t* k_strides,
                                        const int64_t* v_strides, const int64_t* o_strides,
                                        float scale, const int64_t* key_len, int key_len_add,
                                        int mode, void* stream) {
  TVR_CHECK(key_len != nullptr && reinterpret_cast<uintptr_t>(key_len) % 8 == 0,
            "attention_keylen: null or unaligned key length");
  return attention_impl(q, k, v, out, nullptr, batch, heads, seq_q, seq_k, head_dim, q_strides,
                        k_strides, v_strides, o_strides, scale, 0, mode, key_len, key_len_add,
                        stream);
}

extern "C" int tvr_kv_append(float* cache, const float* src, int64_t batch, int64_t heads,
                             int64_t seq_new, int64_t dim, int64_t max_len,
                             const int64_t* cache_strides, const int64_t* src_strides,
                             const int64_t* pos, void* stream) {
  TVR_CHECK(batch >= 0 && heads >= 0 && seq_new >= 0 && dim >= 0 && max_len >= 0,
            "kv_append: negative size");
  const int64_t total = batch * heads * seq_new * dim;
  if (total == 0) return TVR_OK;
  TVR_CHECK(cache && src && cache_strides && src_strides && pos, "kv_append: null pointer");
  TVR_CHECK(reinterpret_cast<uintptr_t>(pos) % 8 == 0, "kv_append: unaligned position");
  const int dev = current_device();
  kv_append_kernel<<<elementwise_grid(total, 256, dev), 256, 0, as_stream(stream)>>>(
      cache, src, heads, seq_new, dim, max_len, cache_strides[0], cache_strides[1],
      cache_strides[2], src_strides[0], src_strides[1], src_strides[2], pos, total,
      device_status_ptr(dev));
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

extern "C" int tvr_counter_add(int64_t* counter, int64_t delta, void* stream) {
  TVR_CHECK(counter != nullptr && reinterpret_cast<uintptr_t>(counter) % 8 == 0,
            "counter_add: null or unaligned counter");
  counter_add_kernel<<<1, 1, 0, as_stream(stream)>>>(counter, delta);
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

// Tensor-core fp32 GEMM for sm_100a: tcgen05.mma kind::tf32, accumulators in
// tensor memory, operands staged by TMA into 128-byte-swizzled shared memory.
//
// Computes C = act(alpha * A * op(B) + beta * P) for the linear / addmm / mm
// / bmm family — the reference's host::gemm_bias_act_f32 and host::bmm_f32
// (csrc/kernels/host/HostKernels.cpp:100-172), there a scalar 32^3-tiled loop.
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A tile [128 x 32] and B tile [BN x 32] per
//               k-block into a STAGES-deep ring (mbarrier full/empty pairs)
//   warp 1      allocates TMEM; one lane issues the MMAs (4 x K=8 per
//               k-block, 12 in 3xTF32 mode) and commits each stage back
//   warps 2-9   epilogue: tcgen05.ld of the 128 x BN accumulator in 32 x 32
//               chunks, each staged through a 128-byte-swizzled shared
//               buffer; bias / alpha / beta / activation, and optionally a
//               pointwise program (PROG), applied on the way; the chunk
//               leaves through one TMA bulk-tensor store (TMA_C, PROG) or
//               coalesced register stores (split-K partials, outputs read
//               back as beta * C, outputs a tensor map cannot describe)
// The accumulator is double-buffered in TMEM (2 x BN columns) so the
// epilogue of tile i overlaps the main loop of tile i+1.
//
// Two precisions (TVR_GEMM_TF32 / TVR_GEMM_3XTF32).  kind::tf32 reads the
// top 19 bits of each fp32 operand.  3xTF32 splits each operand into
// hi = x with the low 13 mantissa bits cleared and lo = x - hi (exact in
// fp32) and accumulates lo*hi + hi*lo + hi*hi, which restores fp32-level
// accuracy at three times the tensor work.
//
// Every wait on an mbarrier is bounded.  A wait that expires records a
// TVR_DEV_* code in the device status word and sets a CTA-wide abort flag;
// all roles then leave their loops, in-flight TMA loads and MMAs are
// drained (again with bounded waits), TMEM is freed and the kernel returns.
//
// No TMA load uses cluster multicast.
#include "internal.h"

#include <atomic>
#include <cstdlib>
#include <mutex>

#include "epilogue_prog.cuh"
#include "gemm_common.cuh"
#include "nvls_common.cuh"
#include "tc_ptx.cuh"

// TMA_C instances leave the chunk loop early (`continue`), so the register-
// store epilogue after it is unreachable there by design.
#pragma nv_diag_suppress 128

namespace tvr {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 32;  // fp32 elements per k-block = 128 bytes = one swizzle row
constexpr int EPI_WARPS = 8;
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;  // producer, MMA, epilogue warps
constexpr int STAGE_SMEM = 192 * 1024;
constexpr int EPI_BUF_BYTES = 32 * 32 * 4;                 // one 32 x 32 fp32 sub-tile
constexpr int EPI_SMEM = EPI_WARPS * EPI_BUF_BYTES;        // one staging buffer per warp
// Tile raster: units walk groups of tile rows (or columns) small enough that
// the group's panels of one operand stay in L2 while the other operand
// streams past them (pick_raster).
constexpr int64_t kRasterL2Bytes = int64_t(48) << 20;

template <int BN, bool SPLIT3>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int OPERANDS = SPLIT3 ? 2 : 1;
  static constexpr int STAGE_BYTES = OPERANDS * (A_BYTES + B_BYTES);
  static constexpr int STAGES = STAGE_SMEM / STAGE_BYTES;
  // two accumulators (one being filled while the epilogue drains the
  // other); 3xTF32 adds the running sum of a tile's K chunks (at column
  // 2 * BN).  Allocations are powers of two.
  static constexpr int TMEM_COLS = SPLIT3 ? (BN == 64 ? 256 : 512) : (BN == 192 ? 512 : 2 * BN);
  static constexpr int BAR_BYTES = 8 * (2 * STAGES + 5) + 8;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_SMEM + BAR_BYTES;
  static_assert(SMEM_BYTES <= 232448 - 64, "shared memory budget");
  static_assert(BN == 64 || BN == 128 || BN == 192 || BN == 256, "BN");
  static_assert(BN != 192 || !SPLIT3, "192-wide tiles are TF32 only");
  static_assert(!SPLIT3 || BN <= 128, "3xTF32 tiles keep a running sum beside two accumulators");
};

// 3xTF32: k-blocks per accumulation chunk.  The tensor core adds each MMA's
// products into its fp32 accumulator with truncation, so the accumulator's
// error grows with the number of MMAs added into it (3 per k-step in
// 3xTF32): over K = 4096 that is ~3e-5 relative, over K = 256 ~3e-6.  Each
// chunk of 256 K therefore starts a fresh accumulator, and the epilogue
// warps add the chunks in fp32 (round to nearest) into a running sum kept in
// tensor memory.  (512-wide chunks left a Llama MLP layer, three GEMMs
// deep with K up to 11008, at 1.2e-5 against the 1e-5 bar.)
constexpr int SPLIT3_KCHUNK = 8;

struct Params {
  CUtensorMap tma_a;     // A or A_hi: dims {K, M, batch}
  CUtensorMap tma_b;     // B or B_hi: {K, N, batch} (K-major) or {N, K, batch} (N-major)
  CUtensorMap tma_a_lo;  // 3xTF32 low parts, same geometry
  CUtensorMap tma_b_lo;  // or, for a gated GEMM, the up-projection weight {K, N, 1}
  CUtensorMap tma_c;     // TMA_C kernels: the output {N, M, batch}, 32 x 32 boxes, 128B swizzle
  const float* resid;    // TMA_C kernels, non-null: add resid[row * resid_ld + col] last
  int64_t resid_ld;
  const float* bias;
  float* c;
  int64_t ldc;
  int64_t stride_c;
  float alpha;
  float beta;
  int act;
  int use_prev;
  int c_vec;        // 1: output rows and base allow 16-byte stores
  int m, n, k;
  int batch;
  int b_broadcast;  // every batch entry uses B[0]
  int tiles_m, tiles_n;
  int group;        // raster group: tile rows (raster_n == 0) or tile columns (1)
  int raster_n;
  int splits;       // > 1: split-K, raw partial sums to the workspace at c
  int kb_per_split;
  int kchunk;       // 3xTF32: k-blocks per accumulation chunk
  int num_kb;
  int total_units;
  int* status;
  EpiProg prog;  // PROG kernels: pointwise program applied to each output element
  // NVLS kernels (tvr_gemm_nvls_all_reduce_f32): the output summed over ranks
  float* nv_mc;               // multicast address of c
  nvls::PeerFlags nv_flags;   // every rank's flag array
  const uint32_t* nv_epoch;   // this call's epoch (advanced before the launch)
  int nv_rank, nv_world;
  int nv_gemm_ctas;           // CTAs [0, nv_gemm_ctas) compute tiles, the rest reduce them
};

// N-major tile: 32-wide N atoms of [BK rows x 128 B] placed BK*128 B apart
// (leading offset); 32-byte chunks swizzled over 4 rows, so K groups are
// 4 rows = 512 B apart (stride offset).
__device__ __forceinline__ uint64_t desc_nmajor(uint32_t saddr) {
  return make_desc(saddr, BK * 128, 512, 1);
}

// Instruction descriptor of the BM x N x 8 MMA.
__host__ __device__ constexpr uint32_t make_idesc(int n, bool b_nmajor) {
  return idesc_tf32(BM, n, b_nmajor);
}

// Work unit -> (operand batch index, k split, tile row, tile column).
// Tiles are rastered in groups of p.group tile rows (M fastest inside a
// group), or with raster_n of p.group tile columns (N fastest), so the CTAs
// running at the same time share panels, and the group's panels of one
// operand stay in L2 while the whole other operand streams past them once.
__device__ __forceinline__ void decode_unit(const Params& p, int u, int& b, int& s, int& tm,
                                            int& tn) {
  const int per = p.tiles_m * p.tiles_n;
  const int outer = u / per;
  const int r = u - outer * per;
  b = outer / p.splits;
  s = outer - b * p.splits;
  const int G = p.group;
  if (p.raster_n == 0) {
    const int span = G * p.tiles_n;
    const int g = r / span;
    const int first_m = g * G;
    const int gm = min(p.tiles_m - first_m, G);
    const int rr = r - g * span;
    tm = first_m + rr % gm;
    tn = rr / gm;
  } else {
    const int span = G * p.tiles_m;
    const int g = r / span;
    const int first_n = g * G;
    const int gn = min(p.tiles_n - first_n, G);
    const int rr = r - g * span;
    tn = first_n + rr % gn;
    tm = rr / gn;
  }
}

// Raster for a tiles_m x tiles_n grid whose A panels (one tile row over the
// whole K) take panel_a bytes and B panels panel_b: hold a group of A panels
// in L2 and stream B once per group, or the other way round, whichever
// moves fewer bytes from HBM when a group may take kRasterL2Bytes.
inline void pick_raster(Params& p, int64_t panel_a, int64_t panel_b) {
  const int64_t budget = kRasterL2Bytes;
  const int64_t tm = p.tiles_m, tn = p.tiles_n;
  const int64_t gm = std::max<int64_t>(1, std::min<int64_t>(tm, budget / std::max<int64_t>(1, panel_a)));
  const int64_t gn = std::max<int64_t>(1, std::min<int64_t>(tn, budget / std::max<int64_t>(1, panel_b)));
  const int64_t bytes_m = tm * panel_a + tn * panel_b * ceil_div(tm, gm);
  const int64_t bytes_n = tn * panel_b + tm * panel_a * ceil_div(tn, gn);
  if (bytes_n < bytes_m) {
    p.raster_n = 1;
    p.group = static_cast<int>(gn);
  } else {
    p.raster_n = 0;
    p.group = static_cast<int>(gm);
  }
}

// NVLS kernels: the CTAs past the GEMM's sum this rank's output tiles (unit
// u with u % world == rank) over all ranks.  Each epilogue warp of every
// rank counts its part of tile u, once stored, in the owner's counter u; a
// reducer waits for all EPI_WARPS x world arrivals, resets the counter for
// the next call, reads the tile's sum through the switch and stores it to
// every rank.  The closing barrier keeps every rank in the kernel until all
// ranks' reducers are done, so each rank's c holds the whole sum when the
// kernel ends.
template <int OUT_BN>
__device__ __forceinline__ void nvls_reduce_tiles(const Params& p) {
  using namespace nvls;
  __shared__ int expired;
  constexpr int kUnroll = 4;
  const int rc = static_cast<int>(blockIdx.x) - p.nv_gemm_ctas;
  const int nred = static_cast<int>(gridDim.x) - p.nv_gemm_ctas;
  const int rank = p.nv_rank, world = p.nv_world;
  const uint32_t epoch = *p.nv_epoch;
  const uint32_t arrivals = static_cast<uint32_t>(EPI_WARPS * world);
  uint32_t* mine = p.nv_flags.flags[rank] + kTileCounters;
  if (threadIdx.x == 0) expired = 0;
  __syncthreads();
  for (int i = rc;; i += nred) {
    const int u = rank + world * i;
    if (u >= p.total_units) break;
    if (threadIdx.x == 0) {
      if (wait_at_least(mine + u, arrivals, p.status)) {
        mine[u] = 0;  // every arrival of this call is in; the next call counts afresh
      } else {
        expired = 1;
      }
    }
    __syncthreads();
    if (expired) break;
    int b, s, tm, tn;
    decode_unit(p, u, b, s, tm, tn);
    const int row0 = tm * BM, col0 = tn * OUT_BN;
    const int c4 = min(OUT_BN, p.n - col0) / 4;  // n % 4 == 0
    const int total = min(BM, p.m - row0) * c4;
    const int nt = static_cast<int>(blockDim.x);
    for (int e = static_cast<int>(threadIdx.x); e < total; e += kUnroll * nt) {
      float4 v[kUnroll];
      float* at[kUnroll];
#pragma unroll
      for (int q = 0; q < kUnroll; ++q) {
        const int idx = e + q * nt;
        const int r = idx / c4;
        at[q] = p.nv_mc + static_cast<int64_t>(row0 + r) * p.ldc + col0 + 4 * (idx - r * c4);
        if (idx < total) v[q] = multimem_ld_reduce_add(at[q]);
      }
#pragma unroll
      for (int q = 0; q < kUnroll; ++q) {
        if (e + q * nt < total) multimem_st(at[q], v[q]);
      }
    }
  }
  rank_barrier(p.nv_flags, rank, world, 2, rc, epoch, p.status, &expired);
}

// GATED (TF32, K-major weights, BN = 256): the B tile stacks 128 rows of the
// gate weight (tma_b) over the same 128 rows of the up weight (tma_b_lo), the
// MMA fills accumulator columns 0..127 with x.Wg^T and 128..255 with x.Wu^T,
// and the epilogue writes silu(gate) * up: a 128 x 128 output tile.
//
// PROG (K-major weights, no split-K): after bias and activation, the epilogue
// runs the pointwise program p.prog on each output element, reading the
// program's other inputs at the element's position, and stores its result.
//
// TMA_C (no split-K, no program, output not read back): bias and activation
// are applied to each thread's row in registers, the 32 x 32 chunk is staged
// in the 128-byte-swizzled layout a TMA box of the output has, and one lane
// stores it with cp.async.bulk.tensor — no warp issues global stores.  This
// is what small-K GEMMs (batched attention scores, K = 64..128), whose time
// is the output stream, need.
template <int BN, bool SPLIT3, bool B_NMAJOR, bool GATED = false, bool PROG = false,
          bool TMA_C = false, bool NVLS = false>
__global__ void __launch_bounds__(NUM_THREADS, 1) gemm_tc_kernel(const __grid_constant__ Params p) {
  using Cf = Cfg<BN, SPLIT3>;
  static_assert(!GATED || (BN == 256 && !SPLIT3 && !B_NMAJOR), "gated GEMM shape");
  static_assert(!PROG || (!GATED && !B_NMAJOR), "pointwise-epilogue GEMM shape");
  static_assert(!TMA_C || (!GATED && !PROG), "TMA-store epilogue");
  static_assert(!NVLS || (TMA_C && !SPLIT3 && !B_NMAJOR), "GEMM + NVLS all-reduce shape");
  constexpr int OUT_BN = GATED ? BN / 2 : BN;  // output columns per tile
  constexpr int STAGES = Cf::STAGES;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_abort;
  if constexpr (NVLS) {
    // CTAs past the first nv_gemm_ctas reduce; the tile loops below stride
    // over the GEMM CTAs only
    if (static_cast<int>(blockIdx.x) >= p.nv_gemm_ctas) {
      nvls_reduce_tiles<OUT_BN>(p);
      return;
    }
  }

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t stage0 = base;
  const uint32_t epi0 = base + STAGES * Cf::STAGE_BYTES;
  const uint32_t bar0 = epi0 + EPI_SMEM;
  const uint32_t full_bar = bar0;                       // [STAGES]
  const uint32_t empty_bar = bar0 + 8 * STAGES;         // [STAGES]
  const uint32_t tfull_bar = bar0 + 16 * STAGES;        // [2]
  const uint32_t tempty_bar = tfull_bar + 16;           // [2]
  const uint32_t drain_bar = tempty_bar + 16;           // [1]
  const uint32_t holder = drain_bar + 8;                // TMEM base address
  uint32_t* holder_ptr = reinterpret_cast<uint32_t*>(smem_raw + (holder - raw));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const volatile int* abort_flag = &s_abort;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar + 8 * s, 1);
      mbar_init(empty_bar + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar + 8 * b, 1);
      mbar_init(tempty_bar + 8 * b, EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(holder),
                 "r"(Cf::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(holder_ptr);

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0;  // stages with a load issued
      uint32_t issued_parity = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.total_units; u += NVLS ? static_cast<unsigned>(p.nv_gemm_ctas) : gridDim.x) {
        int b, s, tm, tn;
        decode_unit(p, u, b, s, tm, tn);
        const int kb0 = s * p.kb_per_split;
        const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        const int zb = p.b_broadcast ? 0 : b;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(empty_bar + 8 * stage, phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = full_bar + 8 * stage;
          mbar_expect_tx(fb, Cf::STAGE_BYTES);
          const uint32_t sa = stage0 + stage * Cf::STAGE_BYTES;
          const uint32_t sb = sa + Cf::A_BYTES;
          const int kx = kb * BK;
          tma_load_3d(sa, &p.tma_a, fb, kx, tm * BM, b);
          if (GATED) {
            tma_load_3d(sb, &p.tma_b, fb, kx, tn * OUT_BN, zb);
            tma_load_3d(sb + OUT_BN * BK * 4, &p.tma_b_lo, fb, kx, tn * OUT_BN, zb);
          } else if (B_NMAJOR) {
#pragma unroll
            for (int j = 0; j < BN / 32; ++j)
              tma_load_3d(sb + j * (BK * 128), &p.tma_b, fb, tn * BN + 32 * j, kx, zb);
          } else {
            tma_load_3d(sb, &p.tma_b, fb, kx, tn * BN, zb);
          }
          if (SPLIT3) {
            const uint32_t sa_lo = sb + Cf::B_BYTES;
            const uint32_t sb_lo = sa_lo + Cf::A_BYTES;
            tma_load_3d(sa_lo, &p.tma_a_lo, fb, kx, tm * BM, b);
            if (B_NMAJOR) {
#pragma unroll
              for (int j = 0; j < BN / 32; ++j)
                tma_load_3d(sb_lo + j * (BK * 128), &p.tma_b_lo, fb, tn * BN + 32 * j, kx, zb);
            } else {
              tma_load_3d(sb_lo, &p.tma_b_lo, fb, kx, tn * BN, zb);
            }
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        record_status(p.status, TVR_DEV_TIMEOUT_PRODUCER);
        *const_cast<volatile int*>(abort_flag) = 1;
      }
      // Every issued load must land before the CTA may exit.
      for (int st = 0; st < STAGES; ++st) {
        if (issued_mask & (1u << st)) {
          if (!mbar_wait(full_bar + 8 * st, (issued_parity >> st) & 1u, nullptr)) {
            record_status(p.status, TVR_DEV_TIMEOUT_DRAIN);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(BN, B_NMAJOR);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued = false;
      for (int u = blockIdx.x; ok && u < p.total_units; u += NVLS ? static_cast<unsigned>(p.nv_gemm_ctas) : gridDim.x) {
        int b, s, tm, tn;
        decode_unit(p, u, b, s, tm, tn);
        const int kb0 = s * p.kb_per_split;
        const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        // one accumulation chunk per unit, or (3xTF32) one per p.kchunk
        // k-blocks, each into the next accumulator buffer
        const int kc = SPLIT3 ? p.kchunk : kb1 - kb0;
        for (int c0 = kb0; c0 < kb1; c0 += kc) {
          const int c1 = min(kb1, c0 + kc);
          if (!mbar_wait(tempty_bar + 8 * acc, acc_phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
          for (int kb = c0; kb < c1; ++kb) {
            if (!mbar_wait(full_bar + 8 * stage, phase, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = stage0 + stage * Cf::STAGE_BYTES;
            const uint32_t sb = sa + Cf::A_BYTES;
#pragma unroll
            for (int kk = 0; kk < BK / 8; ++kk) {
              const uint64_t da = desc_kmajor(sa + kk * 32);
              const uint64_t db = B_NMAJOR ? desc_nmajor(sb + kk * 1024) : desc_kmajor(sb + kk * 32);
              const uint32_t first = (kb > c0 || kk > 0) ? 1u : 0u;
              if (SPLIT3) {
                const uint32_t sa_lo = sb + Cf::B_BYTES;
                const uint32_t sb_lo = sa_lo + Cf::A_BYTES;
                const uint64_t da_lo = desc_kmajor(sa_lo + kk * 32);
                const uint64_t db_lo =
                    B_NMAJOR ? desc_nmajor(sb_lo + kk * 1024) : desc_kmajor(sb_lo + kk * 32);
                mma_tf32(d, da_lo, db, idesc, first);
                mma_tf32(d, da, db_lo, idesc, 1u);
                mma_tf32(d, da, db, idesc, 1u);
              } else {
                mma_tf32(d, da, db, idesc, first);
              }
            }
            issued = true;
            mma_commit(empty_bar + 8 * stage);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          mma_commit(tfull_bar + 8 * acc);
          acc ^= 1;
          if (acc == 0) acc_phase ^= 1u;
        }
        if (!ok) break;
      }
      if (!ok) {
        record_status(p.status, TVR_DEV_TIMEOUT_MMA);
        *const_cast<volatile int*>(abort_flag) = 1;
      }
      // All issued MMAs must retire before TMEM is released.
      if (issued) {
        mma_commit(drain_bar);
        if (!mbar_wait(drain_bar, 0, nullptr)) record_status(p.status, TVR_DEV_TIMEOUT_DRAIN);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue ------------------------------
    // Eight warps: warp w reads TMEM lane quarter (w % 4) (rows 32q..32q+31
    // of the tile) and one half of the columns, 32 columns at a time; the
    // TMEM buffer goes back to the MMA warp after the last chunk is read
    // (the other buffer keeps the tensor cores busy meanwhile).  Each 32x32
    // chunk is transposed through a swizzled 4 KB shared buffer so that the
    // epilogue math works on four consecutive columns per lane and 8 lanes
    // write one 128-byte row segment.
    const int q = warp & 3;
    const int ew = warp - 2;
    const int half = ew >> 2;
    constexpr int HC = OUT_BN / 2;  // output columns per warp
    constexpr int CH = HC / 32;     // 32-column chunks per warp
    constexpr uint32_t UP = BN / 2;  // gated: TMEM column offset of the up half
    const uint32_t sbuf = epi0 + ew * EPI_BUF_BYTES;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.total_units; u += NVLS ? static_cast<unsigned>(p.nv_gemm_ctas) : gridDim.x) {
      int b, s, tm, tn;
      decode_unit(p, u, b, s, tm, tn);
      const uint32_t lanes = static_cast<uint32_t>(32 * q) << 16;
      uint32_t tcol = tmem_base + lanes + static_cast<uint32_t>(acc * BN + half * HC);
      // 3xTF32 with more than one accumulation chunk: each chunk's
      // accumulator is added into the running sum (column 2 * BN) and handed
      // back; the tile's epilogue then reads the running sum.
      bool folded = false;
      if constexpr (SPLIT3) {
        const int kb0 = s * p.kb_per_split;
        const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        const int nch = (kb1 - kb0 + p.kchunk - 1) / p.kchunk;
        if (nch > 1) {
          const uint32_t scol = tmem_base + lanes + static_cast<uint32_t>(2 * BN + half * HC);
          for (int ci = 0; ci < nch; ++ci) {
            const bool got = mbar_wait(tfull_bar + 8 * acc, acc_phase, abort_flag);
            if (!__all_sync(0xffffffffu, got)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t acol = tmem_base + lanes + static_cast<uint32_t>(acc * BN + half * HC);
#pragma unroll
            for (int c = 0; c < CH; ++c) {
              float a[32];
              tmem_load_32_async(acol + 32 * c, a);
              if (ci > 0) {
                float r[32];
                tmem_load_32_async(scol + 32 * c, r);
                tmem_wait_loads();
#pragma unroll
                for (int i = 0; i < 32; ++i) a[i] = __fadd_rn(r[i], a[i]);
              } else {
                tmem_wait_loads();
              }
              tmem_store_32(scol + 32 * c, a);
            }
            tmem_wait_stores();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar + 8 * acc);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
          }
          if (!ok) break;
          tc_fence_after();
          tcol = scol;
          folded = true;
        }
      }
      if (!folded) {
        const bool got = mbar_wait(tfull_bar + 8 * acc, acc_phase, abort_flag);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      const int zc = p.splits > 1 ? s : b;
      float* cbase = p.c + static_cast<int64_t>(zc) * p.stride_c;
      const int64_t row0 = static_cast<int64_t>(tm) * BM + 32 * q;
      const bool finish = p.splits == 1;
      // chunk c+1 is read from TMEM while chunk c is transposed and stored
      float v[32];
      float up[GATED ? 32 : 1];
      tmem_load_32_async(tcol, v);
      if constexpr (GATED) tmem_load_32_async(tcol + UP, up);
      tmem_wait_loads();
      if constexpr (GATED) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = act_fixed<TVR_ACT_SILU>(v[i]) * up[i];
      }
      const bool plain = GATED || (p.alpha == 1.f && p.act == TVR_ACT_NONE &&
                                   (p.beta == 0.f || (p.bias == nullptr && !p.use_prev)));
      // A pointwise program makes each chunk's code long: keep one copy of
      // it (instruction-cache misses otherwise stall every warp of the CTA).
      constexpr int CH_UNROLL = PROG ? 1 : CH;
#pragma unroll CH_UNROLL
      for (int c = 0; c < CH; ++c) {
        if (c == CH - 1 && !folded) {
          // accumulator fully read: hand the TMEM buffer back to the MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tempty_bar + 8 * acc);
        }
        if constexpr (TMA_C) {
          const int col0 = tn * OUT_BN + half * HC + 32 * c;
          // A residual add (the epilogue program Load y, Load r, Add, run
          // natively): the chunk's 32 x 32 residual block, loaded first in
          // the coalesced layout (rows 4i + lane / 8, columns 4 (lane % 8)),
          // added to the staged chunk after the bias step as the program
          // adds it (one IEEE addition)
          float4 rv[8];
          const bool resid = p.resid != nullptr;
          if (resid) {
            const int cj = col0 + 4 * (lane & 7);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int64_t row = row0 + 4 * i + (lane >> 3);
              const float* rs = p.resid + row * p.resid_ld + cj;
              rv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
              if (row < p.m) {
                if (cj + 3 < p.n) {
                  rv[i] = __ldg(reinterpret_cast<const float4*>(rs));
                } else {
                  if (cj < p.n) rv[i].x = __ldg(rs);
                  if (cj + 1 < p.n) rv[i].y = __ldg(rs + 1);
                  if (cj + 2 < p.n) rv[i].z = __ldg(rs + 2);
                }
              }
            }
          }
          if (!plain) {
            // act(alpha * acc + beta * bias): epilogue4's arithmetic, per
            // element; one straight-line loop per activation (with the choice
            // inside the loop every element would pay for the SiLU path)
            float bv[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              bv[j] = p.bias != nullptr && col0 + j < p.n ? __ldg(p.bias + col0 + j) : 0.f;
            }
            if (p.act == TVR_ACT_SILU) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                v[j] = act_fixed<TVR_ACT_SILU>(__fadd_rn(__fmul_rn(p.alpha, v[j]), __fmul_rn(p.beta, bv[j])));
            } else if (p.act == TVR_ACT_RELU) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                v[j] = act_fixed<TVR_ACT_RELU>(__fadd_rn(__fmul_rn(p.alpha, v[j]), __fmul_rn(p.beta, bv[j])));
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                v[j] = __fadd_rn(__fmul_rn(p.alpha, v[j]), __fmul_rn(p.beta, bv[j]));
            }
          }
          // the previous chunk's store must have read the staging buffer
          if (lane == 0) bulk_wait_read();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t addr = sbuf + lane * 128 + ((j ^ (lane & 7)) << 4);
            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v[4 * j]),
                         "f"(v[4 * j + 1]), "f"(v[4 * j + 2]), "f"(v[4 * j + 3])
                         : "memory");
          }
          if (resid) {
            __syncwarp();
            const int jj = lane & 7;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int rr = 4 * i + (lane >> 3);
              const uint32_t addr = sbuf + rr * 128 + ((jj ^ (rr & 7)) << 4);
              float4 x;
              asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                           : "=f"(x.x), "=f"(x.y), "=f"(x.z), "=f"(x.w)
                           : "r"(addr));
              x.x = __fadd_rn(x.x, rv[i].x);
              x.y = __fadd_rn(x.y, rv[i].y);
              x.z = __fadd_rn(x.z, rv[i].z);
              x.w = __fadd_rn(x.w, rv[i].w);
              asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(x.x),
                           "f"(x.y), "f"(x.z), "f"(x.w)
                           : "memory");
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && col0 < p.n && row0 < p.m) {  // (boxes past the edge are clipped)
            tma_store_3d(&p.tma_c, sbuf, col0, static_cast<int>(row0), zc);
            bulk_commit();
          }
          if (c + 1 < CH) {
            tmem_load_32_async(tcol + 32 * (c + 1), v);
            tmem_wait_loads();
          }
          continue;
        }
        if constexpr (PROG) {
          // the previous chunk's TMA store must have read the staging buffer
          if (lane == 0) bulk_wait_read();
          __syncwarp();
        }
        // stage: thread = row, 16-byte chunk j of row r at chunk j ^ (r & 7)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t addr = sbuf + lane * 128 + ((j ^ (lane & 7)) << 4);
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v[4 * j]),
                       "f"(v[4 * j + 1]), "f"(v[4 * j + 2]), "f"(v[4 * j + 3])
                       : "memory");
        }
        // (with a program, the next chunk is read after this one is stored:
        // its 32 registers hold the program's prefetched input meanwhile)
        if (!PROG && c + 1 < CH) {
          tmem_load_32_async(tcol + 32 * (c + 1), v);
          if constexpr (GATED) tmem_load_32_async(tcol + UP + 32 * (c + 1), up);
        }
        __syncwarp();
        const int jj = lane & 7;
        const int col = tn * OUT_BN + half * HC + 32 * c + 4 * jj;
        float4 bias4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (finish && p.bias != nullptr) {
          if (p.c_vec && col + 3 < p.n) {
            bias4 = __ldg(reinterpret_cast<const float4*>(p.bias + col));
          } else {
            bias4.x = col < p.n ? __ldg(p.bias + col) : 0.f;
            bias4.y = col + 1 < p.n ? __ldg(p.bias + col + 1) : 0.f;
            bias4.z = col + 2 < p.n ? __ldg(p.bias + col + 2) : 0.f;
            bias4.w = col + 3 < p.n ? __ldg(p.bias + col + 3) : 0.f;
          }
        }
        const bool full4 = p.c_vec && col + 3 < p.n;
        if constexpr (PROG) {
          // The program as stack code (EpiProg::sop), each operation applied
          // to 16 values of this lane at once: rows row0 + 4i + lane/8 for
          // i in [4h, 4h + 4), columns col..col+3, for the two halves h of
          // the chunk.  Slot 0 ends as the result.
          const bool read_prev = finish && p.bias == nullptr && p.use_prev;
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            float s0[16], s1[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) s0[j] = s1[j] = 0.f;
#pragma unroll 1
            for (int pc = 0; pc < p.prog.n_ops; ++pc) {
              const int op = p.prog.sop[pc];
              const float sv = p.prog.sval[pc];
              const bool rv = p.prog.rev[pc] != 0;
              if (op <= kStPushC) {
#pragma unroll
                for (int j = 0; j < 16; ++j) s1[j] = s0[j];
              }
              switch (op) {
                case kStPushY: {
                  // one row at a time: no temporaries beside the two slots
#pragma unroll
                  for (int i = 0; i < 4; ++i) {
                    const int rr = 4 * (4 * h + i) + (lane >> 3);
                    const uint32_t addr = sbuf + rr * 128 + ((jj ^ (rr & 7)) << 4);
                    float4 x;
                    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                                 : "=f"(x.x), "=f"(x.y), "=f"(x.z), "=f"(x.w)
                                 : "r"(addr));
                    if (finish && !plain) {
                      float4 prev = bias4;
                      const int64_t row = row0 + rr;
                      if (read_prev && row < p.m && col < p.n) {
                        const float* src = cbase + row * p.ldc + col;
                        if (full4) {
                          prev = *reinterpret_cast<const float4*>(src);
                        } else {
                          prev.x = src[0];
                          prev.y = col + 1 < p.n ? src[1] : 0.f;
                          prev.z = col + 2 < p.n ? src[2] : 0.f;
                          prev.w = col + 3 < p.n ? src[3] : 0.f;
                        }
                      }
                      if (p.act == TVR_ACT_SILU) epilogue4<TVR_ACT_SILU>(x, prev, p.alpha, p.beta);
                      else if (p.act == TVR_ACT_RELU) epilogue4<TVR_ACT_RELU>(x, prev, p.alpha, p.beta);
                      else epilogue4<TVR_ACT_NONE>(x, prev, p.alpha, p.beta);
                    }
                    s0[4 * i] = x.x;
                    s0[4 * i + 1] = x.y;
                    s0[4 * i + 2] = x.z;
                    s0[4 * i + 3] = x.w;
                  }
                  break;
                }
                case kStPushX:
#pragma unroll
                  for (int i = 0; i < 4; ++i) {
                    const float4 e =
                        epi_load4(p.prog, 0, row0 + 4 * (4 * h + i) + (lane >> 3), col, p.m, p.n);
                    s0[4 * i] = e.x;
                    s0[4 * i + 1] = e.y;
                    s0[4 * i + 2] = e.z;
                    s0[4 * i + 3] = e.w;
                  }
                  break;
                case kStPushC:
#pragma unroll
                  for (int j = 0; j < 16; ++j) s0[j] = sv;
                  break;
                case kStAdd:
#pragma unroll
                  for (int j = 0; j < 16; ++j) {
                    const float a = rv ? s0[j] : s1[j], b = rv ? s1[j] : s0[j];
                    s0[j] = __fadd_rn(a, __fmul_rn(sv, b));
                  }
                  break;
                case kStSub:
#pragma unroll
                  for (int j = 0; j < 16; ++j) {
                    const float a = rv ? s0[j] : s1[j], b = rv ? s1[j] : s0[j];
                    s0[j] = __fadd_rn(a, __fmul_rn(-sv, b));
                  }
                  break;
                case kStMul:
#pragma unroll
                  for (int j = 0; j < 16; ++j) s0[j] = __fmul_rn(s1[j], s0[j]);
                  break;
                case kStRelu:
#pragma unroll
                  for (int j = 0; j < 16; ++j) s0[j] = s0[j] > 0.f ? s0[j] : 0.f;
                  break;
                case kStSilu:
#pragma unroll
                  for (int j = 0; j < 16; ++j) s0[j] = s0[j] / (1.f + expf(-s0[j]));
                  break;
                case kStNeg:
#pragma unroll
                  for (int j = 0; j < 16; ++j) s0[j] = -s0[j];
                  break;
                case kStScale:
#pragma unroll
                  for (int j = 0; j < 16; ++j) s0[j] = __fmul_rn(sv, s0[j]);
                  break;
                case kStSigmoid:
#pragma unroll
                  for (int j = 0; j < 16; ++j) s0[j] = 1.f / (1.f + expf(-s0[j]));
                  break;
                case kStExp:
#pragma unroll
                  for (int j = 0; j < 16; ++j) s0[j] = expf(s0[j]);
                  break;
                default:  // kStAbs
#pragma unroll
                  for (int j = 0; j < 16; ++j) s0[j] = fabsf(s0[j]);
                  break;
              }
            }
            // results back into the staged chunk (these rows' PushY reads
            // are done); the chunk leaves through one TMA store below
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int rr = 4 * (4 * h + i) + (lane >> 3);
              const uint32_t addr = sbuf + rr * 128 + ((jj ^ (rr & 7)) << 4);
              asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(s0[4 * i]),
                           "f"(s0[4 * i + 1]), "f"(s0[4 * i + 2]), "f"(s0[4 * i + 3])
                           : "memory");
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          const int col0 = tn * OUT_BN + half * HC + 32 * c;
          if (lane == 0 && col0 < p.n && row0 < p.m) {  // (boxes past the edge are clipped)
            tma_store_3d(&p.tma_c, sbuf, col0, static_cast<int>(row0), zc);
            bulk_commit();
          }
        } else if (!p.c_vec) {
          // Rows not 16-byte aligned (an LM head's N = 50257): lane = column,
          // one row of 32 consecutive floats per store instruction, which
          // writes a few whole sectors of that row.  (Lane = row with four
          // scalar stores per lane made every store instruction 32 separate
          // sector writes.)  Loads first, then stores, as below.
          const int colj = tn * OUT_BN + half * HC + 32 * c + lane;
          float xr[32];
#pragma unroll
          for (int r = 0; r < 32; ++r) {
            const uint32_t addr =
                sbuf + r * 128 + ((((lane >> 2) ^ (r & 7)) << 4) | ((lane & 3) << 2));
            asm volatile("ld.shared.f32 %0, [%1];" : "=f"(xr[r]) : "r"(addr));
          }
          if (finish && !plain) {
            const bool read_prev = p.bias == nullptr && p.use_prev;
            const float bj = p.bias != nullptr && colj < p.n ? __ldg(p.bias + colj) : 0.f;
            float prev[32];
#pragma unroll
            for (int r = 0; r < 32; ++r) {
              const int64_t row = row0 + r;
              prev[r] = read_prev && row < p.m && colj < p.n ? cbase[row * p.ldc + colj] : bj;
            }
            // epilogue4's arithmetic, element by element
            if (p.act == TVR_ACT_SILU) {
#pragma unroll
              for (int r = 0; r < 32; ++r)
                xr[r] = act_fixed<TVR_ACT_SILU>(__fadd_rn(__fmul_rn(p.alpha, xr[r]), __fmul_rn(p.beta, prev[r])));
            } else if (p.act == TVR_ACT_RELU) {
#pragma unroll
              for (int r = 0; r < 32; ++r)
                xr[r] = act_fixed<TVR_ACT_RELU>(__fadd_rn(__fmul_rn(p.alpha, xr[r]), __fmul_rn(p.beta, prev[r])));
            } else {
#pragma unroll
              for (int r = 0; r < 32; ++r)
                xr[r] = __fadd_rn(__fmul_rn(p.alpha, xr[r]), __fmul_rn(p.beta, prev[r]));
            }
          }
          asm volatile("" ::: "memory");
#pragma unroll
          for (int r = 0; r < 32; ++r) {
            const int64_t row = row0 + r;
            if (row < p.m && colj < p.n) cbase[row * p.ldc + colj] = xr[r];
          }
        } else {
          // All shared-memory reads (and reads of the previous output, when
          // beta applies to it) are issued before any global store: a warp's
          // memory instructions drain in order, so a load queued behind a
          // store would wait for that store.
          float4 xs[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int rr = 4 * i + (lane >> 3);
            const uint32_t addr = sbuf + rr * 128 + ((jj ^ (rr & 7)) << 4);
            asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(xs[i].x), "=f"(xs[i].y), "=f"(xs[i].z), "=f"(xs[i].w)
                         : "r"(addr));
          }
          if (finish && !plain) {
            const bool read_prev = p.bias == nullptr && p.use_prev;
            float4 prev[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int64_t row = row0 + 4 * i + (lane >> 3);
              prev[i] = bias4;
              if (read_prev && row < p.m && col < p.n) {
                const float* src = cbase + row * p.ldc + col;
                if (full4) {
                  prev[i] = *reinterpret_cast<const float4*>(src);
                } else {
                  prev[i].x = src[0];
                  prev[i].y = col + 1 < p.n ? src[1] : 0.f;
                  prev[i].z = col + 2 < p.n ? src[2] : 0.f;
                  prev[i].w = col + 3 < p.n ? src[3] : 0.f;
                }
              }
            }
            // One straight-line loop per activation: with the choice inside
            // the element loop the compiler evaluates the SiLU path for
            // every element.
            if (p.act == TVR_ACT_SILU) {
#pragma unroll
              for (int i = 0; i < 8; ++i) epilogue4<TVR_ACT_SILU>(xs[i], prev[i], p.alpha, p.beta);
            } else if (p.act == TVR_ACT_RELU) {
#pragma unroll
              for (int i = 0; i < 8; ++i) epilogue4<TVR_ACT_RELU>(xs[i], prev[i], p.alpha, p.beta);
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) epilogue4<TVR_ACT_NONE>(xs[i], prev[i], p.alpha, p.beta);
            }
          }
          // compiler barrier: keeps the stores below every load above
          asm volatile("" ::: "memory");
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int64_t row = row0 + 4 * i + (lane >> 3);
            if (row >= p.m || col >= p.n) continue;
            float* dst = cbase + row * p.ldc + col;
            if (full4) {
              *reinterpret_cast<float4*>(dst) = xs[i];
            } else {
              dst[0] = xs[i].x;
              if (col + 1 < p.n) dst[1] = xs[i].y;
              if (col + 2 < p.n) dst[2] = xs[i].z;
              if (col + 3 < p.n) dst[3] = xs[i].w;
            }
          }
        }
        if (PROG && c + 1 < CH) tmem_load_32_async(tcol + 32 * (c + 1), v);
        if (c + 1 < CH) {
          tmem_wait_loads();
          if constexpr (GATED) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = act_fixed<TVR_ACT_SILU>(v[i]) * up[i];
          }
        }
        __syncwarp();  // the staging buffer is rewritten by the next chunk
      }
      if constexpr (NVLS) {
        // this warp's 32 x HC part of tile u is in c: count it at the tile's
        // owner once the stores are complete and ordered before the count
        if (lane == 0) {
          bulk_wait_all();
          asm volatile("fence.proxy.async.global;" ::: "memory");
          nvls::fence_sys();
          nvls::red_release_sys_add(
              p.nv_flags.flags[u % p.nv_world] + nvls::kTileCounters + u, 1u);
        }
        __syncwarp();
      }
      if (!folded) {
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
    // every store this warp issued is complete before the CTA exits
    if ((TMA_C || PROG) && lane == 0) bulk_wait_all();
    __syncwarp();
    if (!ok) {
      record_status(p.status, TVR_DEV_TIMEOUT_EPILOGUE);
      *const_cast<volatile int*>(abort_flag) = 1;
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(Cf::TMEM_COLS)
                 : "memory");
  }
}

// hi = x with the low 13 mantissa bits cleared, lo = x - hi (exact).
__global__ void __launch_bounds__(256) split_tf32_kernel(const float* __restrict__ src,
                                                         float* __restrict__ hi,
                                                         float* __restrict__ lo, int64_t rows,
                                                         int64_t cols, int64_t ld,
                                                         int64_t batch_stride, int64_t ld_out,
                                                         int64_t batch) {
  const int64_t per = rows * cols;
  const int64_t total = per * batch;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const int64_t bb = i / per;
    const int64_t rem = i - bb * per;
    const int64_t r = rem / cols, c = rem - (rem / cols) * cols;
    const float x = src[bb * batch_stride + r * ld + c];
    const float h = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
    const int64_t o = (bb * rows + r) * ld_out + c;
    hi[o] = h;
    lo[o] = x - h;
  }
}

__global__ void __launch_bounds__(256) split_tf32_vec4_kernel(const float4* __restrict__ src,
                                                              float4* __restrict__ hi,
                                                              float4* __restrict__ lo,
                                                              int64_t n4) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += stride) {
    const float4 x = src[i];
    float4 h, l;
    h.x = __uint_as_float(__float_as_uint(x.x) & 0xFFFFE000u);
    h.y = __uint_as_float(__float_as_uint(x.y) & 0xFFFFE000u);
    h.z = __uint_as_float(__float_as_uint(x.z) & 0xFFFFE000u);
    h.w = __uint_as_float(__float_as_uint(x.w) & 0xFFFFE000u);
    l.x = x.x - h.x;
    l.y = x.y - h.y;
    l.z = x.z - h.z;
    l.w = x.w - h.w;
    hi[i] = h;
    lo[i] = l;
  }
}

// Split-K finalisation: C = act(alpha * sum_s W[s] + beta * P), summed in
// split order so the result does not depend on scheduling.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(
    const float* __restrict__ ws, int splits, const float* __restrict__ bias,
    float* __restrict__ c, int64_t m, int64_t n, int64_t ldc, float alpha, float beta, int act,
    int use_prev) {
  const int64_t total = m * n;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const int64_t r = i / n, col = i - (i / n) * n;
    float acc = ws[i];
    for (int s = 1; s < splits; ++s) acc += ws[static_cast<int64_t>(s) * total + i];
    float prev = 0.f;
    if (bias != nullptr) prev = bias[col];
    else if (use_prev) prev = c[r * ldc + col];
    c[r * ldc + col] = epilogue_value(acc, prev, alpha, beta, act);
  }
}

// ---- host side -----------------------------------------------------------------


template <int BN, bool SPLIT3, bool B_NMAJOR, bool GATED = false, bool PROG = false,
          bool TMA_C = false>
int launch_kernel(const Params& p, int grid, cudaStream_t stream, int dev) {
  using Cf = Cfg<BN, SPLIT3>;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  std::call_once(once[dev & 63], [&]() {
    attr_err[dev & 63] =
        cudaFuncSetAttribute(gemm_tc_kernel<BN, SPLIT3, B_NMAJOR, GATED, PROG, TMA_C>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM_BYTES);
  });
  TVR_CUDA_TRY(attr_err[dev & 63]);
  gemm_tc_kernel<BN, SPLIT3, B_NMAJOR, GATED, PROG, TMA_C>
      <<<grid, NUM_THREADS, Cf::SMEM_BYTES, stream>>>(p);
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

__global__ void nvls_epoch_advance_kernel(uint32_t* counter) { *counter += 1; }

// NVLS kernels: one cooperative launch, so that every GEMM and reducer CTA
// is resident at once (the reducers wait for tiles the GEMM CTAs produce).
int launch_nvls(const Params& p, int grid, cudaStream_t stream, int dev) {
  using Cf = Cfg<256, false>;
  auto kernel = gemm_tc_kernel<256, false, false, false, false, true, true>;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  std::call_once(once[dev & 63], [&]() {
    attr_err[dev & 63] =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM_BYTES);
  });
  TVR_CUDA_TRY(attr_err[dev & 63]);
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = Cf::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  memset(attr, 0, sizeof(attr));
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TVR_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, p));
  return TVR_OK;
}

template <int BN>
int launch_bn(const Params& p, bool split3, bool b_nmajor, int grid, cudaStream_t s, int dev,
              bool prog = false, bool tma_c = false) {
  if constexpr (BN == 192) {
    // TF32 with a K-major weight only (the tile width gemm_tcgen05 picks for
    // N = 768-like outputs)
    if (split3 || b_nmajor) return fail(TVR_ERR_INVALID, "gemm: 192-wide tiles are TF32 K-major");
    if (prog) return launch_kernel<BN, false, false, false, true>(p, grid, s, dev);
    if (tma_c) return launch_kernel<BN, false, false, false, false, true>(p, grid, s, dev);
    return launch_kernel<BN, false, false>(p, grid, s, dev);
  }
  if constexpr (BN <= 128) {
    if (split3) {
      if (prog) return launch_kernel<BN, true, false, false, true>(p, grid, s, dev);
      if (tma_c) {
        return b_nmajor ? launch_kernel<BN, true, true, false, false, true>(p, grid, s, dev)
                        : launch_kernel<BN, true, false, false, false, true>(p, grid, s, dev);
      }
      return b_nmajor ? launch_kernel<BN, true, true>(p, grid, s, dev)
                      : launch_kernel<BN, true, false>(p, grid, s, dev);
    }
  } else {
    if (split3) return fail(TVR_ERR_INVALID, "gemm: 3xTF32 tiles are at most 128 columns wide");
  }
  if (prog) return launch_kernel<BN, false, false, false, true>(p, grid, s, dev);  // K-major only
  if (tma_c) {
    return b_nmajor ? launch_kernel<BN, false, true, false, false, true>(p, grid, s, dev)
                    : launch_kernel<BN, false, false, false, false, true>(p, grid, s, dev);
  }
  return b_nmajor ? launch_kernel<BN, false, true>(p, grid, s, dev)
                  : launch_kernel<BN, false, false>(p, grid, s, dev);
}

// Writes hi / lo parts of a [batch][rows][cols] operand (row stride ld,
// batch stride bs) densely packed with row stride ld_out.
int split_operand(const float* src, float* hi, float* lo, int64_t rows, int64_t cols,
                  int64_t ld, int64_t bs, int64_t ld_out, int64_t batch, cudaStream_t s,
                  int dev) {
  const int64_t total = rows * cols * batch;
  if (total == 0) return TVR_OK;
  const bool dense = ld == cols && ld_out == cols && (batch == 1 || bs == rows * cols);
  if (dense && total % 4 == 0 && al16(src) && al16(hi) && al16(lo)) {
    split_tf32_vec4_kernel<<<elementwise_grid(total / 4, 256, dev), 256, 0, s>>>(
        reinterpret_cast<const float4*>(src), reinterpret_cast<float4*>(hi),
        reinterpret_cast<float4*>(lo), total / 4);
  } else {
    split_tf32_kernel<<<elementwise_grid(total, 256, dev), 256, 0, s>>>(src, hi, lo, rows, cols,
                                                                         ld, bs, ld_out, batch);
  }
  TVR_LAUNCH_CHECK();
  return TVR_OK;
}

// Per-device cap on the persistent kernel's grid (tvr_set_gemm_sm_limit).
std::atomic<int> g_sm_limit[64];

int grid_sms(int dev, int sms) {
  const int lim = g_sm_limit[dev & 63].load(std::memory_order_relaxed);
  return lim > 0 && lim < sms ? lim : sms;
}

}  // namespace tc

int gemm_tcgen05(const float* a, const float* b, const float* bias, float* c, int64_t m,
                 int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int64_t batch,
                 int64_t sa, int64_t sb, int64_t sc, float alpha, float beta, int act,
                 bool trans_b, bool split3, cudaStream_t stream, const EpiProg* prog) {
  using namespace tc;
  // TMA addressability: 16-byte aligned bases, row and batch strides in
  // multiples of 16 bytes, extents that fit the 32-bit coordinates.
  const bool b_bcast = batch > 1 && sb == 0;
  if (!al16(a) || !al16(b) || lda % 4 != 0 || ldb % 4 != 0 || k < 1 ||
      (batch > 1 && (sa == 0 || sa % 4 != 0)) || (batch > 1 && !b_bcast && sb % 4 != 0) ||
      m > 0x7fffff00 || n > 0x7fffff00 || k > 0x7fffff00 || batch > 65535) {
    return TVR_ERR_UNSUPPORTED;
  }
  const int dev = current_device();
  const int sms = sm_count(dev);
  const int num_kb = static_cast<int>(ceil_div(k, BK));

  // Tile width: the widest BN (not wider than N rounded up) that still gives
  // ~a full wave of tiles; otherwise split K across CTAs.
  int bn = 64;
  int64_t tiles = 0;
  // (3xTF32 tiles keep a chunk running sum in tensor memory: at most 128 wide)
  const int bn_cap = n > 128 && !split3 ? 256 : (n > 64 ? 128 : 64);
  for (int cand : {256, 128, 64}) {
    if (cand > bn_cap) continue;
    const int64_t t = batch * ceil_div(m, BM) * ceil_div(n, cand);
    bn = cand;
    tiles = t;
    if (t >= (sms * 4) / 5) break;
  }
  // A 192-wide tile where it cuts the wave-quantised time of the tiles by
  // more than 15 % (time ~ waves x tile width).  N = 768 at M = 8192: 192
  // tiles of 256 take two waves on 148 SMs, 256 tiles of 192 two waves of
  // three-quarter-size tiles.  Only with a full wave of 256-wide tiles:
  // fewer tiles split K instead (below), which balances them better.
  if (bn == 256 && !split3 && trans_b && batch == 1 && tiles >= (sms * 4) / 5) {
    const int64_t t192 = ceil_div(m, BM) * ceil_div(n, 192);
    const int64_t w256 = ceil_div(tiles, sms), w192 = ceil_div(t192, sms);
    if (w192 * 192 * 100 < w256 * 256 * 85) {
      bn = 192;
      tiles = t192;
    }
  }
  const bool c_vec = al16(c) && ldc % 4 == 0 && (batch == 1 || sc % 4 == 0);
  int splits = 1;
  if (batch == 1 && tiles < (sms * 4) / 5) {
    int s = static_cast<int>(sms / tiles);
    s = std::min(s, std::max(1, num_kb / 4));
    s = std::min(s, 16);
    if (s > 1) splits = s;
  }
  int kb_per_split = static_cast<int>(ceil_div(num_kb, splits));
  splits = static_cast<int>(ceil_div(num_kb, kb_per_split));

  Params p;
  memset(&p, 0, sizeof(p));
  Scratch split_a, split_b, workspace;
  const float* a_hi = a;
  const float* b_hi = b;
  const float* a_lo = nullptr;
  const float* b_lo = nullptr;
  int64_t lda_u = lda, ldb_u = ldb, sa_u = sa, sb_u = sb;
  const int64_t b_rows = trans_b ? n : k;  // B stored as [b_rows][b_cols]
  const int64_t b_cols = trans_b ? k : n;
  const int64_t b_batches = b_bcast ? 1 : batch;
  int rc;
  if (split3) {
    const int64_t lda_p = (k + 3) / 4 * 4;
    const int64_t ldb_p = (b_cols + 3) / 4 * 4;
    const size_t a_elems = static_cast<size_t>(batch * m * lda_p);
    const size_t b_elems = static_cast<size_t>(b_batches * b_rows * ldb_p);
    if ((rc = split_a.alloc(2 * a_elems * sizeof(float), dev, stream)) != TVR_OK) return rc;
    if ((rc = split_b.alloc(2 * b_elems * sizeof(float), dev, stream)) != TVR_OK) return rc;
    float* ah = static_cast<float*>(split_a.ptr);
    float* al = ah + a_elems;
    float* bh = static_cast<float*>(split_b.ptr);
    float* bl = bh + b_elems;
    if ((rc = split_operand(a, ah, al, m, k, lda, sa, lda_p, batch, stream, dev)) != TVR_OK) return rc;
    if ((rc = split_operand(b, bh, bl, b_rows, b_cols, ldb, sb, ldb_p, b_batches, stream, dev)) != TVR_OK)
      return rc;
    a_hi = ah;
    a_lo = al;
    b_hi = bh;
    b_lo = bl;
    lda_u = lda_p;
    ldb_u = ldb_p;
    sa_u = m * lda_p;
    sb_u = b_rows * ldb_p;
  }
  // A: dims {K, M, batch}
  const uint64_t a_bs = static_cast<uint64_t>(batch > 1 ? sa_u : m * lda_u) * 4;
  if ((rc = encode_3d(&p.tma_a, a_hi, k, m, batch, lda_u * 4, a_bs ? a_bs : 16, BK, BM)) != TVR_OK)
    return rc;
  if (split3 &&
      (rc = encode_3d(&p.tma_a_lo, a_lo, k, m, batch, lda_u * 4, a_bs ? a_bs : 16, BK, BM)) != TVR_OK)
    return rc;
  const uint64_t b_bs =
      static_cast<uint64_t>((b_batches > 1) ? sb_u : b_rows * ldb_u) * 4;
  if (trans_b) {
    if ((rc = encode_3d(&p.tma_b, b_hi, k, n, b_batches, ldb_u * 4, b_bs ? b_bs : 16, BK, bn)) != TVR_OK)
      return rc;
    if (split3 &&
        (rc = encode_3d(&p.tma_b_lo, b_lo, k, n, b_batches, ldb_u * 4, b_bs ? b_bs : 16, BK, bn)) != TVR_OK)
      return rc;
  } else {
    // N-major tiles use the 32-byte-chunk swizzle the N-major tf32 MMA reads
    constexpr CUtensorMapSwizzle kSw = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    if ((rc = encode_3d(&p.tma_b, b_hi, n, k, b_batches, ldb_u * 4, b_bs ? b_bs : 16, 32, BK,
                        kSw)) != TVR_OK)
      return rc;
    if (split3 && (rc = encode_3d(&p.tma_b_lo, b_lo, n, k, b_batches, ldb_u * 4,
                                  b_bs ? b_bs : 16, 32, BK, kSw)) != TVR_OK)
      return rc;
  }
  float* out = c;
  int64_t out_ld = ldc, out_bs = sc;
  int out_vec = c_vec ? 1 : 0;
  if (splits > 1) {
    const size_t ws_elems = static_cast<size_t>(splits) * m * n;
    if ((rc = workspace.alloc(ws_elems * sizeof(float), dev, stream)) != TVR_OK) return rc;
    out = static_cast<float*>(workspace.ptr);
    out_ld = n;
    out_bs = m * n;
    out_vec = n % 4 == 0 ? 1 : 0;
  }
  p.bias = bias;
  p.c = out;
  p.ldc = out_ld;
  p.stride_c = out_bs;
  p.alpha = alpha;
  p.beta = beta;
  p.act = act;
  p.use_prev = (bias == nullptr && beta != 0.f) ? 1 : 0;
  p.c_vec = out_vec;
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.batch = static_cast<int>(batch);
  p.b_broadcast = b_bcast ? 1 : 0;
  p.tiles_m = static_cast<int>(ceil_div(m, BM));
  p.tiles_n = static_cast<int>(ceil_div(n, bn));
  // panels over one split's K: 3xTF32 streams hi and lo parts
  {
    const int64_t kk = static_cast<int64_t>(kb_per_split) * BK * 4 * (split3 ? 2 : 1);
    pick_raster(p, BM * kk, bn * kk);
  }
  p.splits = splits;
  p.kb_per_split = kb_per_split;
  p.num_kb = num_kb;
  p.kchunk = SPLIT3_KCHUNK;
  const int64_t units = static_cast<int64_t>(batch) * splits * p.tiles_m * p.tiles_n;
  if (units > 0x7fffffff) return TVR_ERR_UNSUPPORTED;
  p.total_units = static_cast<int>(units);
  p.status = device_status_ptr(dev);
  const int grid = static_cast<int>(std::min<int64_t>(units, grid_sms(dev, sms)));
  const bool b_nmajor = !trans_b;
  // A pointwise program runs in the epilogue when each output element is
  // final there (no split-K, one batch entry, K-major weights); otherwise it
  // runs as a pass over the finished output.
  const bool has_prog = prog != nullptr && prog->n_nodes > 0;
  // Output through TMA stores: whole-K tiles whose output is not read back,
  // describable by a tensor map (16-byte aligned rows and batches), and at
  // least one 32 x 32 box wide.  A program runs in the epilogue only then.
  const bool tma_ok = splits == 1 && p.use_prev == 0 && c_vec && n >= 32 && m >= 32 &&
                      ldc <= (int64_t(1) << 36) / 4;
  // The commonest program, a residual add (Load y, Load r, Add with alpha 1,
  // r a full row-major matrix with 16-byte aligned rows), runs natively in
  // the TMA-store epilogue instead of as stack code.
  const bool resid_native =
      has_prog && tma_ok && batch == 1 && epi_is_residual_add(*prog) && prog->vec[0] != 0;
  if (resid_native) {
    p.resid = prog->in[0];
    p.resid_ld = prog->ld[0];
  }
  const bool prog_in_kernel =
      has_prog && !resid_native && tma_ok && batch == 1 && trans_b && prog->n_ops > 0;
  if (prog_in_kernel) p.prog = *prog;
  const bool tma_c = tma_ok && (!has_prog || resid_native);
  if (tma_c || prog_in_kernel) {
    const uint64_t c_bs = static_cast<uint64_t>(batch > 1 ? sc : m * ldc) * 4;
    if ((rc = encode_3d(&p.tma_c, c, n, m, batch, ldc * 4, c_bs ? c_bs : 16, 32, 32)) != TVR_OK)
      return rc;
  }
  switch (bn) {
    case 256:
      rc = launch_bn<256>(p, split3, b_nmajor, grid, stream, dev, prog_in_kernel, tma_c);
      break;
    case 192:
      rc = launch_bn<192>(p, split3, b_nmajor, grid, stream, dev, prog_in_kernel, tma_c);
      break;
    case 128:
      rc = launch_bn<128>(p, split3, b_nmajor, grid, stream, dev, prog_in_kernel, tma_c);
      break;
    default: rc = launch_bn<64>(p, split3, b_nmajor, grid, stream, dev, prog_in_kernel, tma_c); break;
  }
  if (rc != TVR_OK) return rc;
  if (splits > 1) {
    splitk_reduce_kernel<<<elementwise_grid(m * n, 256, dev), 256, 0, stream>>>(
        out, splits, bias, c, m, n, ldc, alpha, beta, act, p.use_prev);
    TVR_LAUNCH_CHECK();
  }
  if (has_prog && !prog_in_kernel && !resid_native) {
    return epi_prog_inplace(*prog, c, ldc, m, n, stream);
  }
  return TVR_OK;
}

}  // namespace tvr

// ---- gated (SwiGLU) GEMM ----------------------------------------------------------

namespace tvr {

// out[m, n] = silu(x . Wg^T) * (x . Wu^T) in one TF32 tcgen05 pass: each
// 128 x 256 accumulator tile holds 128 gate and the matching 128 up columns.
// Returns TVR_ERR_UNSUPPORTED when the operands cannot be described by TMA maps.
int gemm_tcgen05_swiglu(const float* x, const float* wg, const float* wu, float* out, int64_t m,
                        int64_t n, int64_t k, int64_t ldx, int64_t ldwg, int64_t ldwu,
                        int64_t ldo, cudaStream_t stream) {
  using namespace tc;
  if (!al16(x) || !al16(wg) || !al16(wu) || ldx % 4 != 0 || ldwg % 4 != 0 || ldwu % 4 != 0 ||
      k < 1 || m > 0x7fffff00 || n > 0x7fffff00 || k > 0x7fffff00) {
    return TVR_ERR_UNSUPPORTED;
  }
  const int dev = current_device();
  const int sms = sm_count(dev);
  constexpr int kOutBn = 128;
  Params p;
  memset(&p, 0, sizeof(p));
  int rc;
  if ((rc = encode_3d(&p.tma_a, x, k, m, 1, ldx * 4, m * ldx * 4, BK, BM)) != TVR_OK) return rc;
  if ((rc = encode_3d(&p.tma_b, wg, k, n, 1, ldwg * 4, n * ldwg * 4, BK, kOutBn)) != TVR_OK) return rc;
  if ((rc = encode_3d(&p.tma_b_lo, wu, k, n, 1, ldwu * 4, n * ldwu * 4, BK, kOutBn)) != TVR_OK)
    return rc;
  p.bias = nullptr;
  p.c = out;
  p.ldc = ldo;
  p.stride_c = m * ldo;
  p.alpha = 1.f;
  p.beta = 0.f;
  p.act = TVR_ACT_NONE;
  p.use_prev = 0;
  p.c_vec = (al16(out) && ldo % 4 == 0) ? 1 : 0;
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.batch = 1;
  p.tiles_m = static_cast<int>(ceil_div(m, BM));
  p.tiles_n = static_cast<int>(ceil_div(n, kOutBn));
  pick_raster(p, BM * k * 4, 2 * kOutBn * k * 4);  // a B tile: gate and up rows
  p.splits = 1;
  p.num_kb = static_cast<int>(ceil_div(k, BK));
  p.kb_per_split = p.num_kb;
  const int64_t units = static_cast<int64_t>(p.tiles_m) * p.tiles_n;
  if (units > 0x7fffffff) return TVR_ERR_UNSUPPORTED;
  p.total_units = static_cast<int>(units);
  p.status = device_status_ptr(dev);
  const int grid = static_cast<int>(std::min<int64_t>(units, tc::grid_sms(dev, sms)));
  return launch_kernel<256, false, false, true>(p, grid, stream, dev);
}

// C = A . B^T (TF32, K-major B) with C then summed over the ranks through
// NVLink SHARP inside the same kernel (tvr_gemm_nvls_all_reduce_f32).
int gemm_tcgen05_nvls(const float* a, const float* b, float* c, void* c_multicast, int64_t m,
                      int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                      void* const* peer_flags, int rank, int world, uint32_t* epoch,
                      int reduce_ctas, cudaStream_t stream) {
  using namespace tc;
  TVR_CHECK(al16(a) && al16(b) && al16(c) && al16(c_multicast) && lda % 4 == 0 && ldb % 4 == 0 &&
                ldc % 4 == 0 && n % 4 == 0,
            "gemm_nvls_all_reduce: operands need 16-byte aligned bases, row strides and n %% 4 == 0");
  TVR_CHECK(m >= 32 && n >= 32 && k >= 1 && m <= 0x7fffff00 && n <= 0x7fffff00 &&
                k <= 0x7fffff00 && lda >= k && ldb >= k && ldc >= n && ldc <= (int64_t(1) << 34),
            "gemm_nvls_all_reduce: shape (%lld, %lld, %lld) out of range", (long long)m,
            (long long)n, (long long)k);
  const int dev = current_device();
  const int sms = sm_count(dev);
  TVR_CHECK(reduce_ctas >= 1 && reduce_ctas <= TVR_NVLS_MAX_BLOCKS && reduce_ctas < sms,
            "gemm_nvls_all_reduce: %d reducing CTAs (1..%d, fewer than the %d SMs)", reduce_ctas,
            TVR_NVLS_MAX_BLOCKS, sms);
  constexpr int kBn = 256;
  Params p;
  memset(&p, 0, sizeof(p));
  int rc;
  if ((rc = encode_3d(&p.tma_a, a, k, m, 1, lda * 4, m * lda * 4, BK, BM)) != TVR_OK) return rc;
  if ((rc = encode_3d(&p.tma_b, b, k, n, 1, ldb * 4, n * ldb * 4, BK, kBn)) != TVR_OK) return rc;
  if ((rc = encode_3d(&p.tma_c, c, n, m, 1, ldc * 4, m * ldc * 4, 32, 32)) != TVR_OK) return rc;
  p.c = c;
  p.ldc = ldc;
  p.stride_c = m * ldc;
  p.alpha = 1.f;
  p.beta = 0.f;
  p.act = TVR_ACT_NONE;
  p.c_vec = 1;
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.batch = 1;
  p.tiles_m = static_cast<int>(ceil_div(m, BM));
  p.tiles_n = static_cast<int>(ceil_div(n, kBn));
  pick_raster(p, BM * k * 4, kBn * k * 4);
  p.splits = 1;
  p.num_kb = static_cast<int>(ceil_div(k, BK));
  p.kb_per_split = p.num_kb;
  const int64_t units = static_cast<int64_t>(p.tiles_m) * p.tiles_n;
  TVR_CHECK(units <= TVR_NVLS_MAX_TILES, "gemm_nvls_all_reduce: %lld output tiles (at most %d)",
            (long long)units, TVR_NVLS_MAX_TILES);
  p.total_units = static_cast<int>(units);
  p.status = device_status_ptr(dev);
  TVR_CHECK(p.status != nullptr, "gemm_nvls_all_reduce: device status word unavailable");
  p.nv_mc = static_cast<float*>(c_multicast);
  for (int r = 0; r < world; ++r) p.nv_flags.flags[r] = static_cast<uint32_t*>(peer_flags[r]);
  p.nv_epoch = epoch;
  p.nv_rank = rank;
  p.nv_world = world;
  p.nv_gemm_ctas = static_cast<int>(std::min<int64_t>(units, sms - reduce_ctas));
  // a fresh epoch for the closing barrier on every call (and every replay of
  // a captured graph)
  nvls_epoch_advance_kernel<<<1, 1, 0, stream>>>(epoch);
  TVR_LAUNCH_CHECK();
  return launch_nvls(p, p.nv_gemm_ctas + reduce_ctas, stream, dev);
}

}  // namespace tvr

// ---- allocation-free variant ----------------------------------------------------
//
// Some callers cannot allocate device memory while they run: a host that
// hands out all device memory itself from a budget fixed at start-up, or an
// embedding runtime that forbids the CUDA allocator once it is serving (an
// allocation can synchronize the device, and its latency is unbounded).
// tvr_gemm_bias_act_noalloc serves them: it is the
// TF32 tensor-core GEMM of tvr_gemm_bias_act whose only scratch — the split-K
// partial sums of skinny problems — lives in the fixed device array below
// instead of coming from tvr_malloc.

namespace tvr {
namespace tc {

// 16 MiB of split-K partial sums (4 Mi fp32).  A __device__ array is part of
// the module: every GPU that loads this library holds it until the process
// exits.  Host code must not use the name as a pointer (on the host it names a
// stand-in object); its device address comes from cudaGetSymbolAddress.
constexpr size_t kNoAllocScratchFloats = size_t(4) << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

constexpr int kNoAllocMaxDevices = 64;
std::once_flag g_noalloc_once[kNoAllocMaxDevices];
float* g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};
cudaError_t g_noalloc_err[kNoAllocMaxDevices];

// Device address of the scratch array on `dev` (the current device), looked
// up once per device.
int noalloc_scratch(int dev, float** out) {
  if (dev < 0 || dev >= kNoAllocMaxDevices) {
    return fail(TVR_ERR_INVALID, "tvr_gemm_bias_act_noalloc: device %d out of range", dev);
  }
  std::call_once(g_noalloc_once[dev], [dev]() {
    void* ptr = nullptr;
    g_noalloc_err[dev] = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (g_noalloc_err[dev] == cudaSuccess) g_noalloc_ptr[dev] = static_cast<float*>(ptr);
  });
  if (g_noalloc_err[dev] != cudaSuccess || g_noalloc_ptr[dev] == nullptr) {
    return fail(TVR_ERR_CUDA, "tvr_gemm_bias_act_noalloc: cudaGetSymbolAddress failed: %s",
                cudaGetErrorString(g_noalloc_err[dev]));
  }
  *out = g_noalloc_ptr[dev];
  return TVR_OK;
}

}  // namespace tc

// TF32 tcgen05 GEMM with split-K partials in the fixed scratch.  Returns
// TVR_ERR_UNSUPPORTED when the operands cannot be described by TMA maps.
int gemm_tcgen05_noalloc(const float* a, const float* b, const float* bias, float* c, int64_t m,
                         int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                         float alpha, float beta, int act, bool trans_b, cudaStream_t stream) {
  using namespace tc;
  if (!al16(a) || !al16(b) || lda % 4 != 0 || ldb % 4 != 0 || k < 1 || m > 0x7fffff00 ||
      n > 0x7fffff00 || k > 0x7fffff00) {
    return TVR_ERR_UNSUPPORTED;
  }
  const int dev = current_device();
  float* scratch = nullptr;
  int rc = noalloc_scratch(dev, &scratch);
  if (rc != TVR_OK) return rc;
  const int sms = sm_count(dev);
  const int num_kb = static_cast<int>(ceil_div(k, BK));
  int bn = 64;
  int64_t tiles = 0;
  const int bn_cap = n > 128 ? 256 : (n > 64 ? 128 : 64);
  for (int cand : {256, 128, 64}) {
    if (cand > bn_cap) continue;
    tiles = ceil_div(m, BM) * ceil_div(n, cand);
    bn = cand;
    if (tiles >= (sms * 4) / 5) break;
  }
  int splits = 1;
  if (tiles < (sms * 4) / 5) {
    int s = static_cast<int>(sms / tiles);
    s = std::min(s, std::max(1, num_kb / 4));
    s = std::min(s, 16);
    if (s > 1) splits = s;
  }
  // the partials of every split must fit the fixed scratch
  while (splits > 1 && static_cast<size_t>(splits) * m * n > kNoAllocScratchFloats) --splits;
  int kb_per_split = static_cast<int>(ceil_div(num_kb, splits));
  splits = static_cast<int>(ceil_div(num_kb, kb_per_split));

  Params p;
  memset(&p, 0, sizeof(p));
  if ((rc = encode_3d(&p.tma_a, a, k, m, 1, lda * 4, static_cast<uint64_t>(m * lda) * 4, BK, BM)) != TVR_OK)
    return rc;
  const int64_t b_rows = trans_b ? n : k;
  const uint64_t b_bs = static_cast<uint64_t>(b_rows * ldb) * 4;
  if (trans_b) {
    if ((rc = encode_3d(&p.tma_b, b, k, n, 1, ldb * 4, b_bs, BK, bn)) != TVR_OK) return rc;
  } else {
    if ((rc = encode_3d(&p.tma_b, b, n, k, 1, ldb * 4, b_bs, 32, BK,
                        CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)) != TVR_OK)
      return rc;
  }
  const bool c_vec = al16(c) && ldc % 4 == 0;
  p.bias = bias;
  p.alpha = alpha;
  p.beta = beta;
  p.act = act;
  p.use_prev = (bias == nullptr && beta != 0.f) ? 1 : 0;
  if (splits > 1) {
    // every element of each split's region is written before it is read, so
    // nothing left in the scratch by an earlier call is ever used
    p.c = scratch;
    p.ldc = n;
    p.stride_c = m * n;
    p.c_vec = n % 4 == 0 ? 1 : 0;
  } else {
    p.c = c;
    p.ldc = ldc;
    p.stride_c = 0;
    p.c_vec = c_vec ? 1 : 0;
  }
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.batch = 1;
  p.b_broadcast = 0;
  p.tiles_m = static_cast<int>(ceil_div(m, BM));
  p.tiles_n = static_cast<int>(ceil_div(n, bn));
  {
    const int64_t kk = static_cast<int64_t>(kb_per_split) * BK * 4;
    pick_raster(p, BM * kk, bn * kk);
  }
  p.splits = splits;
  p.kb_per_split = kb_per_split;
  p.num_kb = num_kb;
  const int64_t units = static_cast<int64_t>(splits) * p.tiles_m * p.tiles_n;
  if (units > 0x7fffffff) return TVR_ERR_UNSUPPORTED;
  p.total_units = static_cast<int>(units);
  p.status = device_status_ptr_if_ready(dev);  // never sets the device up (no allocation)
  // the SM limit of tvr_set_gemm_sm_limit applies here too
  const int grid = static_cast<int>(std::min<int64_t>(units, grid_sms(dev, sms)));
  switch (bn) {
    case 256: rc = launch_bn<256>(p, false, !trans_b, grid, stream, dev); break;
    case 128: rc = launch_bn<128>(p, false, !trans_b, grid, stream, dev); break;
    default: rc = launch_bn<64>(p, false, !trans_b, grid, stream, dev); break;
  }
  if (rc != TVR_OK) return rc;
  if (splits > 1) {
    splitk_reduce_kernel<<<elementwise_grid(m * n, 256, dev), 256, 0, stream>>>(
        scratch, splits, bias, c, m, n, ldc, alpha, beta, act, p.use_prev);
    TVR_LAUNCH_CHECK();
  }
  return TVR_OK;
}

}  // namespace tvr

extern "C" int tvr_gemm_bias_act_noalloc(const float* a, const float* b, const float* bias,
                                         float* c, int64_t m, int64_t n, int64_t k, int64_t lda,
                                         int64_t ldb, int64_t ldc, float alpha, float beta,
                                         int act, int trans_b, void* stream) {
  using namespace tvr;
  TVR_CHECK(m >= 0 && n >= 0 && k >= 0, "gemm: negative size (%lld, %lld, %lld)", (long long)m,
            (long long)n, (long long)k);
  TVR_CHECK(act >= 0 && act <= 2, "gemm: unknown activation %d", act);
  if (m == 0 || n == 0) return TVR_OK;
  TVR_CHECK(static_cast<size_t>(m) * static_cast<size_t>(n) <= tc::kNoAllocScratchFloats,
            "tvr_gemm_bias_act_noalloc: the output has %lld elements; this entry point takes at "
            "most %zu (its fixed 16 MiB scratch); use tvr_gemm_bias_act",
            (long long)(m * n), tc::kNoAllocScratchFloats);
  TVR_CHECK(c != nullptr, "gemm: null output");
  TVR_CHECK(k == 0 || (a != nullptr && b != nullptr), "gemm: null operand");
  TVR_CHECK(lda >= k && ldc >= n, "gemm: leading dimension too small");
  TVR_CHECK(trans_b ? ldb >= k : ldb >= n, "gemm: leading dimension of B too small");
  cudaStream_t s = as_stream(stream);
  // the same size threshold as tvr_gemm_bias_act in TF32 mode: tiny problems
  // run on the CUDA cores, which need no scratch either
  if (m * n * k > (int64_t(1) << 21)) {
    const int rc = gemm_tcgen05_noalloc(a, b, bias, c, m, n, k, lda, ldb, ldc, alpha, beta, act,
                                        trans_b != 0, s);
    if (rc != TVR_ERR_UNSUPPORTED) return rc;
  }
  return gemm_simt(a, b, bias, c, m, n, k, lda, ldb, ldc, 1, 0, 0, 0, alpha, beta, act,
                   trans_b != 0, s);
}

extern "C" int tvr_set_gemm_sm_limit(int device, int max_sms) {
  TVR_CHECK(device >= 0 && device < 64, "tvr_set_gemm_sm_limit: device %d out of range", device);
  TVR_CHECK(max_sms >= 0, "tvr_set_gemm_sm_limit: negative limit");
  tvr::tc::g_sm_limit[device].store(max_sms, std::memory_order_relaxed);
  return TVR_OK;
}

extern "C" int tvr_get_gemm_sm_limit(int device, int* max_sms) {
  TVR_CHECK(device >= 0 && device < 64 && max_sms != nullptr, "tvr_get_gemm_sm_limit: bad argument");
  *max_sms = tvr::tc::g_sm_limit[device].load(std::memory_order_relaxed);
  return TVR_OK;
}

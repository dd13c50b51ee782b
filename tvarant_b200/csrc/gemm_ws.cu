// Weight-streaming tensor-core GEMM for few activation rows (decode steps,
// small batches): C[m, n] = act(alpha * sum_k X[m, k] W[n, k] + beta * P),
// m <= 128, W in nn.Linear layout [N, K].
//
// With so few rows the time is the weight read (N = K = 4096: 64 MB), so the
// kernel is built to stream W once at HBM speed:
//   * operands are swapped relative to gemm_tc: the 128-row side of
//     tcgen05.mma kind::tf32 takes 128 weight rows and the narrow side
//     (MMA N = MB in {16, 32, 64, 128}) takes the activation rows, so no
//     tensor work or shared memory is spent on padding rows of X;
//   * K is split over the S CTAs of a thread-block cluster, grid
//     (S, N / 128), sized to fill the SMs: S <= 8 (the portable cluster
//     size), or up to 16 when the weight has so few 128-row tiles that 8
//     splits leave SMs without a CTA (N = 768: 48 CTAs) and the device can
//     hold all the clusters at once; each CTA streams its 128 x K/S
//     weight panel through a TMA ring and accumulates 128 x MB in TMEM;
//   * the S partial tiles are combined through distributed shared memory:
//     every CTA copies its accumulator into its own shared memory, and after
//     a cluster barrier CTA r sums 1/S of the tile over the S CTAs in the
//     fixed order s = 0..S-1 and applies bias / alpha / beta / activation as
//     the reference's epilogue does (csrc/kernels/host/HostKernels.cpp:130-140).
//     One launch, no global workspace, and a result independent of scheduling.
//   * 3xTF32 mode: kind::tf32 reads the top 19 bits of each fp32 operand, so
//     a staged fp32 tile already is its own hi part; four converter warps
//     write only the lo parts, lo = x - (x with the low 13 mantissa bits
//     cleared): W_lo into a second 128 x 32 tile, X_lo into rows MB..2MB-1 of
//     the X tile.  Two MMAs of N = 2*MB per k-step, W x [X; X_lo] and
//     W_lo x [X; X_lo], give hi*hi + lo*hi in accumulator columns 0..MB-1 and
//     hi*lo + lo*lo in columns MB..2MB-1, added in the epilogue.  The weight
//     still crosses HBM once, and the tensor core reads each weight tile
//     twice instead of three times.
//
// Roles: warp 0 TMA producer, warp 1 TMEM owner and MMA issuer, warps 2-5
// copy the accumulator out of TMEM, warps 6-9 write lo parts (3xTF32); all
// threads take part in the cross-CTA reduction.  Every mbarrier wait is
// bounded as in gemm_tc: an expired wait records a TVR_DEV_* code in the
// device status word, raises the CTA abort flag, and every role still
// reaches both cluster barriers, so no CTA of the cluster is left waiting.
// The waits poll in suspensions of at most 32 ns (a call is a chain of a few
// latency-bound hops, and a plain try_wait woke ~0.37 us after a commit).
// No TMA load uses cluster multicast.
#include "internal.h"

#include <algorithm>
#include <cstring>
#include <mutex>

#include "cluster.cuh"
#include "gemm_common.cuh"
#include "tc_ptx.cuh"

namespace tvr {
namespace ws {

using namespace tc;

constexpr int BM = 128;  // weight rows per tile: the MMA's M
constexpr int BK = 32;   // fp32 per k-block: one 128-byte swizzle row
constexpr int MAX_SPLITS = 16;
constexpr int PORTABLE_SPLITS = 8;

template <int MB, bool SPLIT3>
struct Cfg {
  static constexpr int W_BYTES = BM * BK * 4;
  static constexpr int X_ROWS = SPLIT3 ? 2 * MB : MB;  // 3xTF32: X then X_lo
  static constexpr int X_BYTES = X_ROWS * BK * 4;
  static constexpr int LOAD_BYTES = W_BYTES + MB * BK * 4;  // what TMA brings per stage
  // stage: W | X tile | W_lo (3xTF32)
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES + (SPLIT3 ? W_BYTES : 0);
  static constexpr int NACC = SPLIT3 ? 2 * MB : MB;  // MMA N = accumulator columns
  // Two CTAs per SM while a stage is small enough for three of them in
  // half the shared memory.
  static constexpr int CTAS_PER_SM = STAGE_BYTES <= 36 * 1024 ? 2 : 1;
  static constexpr int BUDGET = CTAS_PER_SM == 2 ? 110 * 1024 : 220 * 1024;
  static constexpr int STAGES_FIT = (BUDGET - 2048) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int RED_BYTES = MB * BM * 4;  // partial tile, aliases the ring
  static constexpr int TMEM_COLS = NACC < 32 ? 32 : NACC;
  static constexpr int CONV_WARPS = SPLIT3 ? 4 : 0;
  static constexpr int THREADS = 32 * (6 + CONV_WARPS);
  static constexpr int BAR_BYTES = 8 * (3 * STAGES + 2) + 8;
  static constexpr int SMEM_BYTES = 1024 + RING_BYTES + BAR_BYTES;
  static_assert(STAGES >= 3, "pipeline depth");
  static_assert(RED_BYTES <= RING_BYTES, "partial tile must fit in the ring");
  static_assert(SMEM_BYTES <= BUDGET + 1024, "shared memory budget");
  static_assert(MB == 16 || MB == 32 || MB == 64 || MB == 128, "MMA N");
  static_assert(STAGE_BYTES % 1024 == 0 && X_BYTES % 1024 == 0, "swizzle atom alignment");
};

struct Params {
  CUtensorMap tma_w;  // W: dims {K, N}, box {32, 128}
  CUtensorMap tma_x;  // X: dims {K, M}, box {32, MB}
  const float* bias;
  float* c;
  int64_t ldc;
  const float* resid;  // non-null: added to the result (a residual stream)
  int64_t resid_ld;
  float alpha;
  float beta;
  int act;
  int use_prev;
  int m, n;
  int num_kb;
  int kb_per_split;
  int* status;
};

__device__ __forceinline__ void st_shared(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ float4 ld_shared4(uint32_t addr) {
  float4 x;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(x.x), "=f"(x.y), "=f"(x.z), "=f"(x.w)
               : "r"(addr));
  return x;
}

// lo = x - (x with the low 13 mantissa bits cleared): the part of an fp32
// value that kind::tf32 does not read.
__device__ __forceinline__ float4 tf32_lo(float4 x) {
  float4 l;
  l.x = x.x - __uint_as_float(__float_as_uint(x.x) & 0xFFFFE000u);
  l.y = x.y - __uint_as_float(__float_as_uint(x.y) & 0xFFFFE000u);
  l.z = x.z - __uint_as_float(__float_as_uint(x.z) & 0xFFFFE000u);
  l.w = x.w - __uint_as_float(__float_as_uint(x.w) & 0xFFFFE000u);
  return l;
}

__device__ __forceinline__ void st_shared4(uint32_t addr, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

template <int MB, bool SPLIT3>
__global__ void __launch_bounds__(Cfg<MB, SPLIT3>::THREADS, Cfg<MB, SPLIT3>::CTAS_PER_SM)
    gemm_ws_kernel(const __grid_constant__ Params p) {
  using Cf = Cfg<MB, SPLIT3>;
  constexpr int STAGES = Cf::STAGES;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_abort;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t ring = base;  // [STAGES][W 128x32 | X X_ROWSx32 | W_lo 128x32]
  const uint32_t bar0 = base + Cf::RING_BYTES;
  const uint32_t full_bar = bar0;                  // [STAGES] TMA landed
  const uint32_t conv_bar = bar0 + 8 * STAGES;     // [STAGES] hi / lo written
  const uint32_t empty_bar = bar0 + 16 * STAGES;   // [STAGES] MMAs done with the slot
  const uint32_t tfull_bar = bar0 + 24 * STAGES;   // accumulator complete
  const uint32_t drain_bar = tfull_bar + 8;
  const uint32_t holder = drain_bar + 8;
  uint32_t* holder_ptr = reinterpret_cast<uint32_t*>(smem_raw + (holder - raw));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const volatile int* abort_flag = &s_abort;
  const uint32_t split = cluster_rank();
  const uint32_t nsplit = cluster_size();
  const int tile = blockIdx.y;
  const int kb0 = static_cast<int>(split) * p.kb_per_split;
  const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar + 8 * s, 1);
      mbar_init(conv_bar + 8 * s, Cf::CONV_WARPS > 0 ? Cf::CONV_WARPS : 1);
      mbar_init(empty_bar + 8 * s, 1);
    }
    mbar_init(tfull_bar, 1);
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
  // a programmatic dependent (the next few-row GEMM) may start its own
  // weight prefetch now; it still waits for this grid before reading anything
  if (threadIdx.x == 0) grid_launch_dependents();

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0;
      uint32_t issued_parity = 0;
      bool ok = true;
      {
        // Launched as a programmatic dependent: the kernel before this one
        // on the stream may still run.  The weight panel's first k-blocks
        // start moving from HBM into L2 now; nothing is read into shared
        // memory until that kernel has completed, so a weight it writes is
        // still read as written.
        const int n_pre = min(2 * STAGES, kb1 - kb0);
        for (int i = 0; i < n_pre; ++i) tma_prefetch_l2_3d(&p.tma_w, (kb0 + i) * BK, tile * BM, 0);
        grid_dependency_wait();
      }
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_poll(empty_bar + 8 * stage, phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t fb = full_bar + 8 * stage;
        mbar_expect_tx(fb, Cf::LOAD_BYTES);
        const uint32_t sw = ring + stage * Cf::STAGE_BYTES;
        tma_load_3d(sw, &p.tma_w, fb, kb * BK, tile * BM, 0);
        tma_load_3d(sw + Cf::W_BYTES, &p.tma_x, fb, kb * BK, 0, 0);
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) {
        record_status(p.status, TVR_DEV_TIMEOUT_PRODUCER);
        *const_cast<volatile int*>(abort_flag) = 1;
      }
      for (int st = 0; st < STAGES; ++st) {
        if ((issued_mask & (1u << st)) &&
            !mbar_wait_poll(full_bar + 8 * st, (issued_parity >> st) & 1u, nullptr)) {
          record_status(p.status, TVR_DEV_TIMEOUT_DRAIN);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(BM, Cf::NACC, false);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool issued = false;
      for (int kb = kb0; kb < kb1; ++kb) {
        const uint32_t ready = (SPLIT3 ? conv_bar : full_bar) + 8 * stage;
        if (!mbar_wait_poll(ready, phase, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sw = ring + stage * Cf::STAGE_BYTES;
        const uint32_t sx = sw + Cf::W_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint64_t dw = desc_kmajor(sw + kk * 32);
          const uint64_t dx = desc_kmajor(sx + kk * 32);
          const uint32_t accumulate = (kb > kb0 || kk > 0) ? 1u : 0u;
          if (SPLIT3) {
            const uint64_t dw_lo = desc_kmajor(sx + Cf::X_BYTES + kk * 32);
            mma_tf32(tmem_base, dw_lo, dx, idesc, accumulate);
            mma_tf32(tmem_base, dw, dx, idesc, 1u);
          } else {
            mma_tf32(tmem_base, dw, dx, idesc, accumulate);
          }
        }
        issued = true;
        mma_commit(empty_bar + 8 * stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) {
        mma_commit(tfull_bar);
      } else {
        record_status(p.status, TVR_DEV_TIMEOUT_MMA);
        *const_cast<volatile int*>(abort_flag) = 1;
      }
      if (issued) {
        mma_commit(drain_bar);
        if (!mbar_wait_poll(drain_bar, 0, nullptr)) record_status(p.status, TVR_DEV_TIMEOUT_DRAIN);
      }
    }
    __syncwarp();
  } else if (warp >= 6) {
    // ------------------------------ lo converters ------------------------------
    // The swizzle permutes 16-byte chunks within a row by the row index mod 8,
    // identical for row r and row r + MB (MB is a multiple of 8), so a chunk's
    // lo part goes to the same offset in the W_lo tile, or MB rows further
    // down in the X tile.
    if constexpr (SPLIT3) {
      const int ct = threadIdx.x - 6 * 32;
      constexpr int W_VEC = Cf::W_BYTES / 16 / 128;       // float4 per thread
      constexpr int X_VEC = MB * BK * 4 / 16 / 128;
      static_assert(W_VEC * 128 * 16 == Cf::W_BYTES, "converter share");
      static_assert(X_VEC * 128 * 16 == MB * BK * 4, "converter share");
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        const bool got = mbar_wait_poll(full_bar + 8 * stage, phase, abort_flag);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        const uint32_t sw = ring + stage * Cf::STAGE_BYTES;
        const uint32_t sx = sw + Cf::W_BYTES;
        const uint32_t sw_lo = sx + Cf::X_BYTES;
        float4 w[W_VEC], x[X_VEC];
#pragma unroll
        for (int i = 0; i < W_VEC; ++i) w[i] = ld_shared4(sw + 16u * static_cast<uint32_t>(ct + 128 * i));
#pragma unroll
        for (int i = 0; i < X_VEC; ++i) x[i] = ld_shared4(sx + 16u * static_cast<uint32_t>(ct + 128 * i));
#pragma unroll
        for (int i = 0; i < W_VEC; ++i) st_shared4(sw_lo + 16u * static_cast<uint32_t>(ct + 128 * i), tf32_lo(w[i]));
#pragma unroll
        for (int i = 0; i < X_VEC; ++i)
          st_shared4(sx + MB * BK * 4 + 16u * static_cast<uint32_t>(ct + 128 * i), tf32_lo(x[i]));
        // generic-proxy writes become visible to the tensor core's reads
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(conv_bar + 8 * stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok && lane == 0) {
        record_status(p.status, TVR_DEV_TIMEOUT_CONVERT);
        *const_cast<volatile int*>(abort_flag) = 1;
      }
    }
    __syncwarp();
  } else {
    // --------------------- accumulator -> shared memory ---------------------
    // Warp w may read TMEM lanes 32*(w % 4) .. +31: weight rows of the tile.
    // Row t's MB values go to red[j * 128 + t] (the ring is free by now:
    // every landed stage has been consumed by the MMAs).  In 3xTF32 mode
    // value j is the sum of accumulator columns j and MB + j.
    const int q = warp & 3;
    const bool got = mbar_wait_poll(tfull_bar, 0, abort_flag);
    if (__all_sync(0xffffffffu, got)) {
      tc_fence_after();
      const int t = 32 * q + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(32 * q) << 16);
      if constexpr (SPLIT3 && MB == 16) {
        float v[32];
        tmem_load_32_async(taddr, v);
        tmem_wait_loads();
#pragma unroll
        for (int j = 0; j < 16; ++j) st_shared(ring + 4u * static_cast<uint32_t>(j * BM + t), v[j] + v[16 + j]);
      } else {
#pragma unroll
        for (int c0 = 0; c0 < MB; c0 += 32) {
          float v[32];
          tmem_load_32_async(taddr + c0, v);
          if constexpr (SPLIT3) {
            float u[32];
            tmem_load_32_async(taddr + MB + c0, u);
            tmem_wait_loads();
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] += u[j];
          } else {
            tmem_wait_loads();
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (c0 + j < MB) st_shared(ring + 4u * static_cast<uint32_t>((c0 + j) * BM + t), v[j]);
          }
        }
      }
    } else if (lane == 0) {
      record_status(p.status, TVR_DEV_TIMEOUT_EPILOGUE);
      *const_cast<volatile int*>(abort_flag) = 1;
    }
    __syncwarp();
  }

  // ---------------- cross-CTA reduction through distributed shared memory ----------------
  tc_fence_before();
  cluster_sync();  // every CTA's partial tile is in its shared memory
  constexpr int E = MB * BM;
  const int share = (E + static_cast<int>(nsplit) - 1) / static_cast<int>(nsplit);
  const int e0 = static_cast<int>(split) * share;
  const int e1 = min(E, e0 + share);
  for (int e = e0 + static_cast<int>(threadIdx.x); e < e1; e += Cf::THREADS) {
    const int row = e / BM;
    const int col = tile * BM + (e % BM);
    if (row >= p.m || col >= p.n) continue;
    const uint32_t local = ring + 4u * static_cast<uint32_t>(e);
    // every partial in flight at once, then summed in the fixed order
    // s = 0..S-1: one remote round trip per element instead of S dependent ones
    float part[MAX_SPLITS];
#pragma unroll
    for (int s = 0; s < MAX_SPLITS; ++s) {
      part[s] = s < static_cast<int>(nsplit) ? ld_dsmem(dsmem_addr(local, static_cast<uint32_t>(s))) : 0.f;
    }
    float sum = 0.f;
#pragma unroll
    for (int s = 0; s < MAX_SPLITS; ++s) {
      if (s < static_cast<int>(nsplit)) sum += part[s];
    }
    float* dst = p.c + static_cast<int64_t>(row) * p.ldc + col;
    float prev = 0.f;
    if (p.bias != nullptr) prev = __ldg(p.bias + col);
    else if (p.use_prev) prev = *dst;
    float v = epilogue_value(sum, prev, p.alpha, p.beta, p.act);
    if (p.resid != nullptr) v = __fadd_rn(v, p.resid[static_cast<int64_t>(row) * p.resid_ld + col]);
    *dst = v;
  }
  cluster_sync();  // no CTA leaves while another still reads its shared memory
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(Cf::TMEM_COLS)
                 : "memory");
  }
}

// How many clusters of `splits` CTAs of this kernel the device holds at once
// (cudaOccupancyMaxActiveClusters; 0 when it cannot launch them), cached per
// device and cluster size.  Sizes above 8 are non-portable: they depend on
// how many SMs a GPC has free.
template <int MB, bool SPLIT3>
int resident_clusters(int splits, int dev) {
  using Cf = Cfg<MB, SPLIT3>;
  static std::mutex mu;
  static int cache[64][MAX_SPLITS + 1];
  static bool known[64][MAX_SPLITS + 1];
  std::lock_guard<std::mutex> lock(mu);
  if (known[dev & 63][splits]) return cache[dev & 63][splits];
  int n = 0;
  cudaError_t e = cudaSuccess;
  if (splits > PORTABLE_SPLITS) {
    e = cudaFuncSetAttribute(gemm_ws_kernel<MB, SPLIT3>,
                             cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  }
  if (e == cudaSuccess) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(static_cast<unsigned>(splits), 1, 1);
    cfg.blockDim = dim3(Cf::THREADS, 1, 1);
    cfg.dynamicSmemBytes = Cf::SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    memset(attr, 0, sizeof(attr));
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaOccupancyMaxActiveClusters(&n, gemm_ws_kernel<MB, SPLIT3>, &cfg);
  }
  if (e != cudaSuccess) {
    (void)cudaGetLastError();  // a refused size is an answer, not a sticky error
    n = 0;
  }
  cache[dev & 63][splits] = n;
  known[dev & 63][splits] = true;
  return n;
}

template <int MB, bool SPLIT3>
int launch(Params& p, int tiles, int sms, cudaStream_t stream, int dev) {
  using Cf = Cfg<MB, SPLIT3>;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  std::call_once(once[dev & 63], [&]() {
    attr_err[dev & 63] = cudaFuncSetAttribute(gemm_ws_kernel<MB, SPLIT3>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              Cf::SMEM_BYTES);
  });
  TVR_CUDA_TRY(attr_err[dev & 63]);
  // Splits of K per tile: as many as keep every CTA resident in one wave.
  const int slots = sms * Cf::CTAS_PER_SM;
  auto split_k = [&](int cap) {
    const int s = std::max(1, std::min({slots / tiles, cap, p.num_kb}));
    p.kb_per_split = static_cast<int>(ceil_div(p.num_kb, s));
    return static_cast<int>(ceil_div(p.num_kb, p.kb_per_split));  // no empty split
  };
  // More than 8 splits only for weights so narrow that 8 splits leave SMs
  // without a CTA (N = 768: 6 tiles, 48 CTAs), and only when the device holds
  // every cluster at once.
  int splits = split_k(tiles * PORTABLE_SPLITS <= sms ? MAX_SPLITS : PORTABLE_SPLITS);
  if (splits > PORTABLE_SPLITS && resident_clusters<MB, SPLIT3>(splits, dev) < tiles) {
    splits = split_k(PORTABLE_SPLITS);
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(static_cast<unsigned>(splits), static_cast<unsigned>(tiles), 1);
  cfg.blockDim = dim3(Cf::THREADS, 1, 1);
  cfg.dynamicSmemBytes = Cf::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  memset(attr, 0, sizeof(attr));
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  TVR_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_ws_kernel<MB, SPLIT3>, p));
  return TVR_OK;
}

template <int MB>
int launch_mb(Params& p, bool split3, int tiles, int sms, cudaStream_t s, int dev) {
  return split3 ? launch<MB, true>(p, tiles, sms, s, dev) : launch<MB, false>(p, tiles, sms, s, dev);
}

}  // namespace ws

bool gemm_ws_applies(const float* x, const float* w, int64_t m, int64_t n, int64_t k,
                     int64_t ldx, int64_t ldw, bool trans_b) {
  using tc::al16;
  return trans_b && m >= 1 && m <= 128 && n >= 1 && k >= 1 && al16(x) && al16(w) &&
         ldx % 4 == 0 && ldw % 4 == 0 && ceil_div(n, ws::BM) <= 65535 && k <= 0x7fffff00;
}

int gemm_ws(const float* x, const float* w, const float* bias, float* c, int64_t m, int64_t n,
            int64_t k, int64_t ldx, int64_t ldw, int64_t ldc, float alpha, float beta, int act,
            bool split3, cudaStream_t stream, const float* resid, int64_t resid_ld) {
  using namespace ws;
  const int dev = current_device();
  const int sms = sm_count(dev);
  const int mb = m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : 128;
  const int tiles = static_cast<int>(ceil_div(n, BM));
  const int num_kb = static_cast<int>(ceil_div(k, BK));

  Params p;
  memset(&p, 0, sizeof(p));
  int rc;
  if ((rc = tc::encode_3d(&p.tma_w, w, k, n, 1, ldw * 4, n * ldw * 4, BK, BM)) != TVR_OK) return rc;
  if ((rc = tc::encode_3d(&p.tma_x, x, k, m, 1, ldx * 4, m * ldx * 4, BK, mb)) != TVR_OK) return rc;
  p.bias = bias;
  p.c = c;
  p.ldc = ldc;
  p.resid = resid;
  p.resid_ld = resid_ld;
  p.alpha = alpha;
  p.beta = beta;
  p.act = act;
  p.use_prev = (bias == nullptr && beta != 0.f) ? 1 : 0;
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.num_kb = num_kb;
  p.status = device_status_ptr(dev);
  switch (mb) {
    case 16: return launch_mb<16>(p, split3, tiles, sms, stream, dev);
    case 32: return launch_mb<32>(p, split3, tiles, sms, stream, dev);
    case 64: return launch_mb<64>(p, split3, tiles, sms, stream, dev);
    default: return launch_mb<128>(p, split3, tiles, sms, stream, dev);
  }
}

}  // namespace tvr

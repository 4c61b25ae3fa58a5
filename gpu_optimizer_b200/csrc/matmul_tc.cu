// C = A @ B on the 5th-generation tensor cores (tcgen05) for sm_100a.
//
// Replaces matmul_kernel (compiler/triton/kernels.py:26-65) for 16-bit and
// tf32 candidates whose BLOCK_M is 64, 128 or 256.  A is M x K row-major
// (K-major operand), B is K x N row-major (MN-major operand, the layout the
// reference passes: runner.py:107 stride_bk = N), C is M x N in A's dtype
// (runner.py:101), fp32 accumulation in TMEM.
//
// Config mapping (one instantiation per (dtype, BLOCK_M, BLOCK_N, warps)):
//   BLOCK_M    : 32  -> the M=64 MMA over A atoms of 64 rows of which TMA
//                fills the tile's 32 (the other 32 rows are never stored:
//                an MMA output row depends only on its own A row), so the
//                epilogue's first two warps store 16 rows each.
//                64  -> one M=64 MMA per K step; D row
//                16g + r sits in TMEM lane 32g + r (g < 4, r < 16), so each
//                epilogue warp stores 16 rows.
//                128 -> one M=128 MMA per K step (matmul_tc_kernel).
//                256 -> a CTA pair (cluster of 2, cta_group::2 M=256 MMAs,
//                each CTA staging 128 rows of A and half of B;
//                matmul_tc2_kernel), persistent with 8 warps.  tf32 with
//                BLOCK_N 32 (a 16-column B half cannot take the 32-bit
//                MN-major swizzle) keeps one CTA with two M=128 MMAs into two
//                TMEM accumulators sharing B.
//   BLOCK_N    : MMA N and TMEM columns per accumulator.
//   BLOCK_K    : K extent of one TMA stage (runtime); the MMA issuer walks it
//                in 32-byte K steps (16 bf16/fp16 or 8 tf32 elements).
//   num_stages : depth of the TMA -> MMA shared-memory ring (runtime).
//   GROUP_M    : grouped tile raster for L2 reuse (runtime), as the
//                reference's program-id swizzle (kernels.py:38-46).
//   num_warps  : 4 -> one output tile per CTA; warp 0 lane 0 issues TMA,
//                warp 1 lane 0 issues MMA, then all 4 warps drain TMEM.
//                8 -> persistent CTA per SM, warp-specialised: warp 0 TMA,
//                warp 1 MMA, warp 2 TMEM owner, warps 4-7 epilogue, with two
//                TMEM accumulator buffers so the epilogue of tile i overlaps
//                the main loop of tile i+1.
//
// Shared-memory operand layouts are the canonical UMMA layouts written by
// TMA with hardware swizzle: A as K-atoms of BLOCK_M rows x S_A bytes
// (S_A = min(BLOCK_K*es, 128)), B as N-chunks of BLOCK_K rows x S_B bytes
// (S_B = min(BLOCK_N*es, 128)).  Out-of-bounds rows / columns of partial
// tiles are zero-filled by TMA, so ragged M, N and K need no special path;
// the epilogue masks the stores.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "gpo_common.cuh"
#include "gpo_internal.h"

namespace gpo {

constexpr int kMaxStages = 8;

struct TcShared {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// TMEM allocation (power of two >= 32 columns) for `cols` accumulator columns.
__host__ __device__ constexpr int tc2_tmem_alloc(int cols) {
  return cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : cols <= 256 ? 256 : 512;
}

__device__ __forceinline__ void tile_coords(int tile, int num_pid_m, int num_pid_n, int group_m,
                                            int& pm, int& pn) {
  const int in_group = group_m * num_pid_n;
  const int gid = tile / in_group;
  const int first_m = gid * group_m;
  const int gsize = min(num_pid_m - first_m, group_m);
  pm = first_m + (tile % gsize);
  pn = (tile % in_group) / gsize;
}

// Work items of a persistent CTA-pair matmul over G clusters.  The tiles
// fill W = T / G whole waves; when the R = T - W*G tiles of the last wave
// leave more than half of the clusters idle (2R <= G), each of them is
// split into two column halves, so the last wave takes the time of half a
// tile instead of a whole one.  Item i < W*G (or every item without a
// split) is tile i; the rest are (tile, half) pairs.
struct Tc2Items {
  int full;   // items that are whole tiles
  int count;  // all items
  __device__ __forceinline__ void at(int item, int& tile, int& half) const {
    if (item < full) {
      tile = item;
      half = -1;
    } else {
      tile = full + (item - full) / 2;
      half = (item - full) & 1;
    }
  }
};

__device__ __forceinline__ Tc2Items tc2_items(int num_tiles, int clusters, bool can_split) {
  const int waves = num_tiles / clusters;
  const int rest = num_tiles - waves * clusters;
  if (can_split && rest > 0 && 2 * rest <= clusters)
    return {waves * clusters, waves * clusters + 2 * rest};
  return {num_tiles, num_tiles};
}

// Issue the MMAs of one K block: KS steps of 32 bytes of K (KS =
// BLOCK_K * es / 32, so the A swizzle width min(KS * 32, 128) is known at
// compile time too).  a0 / b0 are the descriptors of this ring slot at K
// step 0; every other descriptor is a compile-time offset from them, which
// keeps the issuing thread's cost at a few integer ops per MMA -- with
// runtime offset arithmetic the single issuing thread, not the tensor pipe,
// bounded the main loop.  AROWS: A rows per swizzle atom column (the CTA's
// A tile height); HALVES M=128 MMAs per step for 1-CTA BLOCK_M 256.
template <int KS, int ES, int AROWS, int SWB, int HALVES, int BN, int FMT, bool PAIR>
__device__ __forceinline__ void issue_kblock(uint32_t d_tmem, uint64_t a0, uint64_t b0,
                                             uint32_t idesc, bool first) {
  constexpr int SWA = KS * 32 < 128 ? KS * 32 : 128;
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
    const uint32_t kbyte = static_cast<uint32_t>(kk) * 32u;
    const uint32_t a_off = (kbyte / SWA) * (AROWS * SWA) + (kbyte % SWA);
    const uint64_t bdesc = b0 + ((static_cast<uint32_t>(kk) * (32 / ES) * SWB) >> 4);
    const uint32_t acc = (!first || kk > 0) ? 1u : 0u;
#pragma unroll
    for (int h = 0; h < HALVES; ++h) {
      const uint64_t adesc = a0 + ((a_off + h * 128 * SWA) >> 4);
      if constexpr (PAIR) {
        if constexpr (FMT == 2)
          mma_tf32_ss_pair(d_tmem + h * BN, adesc, bdesc, idesc, acc);
        else
          mma_f16_ss_pair(d_tmem + h * BN, adesc, bdesc, idesc, acc);
      } else {
        if constexpr (FMT == 2)
          mma_tf32_ss(d_tmem + h * BN, adesc, bdesc, idesc, acc);
        else
          mma_f16_ss(d_tmem + h * BN, adesc, bdesc, idesc, acc);
      }
    }
  }
}

template <int ES, int AROWS, int SWB, int HALVES, int BN, int FMT, bool PAIR>
__device__ __forceinline__ void issue_kblock_any(int ksteps, uint32_t d_tmem, uint64_t a0,
                                                 uint64_t b0, uint32_t idesc, bool first) {
  switch (ksteps) {
    case 1: issue_kblock<1, ES, AROWS, SWB, HALVES, BN, FMT, PAIR>(d_tmem, a0, b0, idesc, first); break;
    case 2: issue_kblock<2, ES, AROWS, SWB, HALVES, BN, FMT, PAIR>(d_tmem, a0, b0, idesc, first); break;
    case 4: issue_kblock<4, ES, AROWS, SWB, HALVES, BN, FMT, PAIR>(d_tmem, a0, b0, idesc, first); break;
    case 8: issue_kblock<8, ES, AROWS, SWB, HALVES, BN, FMT, PAIR>(d_tmem, a0, b0, idesc, first); break;
    case 16: issue_kblock<16, ES, AROWS, SWB, HALVES, BN, FMT, PAIR>(d_tmem, a0, b0, idesc, first); break;
    default: issue_kblock<32, ES, AROWS, SWB, HALVES, BN, FMT, PAIR>(d_tmem, a0, b0, idesc, first); break;
  }
}

template <typename T, int FMT, int BM, int BN, bool PERSISTENT>
__global__ void __launch_bounds__(PERSISTENT ? 256 : 128, 1)
    matmul_tc_kernel(const __grid_constant__ CUtensorMap tma_a,
                     const __grid_constant__ CUtensorMap tma_b, T* __restrict__ C, int M, int N,
                     int K, int BK, int stages, int group_m, int swa, unsigned int* err) {
  constexpr int ES = sizeof(T);
  constexpr int SWB = (BN * ES) < 128 ? (BN * ES) : 128;
  // BLOCK_M 64: one M=64 MMA per K step; its D rows 16g..16g+15 land in
  // TMEM lanes 32g..32g+15 (g = 0..3), columns as N (measured layout)
  constexpr int AROWS = BM < 64 ? 64 : BM;  // rows of an A atom in shared memory
  constexpr int MMA_M = AROWS < 128 ? AROWS : 128;
  constexpr int HALVES = BM < 128 ? 1 : BM / 128;
  constexpr int COLS = HALVES * BN;  // TMEM columns per accumulator buffer
  constexpr int ACC_STAGES = (PERSISTENT && 2 * COLS <= 512) ? 2 : 1;
  constexpr int ALLOC = (ACC_STAGES * COLS) <= 32    ? 32
                        : (ACC_STAGES * COLS) <= 64  ? 64
                        : (ACC_STAGES * COLS) <= 128 ? 128
                        : (ACC_STAGES * COLS) <= 256 ? 256
                                                     : 512;
  constexpr int KSTEP = 32 / ES;  // K elements per MMA instruction
  constexpr uint32_t IDESC = make_idesc(FMT, MMA_M, BN, false, true);

  __shared__ TcShared sh;
  extern __shared__ uint8_t dyn_smem[];
  const uint32_t smem_base = (smem_u32(dyn_smem) + 1023u) & ~1023u;
  const uint32_t a_bytes = static_cast<uint32_t>(AROWS) * BK * ES;  // shared memory
  const uint32_t a_tx = static_cast<uint32_t>(BM) * BK * ES;         // loaded by TMA
  const uint32_t b_bytes = static_cast<uint32_t>(BK) * BN * ES;
  const uint32_t stage_bytes = (a_bytes + b_bytes + 1023u) & ~1023u;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_pid_m = (M + BM - 1) / BM;
  const int num_pid_n = (N + BN - 1) / BN;
  const int num_tiles = num_pid_m * num_pid_n;
  const int num_kb = (K + BK - 1) / BK;
  const int tile_step = PERSISTENT ? gridDim.x : num_tiles;
  const int alloc_warp = PERSISTENT ? 2 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&sh.full[s]), 1);
      mbar_init(smem_u32(&sh.empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&sh.acc_full[b]), 1);
      mbar_init(smem_u32(&sh.acc_empty[b]), 4);
    }
    mbar_init(smem_u32(&sh.drain), 1);
    sh.abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == alloc_warp) {
    tmem_alloc(smem_u32(&sh.tmem_base), ALLOC);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = sh.tmem_base;
  volatile int* abort_flag = &sh.abort;

  // ------------------------------------------------------------ producer
  if (warp == 0 && lane == 0) {
    int it = 0, s = 0;  // K blocks issued; ring slot and phase of the next one
    uint32_t ph = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += tile_step) {
      int pm, pn;
      tile_coords(tile, num_pid_m, num_pid_n, group_m, pm, pn);
      for (int kb = 0; kb < num_kb; ++kb, ++it) {
        if (!mbar_wait(smem_u32(&sh.empty[s]), ph ^ 1u, abort_flag, err, kErrWaitProducer)) {
          ok = false;
          break;
        }
        const uint32_t full = smem_u32(&sh.full[s]);
        mbar_arrive_expect_tx(full, a_tx + b_bytes);
        const uint32_t sa = smem_base + s * stage_bytes;
        const uint32_t sb = sa + a_bytes;
        const int a_atoms = (BK * ES) / swa;
        for (int a = 0; a < a_atoms; ++a)
          tma_load_2d(sa + a * AROWS * swa, &tma_a, full, kb * BK + a * (swa / ES), pm * BM);
#pragma unroll
        for (int c = 0; c < (BN * ES) / SWB; ++c)
          tma_load_2d(sb + c * BK * SWB, &tma_b, full, pn * BN + c * (SWB / ES), kb * BK);
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
    if (!ok) {
      // drain every load still in flight before the CTA may exit
      for (int j = max(0, it - stages); j < it; ++j)
        mbar_wait_drain(smem_u32(&sh.full[j % stages]), static_cast<uint32_t>(j / stages) & 1u,
                        err);
    }
  }
  // ---------------------------------------------------------- MMA issuer
  else if (warp == 1 && lane == 0) {
    int tcount = 0, s = 0;  // ring slot and phase of the next K block
    uint32_t ph = 0;
    bool ok = true;
    // Descriptors of slot 0 at K step 0.  A slot or K step only moves the
    // start-address field (16-byte units; shared addresses stay below
    // 2^18 bytes, so adding to the 14-bit field never carries), which keeps
    // the per-MMA issue cost to a few integer adds.
    const uint64_t adesc0 = make_smem_desc(smem_base, 16, 8 * swa, swa);
    // MN-major B.  16-bit: 128/64/32-byte swizzle atoms of 8 K rows.  tf32:
    // 32-bit MN-major operands use the 128-byte swizzle with 32-byte atoms
    // (layout type 1) and 4-row K groups.
    const uint64_t bdesc0 =
        FMT == 2 ? (make_smem_desc(smem_base + a_bytes, BK * SWB, 4 * SWB, 0) | (1ull << 61))
                 : make_smem_desc(smem_base + a_bytes, BK * SWB, 8 * SWB, SWB);
    const int ksteps = BK / KSTEP;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += tile_step, ++tcount) {
      const int buf = tcount % ACC_STAGES;
      const uint32_t use = static_cast<uint32_t>(tcount / ACC_STAGES);
      if (PERSISTENT) {
        if (!mbar_wait(smem_u32(&sh.acc_empty[buf]), (use & 1u) ^ 1u, abort_flag, err,
                       kErrWaitMma)) {
          ok = false;
          break;
        }
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * COLS);
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(smem_u32(&sh.full[s]), ph, abort_flag, err, kErrWaitMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t so4 = (static_cast<uint32_t>(s) * stage_bytes) >> 4;
        issue_kblock_any<ES, AROWS, SWB, HALVES, BN, FMT, false>(ksteps, d_tmem, adesc0 + so4,
                                                                 bdesc0 + so4, IDESC, kb == 0);
        mma_commit(smem_u32(&sh.empty[s]));  // stage reusable once these MMAs finish
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (!ok) break;
      mma_commit(smem_u32(&sh.acc_full[buf]));
    }
    if (!ok) {
      mma_commit(smem_u32(&sh.drain));
      mbar_wait_drain(smem_u32(&sh.drain), 0, err);
    }
  }

  // ------------------------------------------------------------ epilogue
  const bool epi_warp = PERSISTENT ? (warp >= 4) : true;
  if (epi_warp) {
    __syncwarp();
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int tcount = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += tile_step, ++tcount) {
      const int buf = tcount % ACC_STAGES;
      const uint32_t use = static_cast<uint32_t>(tcount / ACC_STAGES);
      if (!mbar_wait_idle(smem_u32(&sh.acc_full[buf]), use & 1u, abort_flag, err,
                          kErrWaitEpilogue))
        break;
      tc_fence_after();
      int pm, pn;
      tile_coords(tile, num_pid_m, num_pid_n, group_m, pm, pn);
#pragma unroll
      for (int h = 0; h < HALVES; ++h) {
        // BLOCK_M 64: lanes 16..31 of each quarter hold no row; BLOCK_M 32:
        // quarters 2 and 3 hold only the rows past the tile
        const int row = BM < 128 ? (lane < 16 && q * 16 < BM ? pm * BM + q * 16 + lane : M)
                                 : pm * BM + h * 128 + q * 32 + lane;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                        static_cast<uint32_t>(buf * COLS + h * BN + c * 32),
                    r);
          tmem_wait_ld();
          const int col0 = pn * BN + c * 32;
          if (row < M) {
            T* dst = C + static_cast<int64_t>(row) * N + col0;
            if (col0 + 32 <= N) {
              if constexpr (ES == 2) {
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const float lo = __uint_as_float(r[2 * i]), hi = __uint_as_float(r[2 * i + 1]);
                  pk[i] = (FMT == 1) ? pack_bf16(lo, hi) : pack_f16(lo, hi);
                }
                uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  d4[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
              } else {
                uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  d4[i] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (col0 + i < N) dst[i] = Elem<T>::from_f(__uint_as_float(r[i]));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sh.acc_empty[buf]));
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == alloc_warp) tmem_dealloc(tmem_base, ALLOC);
}

// --------------------------------------------------- CTA-pair (2-SM) tile
// BLOCK_M = 256: a cluster of two CTAs computes one 256 x BLOCK_N tile with
// M=256 tcgen05 MMAs issued by the even CTA (cta_group::2).  CTA r holds A
// rows [128r, 128r+128) and B columns [r*BN/2, (r+1)*BN/2) of the tile, so
// each CTA stages only half of B: 32 KB per 64-deep K stage for a 256x256
// tile instead of 48 KB for a single-CTA 128x256 tile, which lets more
// stages (more load latency cover) fit per SM.  Each CTA's TMEM receives its
// own 128 rows of D.
//
// num_warps 4: one tile per cluster (grid = 2 x tiles); all four warps drain
// TMEM after the main loop.
// num_warps 8 (PERSISTENT): one cluster per SM pair walks the tiles
// (tile = cluster id + k x clusters, grouped raster).  Warp 0 issues TMA,
// warp 1 of the even CTA issues MMAs, warps 4-7 of both CTAs drain TMEM;
// two TMEM accumulator buffers let the epilogue of tile i overlap the main
// loop of tile i+1.  The even CTA's acc_empty[b] collects the arrivals of
// all eight epilogue warps of the pair before buffer b is overwritten.
//
// Barriers: full[s] lives in the even CTA only; its producer arms it with
// the bytes of both CTAs and both producers' TMA loads count their bytes on
// it.  empty[s] and acc_full live in both CTAs; the even CTA's MMA thread
// commits to its own and (through the cluster address) to the peer's.
// All waits are bounded; a CTA that gives up drains and still reaches the
// final cluster barrier, so neither CTA exits while the other can signal it.
template <typename T, int FMT, int BN, bool PERSISTENT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PERSISTENT ? 256 : 128, 1)
    matmul_tc2_kernel(const __grid_constant__ CUtensorMap tma_a,
                      const __grid_constant__ CUtensorMap tma_b, T* __restrict__ C, int M, int N,
                      int K, int BK, int stages, int group_m, int swa, unsigned int* err) {
  constexpr int ES = sizeof(T);
  constexpr int BNH = BN / 2;                                 // B columns per CTA
  constexpr int SWB = (BNH * ES) < 128 ? (BNH * ES) : 128;    // B chunk width (bytes)
  constexpr int ACC = PERSISTENT ? 2 : 1;                     // TMEM accumulator buffers
  constexpr int ALLOC = tc2_tmem_alloc(ACC * BN);
  constexpr int KSTEP = 32 / ES;
  constexpr uint32_t IDESC = make_idesc(FMT, 256, BN, false, true);
  // A half tile (last wave of a persistent grid) covers BN/2 columns: each
  // CTA stages one B chunk instead of two and the MMAs run with N = BN/2.
  constexpr bool CAN_SPLIT = PERSISTENT && FMT != 2 && (BNH * ES) / SWB == 2;
  constexpr uint32_t IDESC_HALF = make_idesc(FMT, 256, BN / 2, false, true);

  __shared__ TcShared sh;
  extern __shared__ uint8_t dyn_smem[];
  const uint32_t smem_base = (smem_u32(dyn_smem) + 1023u) & ~1023u;
  const uint32_t a_bytes = 128u * BK * ES;
  const uint32_t b_bytes = static_cast<uint32_t>(BK) * BNH * ES;
  const uint32_t stage_bytes = (a_bytes + b_bytes + 1023u) & ~1023u;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int num_pid_m = (M + 255) / 256;
  const int num_pid_n = (N + BN - 1) / BN;
  const int num_tiles = num_pid_m * num_pid_n;
  const int first_tile = static_cast<int>(blockIdx.x >> 1);
  const int tile_step = PERSISTENT ? static_cast<int>(gridDim.x >> 1) : num_tiles;
  const Tc2Items items = tc2_items(num_tiles, tile_step, CAN_SPLIT);
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&sh.full[s]), 1);
      mbar_init(smem_u32(&sh.empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&sh.acc_full[b]), 1);
      mbar_init(smem_u32(&sh.acc_empty[b]), 8);  // 4 epilogue warps x 2 CTAs
    }
    mbar_init(smem_u32(&sh.drain), 1);
    sh.abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 0) {
    tmem_alloc_pair(smem_u32(&sh.tmem_base), ALLOC);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised before any remote signal
  tc_fence_after();
  const uint32_t tmem_base = sh.tmem_base;
  volatile int* abort_flag = &sh.abort;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------ producers (both)
    const uint32_t full0 = mapa_shared(smem_u32(&sh.full[0]), 0);  // even CTA's full[0]
    int it = 0, s = 0;  // K blocks issued; ring slot and phase of the next one
    uint32_t ph = 0;
    bool ok = true;
    for (int item = first_tile; item < items.count && ok; item += tile_step) {
      int tile, half, pm, pn;
      items.at(item, tile, half);
      tile_coords(tile, num_pid_m, num_pid_n, group_m, pm, pn);
      // B columns this CTA stages: [n0, n0 + chunks * SWB / ES)
      const int chunks = half < 0 ? (BNH * ES) / SWB : 1;
      const int n0 = half < 0 ? pn * BN + static_cast<int>(rank) * BNH
                              : pn * BN + half * BNH + static_cast<int>(rank) * (BNH / 2);
      const uint32_t stage_tx = 2u * (a_bytes + (half < 0 ? b_bytes : b_bytes / 2));
      for (int kb = 0; kb < num_kb; ++kb, ++it) {
        if (!mbar_wait(smem_u32(&sh.empty[s]), ph ^ 1u, abort_flag, err, kErrWaitProducer)) {
          ok = false;
          break;
        }
        const uint32_t full = full0 + static_cast<uint32_t>(s) * 8u;
        if (rank == 0) mbar_arrive_expect_tx(smem_u32(&sh.full[s]), stage_tx);
        const uint32_t sa = smem_base + s * stage_bytes;
        const uint32_t sb = sa + a_bytes;
        const int a_atoms = (BK * ES) / swa;
        for (int a = 0; a < a_atoms; ++a)
          tma_load_2d_pair(sa + a * 128 * swa, &tma_a, full, kb * BK + a * (swa / ES),
                           pm * 256 + static_cast<int>(rank) * 128);
        for (int c = 0; c < chunks; ++c)
          tma_load_2d_pair(sb + c * BK * SWB, &tma_b, full, n0 + c * (SWB / ES), kb * BK);
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
    if (!ok) {
      if (rank == 0) {
        for (int j = max(0, it - stages); j < it; ++j)
          mbar_wait_drain(smem_u32(&sh.full[j % stages]), static_cast<uint32_t>(j / stages) & 1u,
                          err);
      } else {
        // the odd CTA's loads complete on the even CTA's barrier, which it
        // cannot poll: give in-flight copies time to land before exiting
        const unsigned long long t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // --------------------------------------------- MMA issuer (even CTA)
    const uint32_t peer_empty0 = mapa_shared(smem_u32(&sh.empty[0]), 1);
    const uint32_t peer_acc0 = mapa_shared(smem_u32(&sh.acc_full[0]), 1);
    int tcount = 0, s = 0;  // ring slot and phase of the next K block
    uint32_t ph = 0;
    bool ok = true;
    // slot-0 / K-step-0 descriptors; slots and K steps add to the start
    // address field only (see matmul_tc_kernel)
    const uint64_t adesc0 = make_smem_desc(smem_base, 16, 8 * swa, swa);
    const uint64_t bdesc0 =
        FMT == 2 ? (make_smem_desc(smem_base + a_bytes, BK * SWB, 4 * SWB, 0) | (1ull << 61))
                 : make_smem_desc(smem_base + a_bytes, BK * SWB, 8 * SWB, SWB);
    const int ksteps = BK / KSTEP;
    for (int item = first_tile; item < items.count && ok; item += tile_step, ++tcount) {
      int tile, half;
      items.at(item, tile, half);
      const uint32_t idesc = half < 0 ? IDESC : IDESC_HALF;
      const int buf = tcount % ACC;
      const uint32_t use = static_cast<uint32_t>(tcount / ACC);
      if (PERSISTENT && !mbar_wait<true>(smem_u32(&sh.acc_empty[buf]), (use & 1u) ^ 1u,
                                         abort_flag, err, kErrWaitMma)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(smem_u32(&sh.full[s]), ph, abort_flag, err, kErrWaitMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t so4 = (static_cast<uint32_t>(s) * stage_bytes) >> 4;
        issue_kblock_any<ES, 128, SWB, 1, BN, FMT, true>(ksteps, d_tmem, adesc0 + so4,
                                                         bdesc0 + so4, idesc, kb == 0);
        mma_commit_pair(smem_u32(&sh.empty[s]));
        mma_commit_pair(peer_empty0 + static_cast<uint32_t>(s) * 8u);
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (!ok) break;
      mma_commit_pair(smem_u32(&sh.acc_full[buf]));
      mma_commit_pair(peer_acc0 + static_cast<uint32_t>(buf) * 8u);
    }
    if (!ok) {
      mma_commit_pair(smem_u32(&sh.drain));
      mbar_wait_drain(smem_u32(&sh.drain), 0, err);
    }
  }

  // ------------------------------------------------------- epilogue (both)
  const bool epi_warp = PERSISTENT ? (warp >= 4) : true;
  if (epi_warp) {
    __syncwarp();
    const int q = warp & 3;
    const uint32_t leader_acc_empty0 = mapa_shared(smem_u32(&sh.acc_empty[0]), 0);
    int tcount = 0;
    for (int item = first_tile; item < items.count; item += tile_step, ++tcount) {
      const int buf = tcount % ACC;
      const uint32_t use = static_cast<uint32_t>(tcount / ACC);
      if (!mbar_wait_idle(smem_u32(&sh.acc_full[buf]), use & 1u, abort_flag, err,
                          kErrWaitEpilogue))
        break;
      tc_fence_after();
      int tile, half, pm, pn;
      items.at(item, tile, half);
      tile_coords(tile, num_pid_m, num_pid_n, group_m, pm, pn);
      const int row = pm * 256 + static_cast<int>(rank) * 128 + q * 32 + lane;
      // a half tile's accumulator holds its BN/2 columns in the first BN/2
      // TMEM columns of the buffer
      const int ncols = half < 0 ? BN : BN / 2;
      const int cbase = pn * BN + (half < 0 ? 0 : half * (BN / 2));
#pragma unroll 1
      for (int c = 0; c < ncols / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                      static_cast<uint32_t>(buf * BN + c * 32),
                  r);
        tmem_wait_ld();
        const int col0 = cbase + c * 32;
        if (row < M) {
          T* dst = C + static_cast<int64_t>(row) * N + col0;
          if (col0 + 32 <= N) {
            if constexpr (ES == 2) {
              uint32_t pk[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float lo = __uint_as_float(r[2 * i]), hi = __uint_as_float(r[2 * i + 1]);
                pk[i] = (FMT == 1) ? pack_bf16(lo, hi) : pack_f16(lo, hi);
              }
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                d4[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
            } else {
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int i = 0; i < 8; ++i)
                d4[i] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i < N) dst[i] = Elem<T>::from_f(__uint_as_float(r[i]));
          }
        }
      }
      if (PERSISTENT) {
        // this warp's TMEM rows of buffer buf are read: free them for the
        // MMA issuer of the pair (even CTA)
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(leader_acc_empty0 + static_cast<uint32_t>(buf) * 8u);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its peer may still signal it
  tc_fence_after();
  if (warp == 0) tmem_dealloc_pair(tmem_base, ALLOC);
}

// ------------------------------------------------------------------- host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// bytes = 128 / 64 / 32; atom32 selects the 128-byte swizzle with 32-byte
// atoms that 32-bit MN-major tensor-core operands need.
static CUtensorMapSwizzle swizzle_enum(int bytes, bool atom32 = false) {
  if (atom32) return CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  return bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
         : bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                       : CU_TENSOR_MAP_SWIZZLE_32B;
}

// 2-D row-major tensor [rows, cols] (cols contiguous) with box
// [box_rows, box_cols].
static bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* ptr, uint64_t rows,
                      uint64_t cols, int es, uint32_t box_cols, uint32_t box_rows, int swz,
                      bool atom32 = false) {
  EncodeTiledFn fn = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * static_cast<uint64_t>(es)};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_enum(swz, atom32),
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Plan: aux[0] = swizzle bytes of A, aux[1] = dynamic smem bytes,
// aux[2] = persistent flag.
gpo_status plan_matmul_tc(const gpo_key& k, Plan& p, std::string& log) {
  const int es = dtype_bytes(k.dtype);
  const int BM = k.block_m, BN = k.block_n, BK = k.block_k;
  const int64_t M = k.shape[0], N = k.shape[1], K = k.shape[2];
  if (BM != 32 && BM != 64 && BM != 128 && BM != 256) {
    log = "tcgen05 family needs BLOCK_M 32, 64, 128 or 256";
    return GPO_BAD_CONFIG;
  }
  if (BN != 32 && BN != 64 && BN != 128 && BN != 256) {
    log = "tcgen05 family needs BLOCK_N in {32, 64, 128, 256}";
    return GPO_BAD_CONFIG;
  }
  if (BK < 1 || (BK & (BK - 1)) || BK * es < 32 || BK > 256) {
    log = "tcgen05 family needs BLOCK_K a power of two with BLOCK_K*es >= 32 and <= 256";
    return GPO_BAD_CONFIG;
  }
  if (k.num_warps != 4 && k.num_warps != 8) {
    log = "tcgen05 family needs num_warps 4 or 8";
    return GPO_BAD_CONFIG;
  }
  if ((K * es) % 16 || (N * es) % 16) {
    log = "TMA needs K*es and N*es multiples of 16 bytes";
    return GPO_BAD_CONFIG;
  }
  if (k.num_stages < 1 || k.num_stages > kMaxStages) {
    log = "num_stages must be in [1, 8]";
    return GPO_BAD_CONFIG;
  }
  if (k.group_m < 1) {
    log = "GROUP_M must be >= 1";
    return GPO_BAD_CONFIG;
  }
  const bool persistent = k.num_warps == 8;
  // BLOCK_M 256 with 4 warps: a CTA pair (cta_group::2), each CTA staging
  // 128 rows of A and BLOCK_N/2 columns of B.  tf32 needs the 128-byte B
  // chunk (BLOCK_N/2 * 4 >= 128) for its 32-bit MN-major layout.
  // With 8 warps the pair is persistent (one cluster per SM pair walking
  // the tiles, two TMEM accumulator buffers).
  const bool pair = BM == 256 && (k.dtype != GPO_TF32 || BN >= 64);
  if (pair) {
    const uint32_t pa = 128u * BK * es, pb = static_cast<uint32_t>(BK) * (BN / 2) * es;
    const uint32_t pst = (pa + pb + 1023u) & ~1023u;
    const int pc = tc2_tmem_alloc((persistent ? 2 : 1) * BN);
    // Never let more CTAs share an SM than its 512 TMEM columns hold: a pair
    // allocation that had to wait on one SM of the pair while holding the
    // other could otherwise wait on a second pair doing the opposite.  The
    // shared-memory request is padded so that at most 512 / columns CTAs fit.
    const uint32_t max_ctas = 512u / static_cast<uint32_t>(pc);
    uint32_t pdyn = pst * static_cast<uint32_t>(k.num_stages) + 1024u;
    pdyn = std::max<uint32_t>(pdyn, 233472u / (max_ctas + 1u) + 64u);
    const uint32_t psmem = pdyn + static_cast<uint32_t>(sizeof(TcShared));
    if (psmem > kMaxSmemPerCta) {
      log = "shared memory " + std::to_string(psmem) + " B per CTA of the pair (" +
            std::to_string(k.num_stages) + " stages x " + std::to_string(pst) +
            " B) exceeds the 232448 B per-CTA limit";
      return GPO_COMPILE_ERROR;
    }
    p.aux[0] = std::min(BK * es, 128);
    p.aux[1] = static_cast<int>(pdyn);
    p.aux[2] = persistent ? 1 : 0;
    p.aux[3] = 1;  // pair
    p.family = "matmul_tc";
    p.res.smem_bytes = psmem;
    p.res.tmem_cols = static_cast<uint32_t>(pc);
    p.res.threads_per_cta = persistent ? 256u : 128u;
    // persistent: clamped to the co-resident cluster count at launch
    p.res.grid_x = static_cast<uint32_t>(2 * cdiv(M, 256) * cdiv(N, BN));
    p.res.grid_y = p.res.grid_z = 1;
    p.res.persistent = persistent ? 1u : 0u;
    p.res.launches_per_call = 1;
    const char* tn = k.dtype == GPO_BFLOAT16 ? "bf16" : k.dtype == GPO_FLOAT16 ? "f16" : "tf32";
    snprintf(p.res.kernel, sizeof(p.res.kernel), "matmul_tc2_kernel<%s,256,%d,cta_pair%s>", tn,
             BN, persistent ? "_persistent" : "");
    return GPO_OK;
  }
  p.aux[3] = 0;
  // BLOCK_M 32 stages A in the 64-row atoms of the M=64 MMA
  const uint32_t a_bytes = static_cast<uint32_t>(std::max(BM, 64)) * BK * es;
  const uint32_t b_bytes = static_cast<uint32_t>(BK) * BN * es;
  const uint32_t stage = (a_bytes + b_bytes + 1023u) & ~1023u;
  const uint32_t dyn = stage * static_cast<uint32_t>(k.num_stages) + 1024u;
  const uint32_t smem = dyn + static_cast<uint32_t>(sizeof(TcShared));
  const int cols = std::max(1, BM / 128) * BN;
  const int acc_stages = (persistent && 2 * cols <= 512) ? 2 : 1;
  int alloc = 32;
  while (alloc < acc_stages * cols) alloc *= 2;
  if (smem > kMaxSmemPerCta) {
    log = "shared memory " + std::to_string(smem) + " B (" + std::to_string(k.num_stages) +
          " stages x " + std::to_string(stage) + " B) exceeds the 232448 B per-CTA limit";
    return GPO_COMPILE_ERROR;
  }
  if (alloc > static_cast<int>(kTmemCols)) {
    log = "TMEM accumulator needs " + std::to_string(alloc) + " columns > 512";
    return GPO_COMPILE_ERROR;
  }
  p.aux[0] = std::min(BK * es, 128);
  p.aux[1] = static_cast<int>(dyn);
  p.aux[2] = persistent ? 1 : 0;
  p.family = "matmul_tc";
  p.res.smem_bytes = smem;
  p.res.tmem_cols = static_cast<uint32_t>(alloc);
  p.res.threads_per_cta = persistent ? 256u : 128u;
  const uint64_t tiles = cdiv(M, BM) * cdiv(N, BN);
  p.res.grid_x = static_cast<uint32_t>(tiles);  // persistent: clamped to the SM count at launch
  p.res.grid_y = p.res.grid_z = 1;
  p.res.persistent = persistent ? 1u : 0u;
  p.res.launches_per_call = 1;
  const char* tn = k.dtype == GPO_BFLOAT16 ? "bf16" : k.dtype == GPO_FLOAT16 ? "f16" : "tf32";
  snprintf(p.res.kernel, sizeof(p.res.kernel), "matmul_tc_kernel<%s,%d,%d,%s>", tn, BM, BN,
           persistent ? "persistent" : "tile");
  return GPO_OK;
}

// CTAs of `func` that one SM holds at once, from the hardware limits:
// shared memory (with the per-block reservation), registers (allocated per
// warp in 256-register units), threads and TMEM columns.  Persistent grids
// of the tensor-core kernels are sized with this: the runtime's occupancy
// queries report one CTA per SM for these kernels although more are
// resident at launch.  Cached per (device, kernel, block size, shared
// memory, TMEM columns).
static int resident_ctas_per_sm(const void* func, int threads, uint32_t dyn, uint32_t tmem_cols,
                                int device) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, int, uint32_t, uint32_t>, int> cache;
  const auto key = std::make_tuple(device, func, threads, dyn, tmem_cols);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  cudaFuncAttributes fa;
  int smem_sm = 0, reserved = 0, regs_sm = 0, thr_sm = 0;
  if (cudaFuncGetAttributes(&fa, func) != cudaSuccess ||
      cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device) !=
          cudaSuccess ||
      cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, device) !=
          cudaSuccess ||
      cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, device) !=
          cudaSuccess ||
      cudaDeviceGetAttribute(&thr_sm, cudaDevAttrMaxThreadsPerMultiProcessor, device) !=
          cudaSuccess) {
    cudaGetLastError();
    return 1;
  }
  const int64_t smem_cta = static_cast<int64_t>(dyn) + fa.sharedSizeBytes + reserved;
  const int warps = (threads + 31) / 32;
  const int64_t regs_warp = ((static_cast<int64_t>(fa.numRegs) * 32 + 255) / 256) * 256;
  int64_t n = std::min<int64_t>(smem_sm / std::max<int64_t>(1, smem_cta),
                                thr_sm / std::max(1, threads));
  n = std::min<int64_t>(n, regs_sm / std::max<int64_t>(1, regs_warp * warps));
  n = std::min<int64_t>(n, static_cast<int64_t>(kTmemCols) / std::max<uint32_t>(1u, tmem_cols));
  const int r = static_cast<int>(std::max<int64_t>(1, n));
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = r;
  return r;
}

template <typename T, int FMT, int BM, int BN, bool P>
static gpo_status run_tc(const gpo_key& k, const Plan& p, const gpo_args& a, const LaunchCtx& c,
                         CUtensorMapDataType dt) {
  const int es = sizeof(T);
  const int64_t M = k.shape[0], N = k.shape[1], K = k.shape[2];
  const int swa = p.aux[0];
  constexpr int SWB = (BN * sizeof(T)) < 128 ? (BN * sizeof(T)) : 128;
  CUtensorMap ma, mb;
  if (!encode_2d(&ma, dt, a.in[0], M, K, es, swa / es, BM, swa)) return GPO_LAUNCH_ERROR;
  if (!encode_2d(&mb, dt, a.in[1], K, N, es, SWB / es, k.block_k, SWB, FMT == 2))
    return GPO_LAUNCH_ERROR;
  auto kern = matmul_tc_kernel<T, FMT, BM, BN, P>;
  const uint32_t dyn = static_cast<uint32_t>(p.aux[1]);
  gpo_status s = ensure_smem_attr(reinterpret_cast<const void*>(kern), dyn);
  if (s != GPO_OK) return s;
  const uint64_t tiles = cdiv(M, BM) * cdiv(N, BN);
  // persistent: every CTA the SMs hold at once (TMEM, shared memory,
  // registers), at most one per tile
  const unsigned grid =
      P ? static_cast<unsigned>(std::min<uint64_t>(
              tiles, static_cast<uint64_t>(c.sm_count) *
                         resident_ctas_per_sm(reinterpret_cast<const void*>(kern), 256, dyn,
                                              p.res.tmem_cols, c.device)))
        : static_cast<unsigned>(tiles);
  kern<<<grid, P ? 256 : 128, dyn, c.stream>>>(ma, mb, static_cast<T*>(a.out),
                                               static_cast<int>(M), static_cast<int>(N),
                                               static_cast<int>(K), k.block_k, k.num_stages,
                                               k.group_m, swa, c.err);
  return launch_status();
}

template <typename T, int FMT, int BN, bool P>
static gpo_status run_tc2(const gpo_key& k, const Plan& p, const gpo_args& a, const LaunchCtx& c,
                          CUtensorMapDataType dt) {
  const int es = sizeof(T);
  const int64_t M = k.shape[0], N = k.shape[1], K = k.shape[2];
  const int swa = p.aux[0];
  constexpr int BNH = BN / 2;
  constexpr int SWB = (BNH * sizeof(T)) < 128 ? (BNH * sizeof(T)) : 128;
  CUtensorMap ma, mb;
  if (!encode_2d(&ma, dt, a.in[0], M, K, es, swa / es, 128, swa)) return GPO_LAUNCH_ERROR;
  if (!encode_2d(&mb, dt, a.in[1], K, N, es, SWB / es, k.block_k, SWB, FMT == 2))
    return GPO_LAUNCH_ERROR;
  auto kern = matmul_tc2_kernel<T, FMT, BN, P>;
  const uint32_t dyn = static_cast<uint32_t>(p.aux[1]);
  gpo_status s = ensure_smem_attr(reinterpret_cast<const void*>(kern), dyn);
  if (s != GPO_OK) return s;
  const int64_t tiles = cdiv(M, 256) * cdiv(N, BN);
  const int threads = P ? 256 : 128;
  // persistent: as many clusters as the SM pairs hold at once (TMEM, shared
  // memory, registers; the cluster-occupancy query reports one CTA per SM
  // for these kernels), at most one per tile
  const unsigned grid =
      2u * (P ? static_cast<unsigned>(std::max<int64_t>(
                    1, std::min<int64_t>(tiles, static_cast<int64_t>(c.sm_count / 2) *
                                                    resident_ctas_per_sm(
                                                        reinterpret_cast<const void*>(kern),
                                                        threads, dyn, p.res.tmem_cols,
                                                        c.device))))
              : static_cast<unsigned>(tiles));
  kern<<<grid, threads, dyn, c.stream>>>(ma, mb, static_cast<T*>(a.out), static_cast<int>(M),
                                     static_cast<int>(N), static_cast<int>(K), k.block_k,
                                     k.num_stages, k.group_m, swa, c.err);
  return launch_status();
}

template <typename T, int FMT>
static gpo_status run_tc2_bn(const gpo_key& k, const Plan& p, const gpo_args& a,
                             const LaunchCtx& c, CUtensorMapDataType dt) {
  const bool P = p.aux[2] != 0;
  switch (k.block_n) {
    case 32: return P ? run_tc2<T, FMT, 32, true>(k, p, a, c, dt)
                      : run_tc2<T, FMT, 32, false>(k, p, a, c, dt);
    case 64: return P ? run_tc2<T, FMT, 64, true>(k, p, a, c, dt)
                      : run_tc2<T, FMT, 64, false>(k, p, a, c, dt);
    case 128: return P ? run_tc2<T, FMT, 128, true>(k, p, a, c, dt)
                       : run_tc2<T, FMT, 128, false>(k, p, a, c, dt);
    case 256: return P ? run_tc2<T, FMT, 256, true>(k, p, a, c, dt)
                       : run_tc2<T, FMT, 256, false>(k, p, a, c, dt);
    default: return GPO_INTERNAL;
  }
}

template <typename T, int FMT, int BM, bool P>
static gpo_status run_tc_bn(const gpo_key& k, const Plan& p, const gpo_args& a,
                            const LaunchCtx& c, CUtensorMapDataType dt) {
  switch (k.block_n) {
    case 32: return run_tc<T, FMT, BM, 32, P>(k, p, a, c, dt);
    case 64: return run_tc<T, FMT, BM, 64, P>(k, p, a, c, dt);
    case 128: return run_tc<T, FMT, BM, 128, P>(k, p, a, c, dt);
    case 256: return run_tc<T, FMT, BM, 256, P>(k, p, a, c, dt);
    default: return GPO_INTERNAL;
  }
}

template <typename T, int FMT>
static gpo_status run_tc_dt(const gpo_key& k, const Plan& p, const gpo_args& a,
                            const LaunchCtx& c, CUtensorMapDataType dt) {
  if (p.aux[3]) return run_tc2_bn<T, FMT>(k, p, a, c, dt);
  const bool P = p.aux[2] != 0;
  if (k.block_m == 32)
    return P ? run_tc_bn<T, FMT, 32, true>(k, p, a, c, dt)
             : run_tc_bn<T, FMT, 32, false>(k, p, a, c, dt);
  if (k.block_m == 64)
    return P ? run_tc_bn<T, FMT, 64, true>(k, p, a, c, dt)
             : run_tc_bn<T, FMT, 64, false>(k, p, a, c, dt);
  if (k.block_m == 128)
    return P ? run_tc_bn<T, FMT, 128, true>(k, p, a, c, dt)
             : run_tc_bn<T, FMT, 128, false>(k, p, a, c, dt);
  return P ? run_tc_bn<T, FMT, 256, true>(k, p, a, c, dt)
           : run_tc_bn<T, FMT, 256, false>(k, p, a, c, dt);
}

gpo_status launch_matmul_tc(const gpo_key& k, const Plan& p, const gpo_args& a,
                            const LaunchCtx& c) {
  if (!a.in[0] || !a.in[1] || !a.out) return GPO_BAD_ARGS;
  if (!aligned16(a.in[0]) || !aligned16(a.in[1]) || !aligned16(a.out)) return GPO_BAD_ARGS;
  if (k.shape[0] == 0 || k.shape[1] == 0) return GPO_OK;
  switch (k.dtype) {
    case GPO_BFLOAT16:
      return run_tc_dt<__nv_bfloat16, 1>(k, p, a, c, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
    case GPO_FLOAT16:
      return run_tc_dt<__half, 0>(k, p, a, c, CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
    case GPO_TF32:
      return run_tc_dt<float, 2>(k, p, a, c, CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
    default:
      return GPO_BAD_ARGS;
  }
}

}  // namespace gpo

// Flash-attention forward on tcgen05 tensor cores (sm_100a), non-causal and
// causal.
//
// Replaces attention_kernel (compiler/triton/kernels.py:212-270) for 16-bit
// inputs with BLOCK_M = 64, 128 or 256.  One CTA per (128-row query tile,
// batch*head) -- 64-row tiles with M=64 MMAs for BLOCK_M 64, a CTA pair on
// two tiles for 256 with 4 warps; causal grids visit the longest query
// tiles first.  BLOCK_M 256 with 8 warps is the persistent two-tile kernel
// further down (its own section describes it); the roles below are those
// of the one-tile kernel.
//
// Warp roles:
//   warp 0  TMA producer of Q (once) and of the K ring (num_stages slots).
//   warp 3  TMA producer of the V ring (num_stages slots).  K slot j is
//           released when S_j's MMAs complete, V slot j when PV_j's do, so
//           neither ring waits on the other.
//   warp 1  MMA issuer:   S_j = Q K_j^T into TMEM buffer j % NB, then
//                         O += P_i V_i for i = j - (NB - 1).  With NB = 3
//                         S/P buffers the S MMAs run two blocks ahead of the
//                         PV MMAs, so the softmax of block j overlaps the
//                         MMAs of S_{j+1}, S_{j+2} and PV_{j-1}.
//   warp 2  TMEM owner.
//   softmax warpgroups (WG = 1 with num_warps 4: warps 4-7; WG = 2 with
//           num_warps 8: warps 4-7 and 8-11): query row r is TMEM lane r,
//           read by warp 4 + r/32 (and 8 + r/32).  With WG = 2 the two
//           warps of a row each take half of the block's columns and of
//           O's columns, exchanging their partial row max through shared
//           memory once per block (a 64-thread named barrier per warp
//           pair), so every SM sub-partition runs two softmax warps and one
//           warp's TMEM / barrier latency hides behind the other's math.
//           Per block: read S_j from TMEM, apply scale, padding and causal
//           masks, keep the running max in the log2 domain, write
//           P_j = exp2(s - m) as 16-bit pairs back into TMEM over the same
//           S buffer (the A operand of the PV MMA, read from TMEM) and
//           accumulate the fp32 row sum.  Scale/shift FMAs and row-sum adds
//           run as packed fp32x2 operations and the row max as three-input
//           max.  The running max used for P is only moved (and O in TMEM
//           rescaled) when a block's max exceeds it by more than 8 (a factor
//           of 256); until then P <= 256, which 16-bit P and the fp32
//           accumulator represent exactly as well as P <= 1.
// TMEM columns: O [0, D), S/P buffers [D + b*BN, D + (b+1)*BN) for b < NB;
// NB = 3 when D + 3*BN <= 512, else 2 -- except that with one softmax
// warpgroup, when that layout needs more than 256 columns but two buffers
// fit in 256 and shared memory holds two CTAs, NB = 2 and two CTAs share
// each SM.
#include <algorithm>
#include <atomic>

#include "gpo_common.cuh"
#include "gpo_internal.h"

namespace gpo {

constexpr int kAttnMaxStages = 4;
constexpr float kRescaleThreshold = 8.0f;
constexpr int kAttnMaxSBufs = 3;  // S/P buffers

// S/P buffers: three when TMEM has room, else two.
__host__ __device__ constexpr int attn_sbufs(int d, int bn) { return d + 3 * bn <= 512 ? 3 : 2; }

// Two S/P buffers when they fit the CTA's TMEM in half of the SM's 512
// columns and the default layout does not (else 0): two CTAs per SM then
// interleave their MMAs and softmax (the plan takes this when shared memory
// also holds two CTAs).  Measured at B*H = 128, S = 4096, D = 128, BLOCK_N
// 64: 744 vs 572 TFLOP/s (full), 653 vs 520 (causal).  One buffer (S_j,
// softmax_j and PV_j in series within the CTA, BLOCK_N 128) measured 597 vs
// 927 for three buffers on one CTA per SM, so it is not offered.
__host__ __device__ constexpr int attn_duo_nb(int d, int bn) {
  return d + attn_sbufs(d, bn) * bn > 256 && d + 2 * bn <= 256 ? 2 : 0;
}

struct AttnShared {
  uint64_t q_full;
  uint64_t k_full[kAttnMaxStages];
  uint64_t k_empty[kAttnMaxStages];
  uint64_t v_full[kAttnMaxStages];
  uint64_t v_empty[kAttnMaxStages];
  uint64_t s_full[kAttnMaxSBufs];
  uint64_t p_full[kAttnMaxSBufs];
  uint64_t pv_done[kAttnMaxSBufs];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// WG = 2 exchange area after the V ring in dynamic shared memory:
// [block parity][warpgroup][row] partial row maxima; the epilogue's partial
// row sums reuse the parity slot the last block did not read.
constexpr uint32_t kAttnXchgBytes = 2u * 2u * 128u * sizeof(float);

__host__ __device__ constexpr int attn_tmem_alloc(int cols) {
  return cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : cols <= 256 ? 256 : 512;
}

// Barrier `id` (1..15) among `count` threads (whole warps).
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// TMEM load / store of C consecutive 32-bit columns (C = 16 or 32).
template <int C>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t* r) {
  if constexpr (C == 32)
    tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(r));
  else
    tmem_ld16(taddr, r);
}
template <int C>
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const uint32_t* r) {
  if constexpr (C == 32)
    tmem_st32(taddr, *reinterpret_cast<const uint32_t(*)[32]>(r));
  else
    tmem_st16(taddr, r);
}

template <typename T, int FMT, int BN, int D, bool CAUSAL, int WG, bool PAIR, int NB, int TM>
__global__ void __launch_bounds__(128 + 128 * WG,
                                  (WG == 1 && !PAIR && attn_duo_nb(D, BN) == NB) ? 2 : 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tma_q,
                   const __grid_constant__ CUtensorMap tma_k,
                   const __grid_constant__ CUtensorMap tma_v, T* __restrict__ O, int S,
                   int stages, float scale_log2, unsigned int* err) {
  constexpr int ES = 2;
  constexpr int SWQ = (D * ES) < 128 ? (D * ES) : 128;  // swizzle of Q/K/V rows
  // TM: query rows per CTA (128, or 64 with M=64 MMAs: D / S row 16g + r
  // sits in TMEM lane 32g + r, and an M=64 MMA reads its A operand (P) from
  // the same lanes)
  static_assert(TM == 128 || (TM == 64 && WG == 1 && !PAIR), "64-row tiles: one warpgroup");
  constexpr uint32_t Q_BYTES = static_cast<uint32_t>(TM) * D * ES;
  // PAIR: each CTA stages half of K's rows and half of V's columns
  constexpr int KROWS = PAIR ? BN / 2 : BN;     // K rows per CTA
  constexpr int VCOLS = PAIR ? D / 2 : D;       // V columns per CTA
  constexpr int SWV = (VCOLS * ES) < 128 ? (VCOLS * ES) : 128;  // swizzle of V rows
  constexpr uint32_t KV_BYTES = static_cast<uint32_t>(KROWS) * D * ES;  // = BN * VCOLS * ES
  constexpr uint32_t KV_SLOT = (KV_BYTES + 1023u) & ~1023u;
  static_assert(NB == 2 || NB == 3, "two or three S/P buffers");
  constexpr int LAG = NB - 1;  // S MMAs run LAG blocks ahead of PV MMAs
  constexpr int COLS = D + NB * BN;
  constexpr int ALLOC = attn_tmem_alloc(COLS);
  constexpr int MMA_M = PAIR ? 256 : TM;
  constexpr uint32_t IDESC_S = make_idesc(FMT, MMA_M, BN, false, false);
  constexpr uint32_t IDESC_O = make_idesc(FMT, MMA_M, D, false, true);
  constexpr int SC = BN / WG;        // S columns per softmax warp
  constexpr int OC = D / WG;         // O columns per softmax warp
  constexpr int SCH = SC < 32 ? SC : 32;  // TMEM access chunk (S)
  constexpr int OCH = OC < 32 ? OC : 32;  // TMEM access chunk (O)
  static_assert(COLS <= 512, "TMEM holds 512 columns");
  static_assert(SC >= 32 && OC >= 16, "softmax warps need >= 32 S and >= 16 O columns");

  __shared__ AttnShared sh;
  extern __shared__ uint8_t dyn_smem[];
  const uint32_t base = (smem_u32(dyn_smem) + 1023u) & ~1023u;
  const uint32_t q_smem = base;
  const uint32_t k_smem = q_smem + Q_BYTES;
  const uint32_t v_smem = k_smem + static_cast<uint32_t>(stages) * KV_SLOT;
  float* xchg = reinterpret_cast<float*>(
      dyn_smem + (v_smem + static_cast<uint32_t>(stages) * KV_SLOT - smem_u32(dyn_smem)));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // PAIR: cluster c holds query tiles 2c (even CTA) and 2c + 1 (odd CTA)
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int units = PAIR ? (S + 255) / 256 : (S + TM - 1) / TM;  // tiles or tile pairs
  const int unit = static_cast<int>(PAIR ? (blockIdx.x >> 1) : blockIdx.x);
  // longest causal rows first; identity order for the non-causal task
  const int ut = CAUSAL ? (units - 1 - unit) : unit;
  const int q0 = PAIR ? (2 * ut + static_cast<int>(rank)) * 128 : ut * TM;
  const int bh = blockIdx.y;
  // K/V blocks the MMAs run over (causal: up to the diagonal of the unit's
  // last tile; the even CTA of a pair masks its extra blocks to P = 0)
  const int kv_len = CAUSAL ? min(S, PAIR ? (2 * ut + 2) * 128 : (ut + 1) * TM) : S;
  const int nblk = (kv_len + BN - 1) / BN;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&sh.q_full), 1);
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&sh.k_full[s]), 1);
      mbar_init(smem_u32(&sh.k_empty[s]), 1);
      mbar_init(smem_u32(&sh.v_full[s]), 1);
      mbar_init(smem_u32(&sh.v_empty[s]), 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(smem_u32(&sh.s_full[b]), 1);
      mbar_init(smem_u32(&sh.p_full[b]), 4 * WG * (PAIR ? 2 : 1));  // PAIR: both CTAs' warps
      mbar_init(smem_u32(&sh.pv_done[b]), 1);
    }
    mbar_init(smem_u32(&sh.drain), 1);
    sh.abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tma_q);
    tma_prefetch_desc(&tma_k);
    tma_prefetch_desc(&tma_v);
  }
  if (warp == 2) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_u32(&sh.tmem_base), ALLOC);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(&sh.tmem_base), ALLOC);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync_all();  // both CTAs' barriers initialised before any remote signal
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* abort_flag = &sh.abort;

  if ((warp == 0 || warp == 3) && lane == 0) {
    // ----------------------------------------------- producers (K: 0, V: 3)
    const bool is_k = warp == 0;
    const CUtensorMap* map = is_k ? &tma_k : &tma_v;
    const uint32_t ring = is_k ? k_smem : v_smem;
    uint64_t* full = is_k ? sh.k_full : sh.v_full;
    uint64_t* empty = is_k ? sh.k_empty : sh.v_empty;
    bool ok = true;
    int issued = 0;
    // PAIR: the even CTA's full barriers count both CTAs' bytes (pair loads)
    const uint32_t mult = PAIR ? 2u : 1u;
    auto lead = [&](const uint64_t* bar) -> uint32_t {
      return PAIR ? mapa_shared(smem_u32(bar), 0) : smem_u32(bar);
    };
    auto load = [&](uint32_t dst, const CUtensorMap* m, uint32_t bar, int x, int y) {
      if constexpr (PAIR)
        tma_load_3d_pair(dst, m, bar, x, y, bh);
      else
        tma_load_3d(dst, m, bar, x, y, bh);
    };
    if (is_k) {
      if (rank == 0) mbar_arrive_expect_tx(smem_u32(&sh.q_full), mult * Q_BYTES);
#pragma unroll
      for (int a = 0; a < (D * ES) / SWQ; ++a)
        load(q_smem + a * TM * SWQ, &tma_q, lead(&sh.q_full), a * (SWQ / ES), q0);
    }
    for (int j = 0; j < nblk; ++j) {
      const int s = j % stages;
      const uint32_t r = static_cast<uint32_t>(j / stages);
      if (!mbar_wait(smem_u32(&empty[s]), (r & 1u) ^ 1u, abort_flag, err, kErrWaitProducer)) {
        ok = false;
        break;
      }
      const uint32_t fb = lead(&full[s]);
      const uint32_t dst = ring + static_cast<uint32_t>(s) * KV_SLOT;
      if (rank == 0) mbar_arrive_expect_tx(smem_u32(&full[s]), mult * KV_BYTES);
      if (is_k) {
        // K rows [j*BN + rank*KROWS, +KROWS), all D columns (K-major atoms)
#pragma unroll
        for (int a = 0; a < (D * ES) / SWQ; ++a)
          load(dst + a * KROWS * SWQ, map, fb, a * (SWQ / ES), j * BN + static_cast<int>(rank) * KROWS);
      } else {
        // V rows [j*BN, +BN), columns [rank*VCOLS, +VCOLS) (MN-major chunks)
#pragma unroll
        for (int a = 0; a < (VCOLS * ES) / SWV; ++a)
          load(dst + a * BN * SWV, map, fb, static_cast<int>(rank) * VCOLS + a * (SWV / ES), j * BN);
      }
      issued = j + 1;
    }
    if (!ok) {
      if (rank == 0) {
        if (is_k) mbar_wait_drain(smem_u32(&sh.q_full), 0, err);
        for (int j = max(0, issued - stages); j < issued; ++j)
          mbar_wait_drain(smem_u32(&full[j % stages]), static_cast<uint32_t>(j / stages) & 1u,
                          err);
      } else {
        // the odd CTA's loads complete on the even CTA's barriers, which it
        // cannot poll: give in-flight copies time to land before exiting
        const unsigned long long t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ----------------------------------------------- MMA issuer (even CTA)
    bool ok = mbar_wait(smem_u32(&sh.q_full), 0, abort_flag, err, kErrWaitMma);
    // commits reach this CTA's barrier and, for a pair, the odd CTA's twin
    auto commit2 = [&](const uint64_t* bar) {
      if constexpr (PAIR) {
        mma_commit_pair(smem_u32(bar));
        mma_commit_pair(mapa_shared(smem_u32(bar), 1));
      } else {
        mma_commit(smem_u32(bar));
      }
    };
    // O += P(i) V(i), then release V slot i.
    auto pv_round = [&](int i) -> bool {
      const int s = i % stages;
      const uint32_t r = static_cast<uint32_t>(i / stages);
      const int b = i % NB;
      const uint32_t u = static_cast<uint32_t>(i / NB);
      if (!mbar_wait(smem_u32(&sh.v_full[s]), r & 1u, abort_flag, err, kErrWaitMma)) return false;
      if (!mbar_wait<PAIR>(smem_u32(&sh.p_full[b]), u & 1u, abort_flag, err, kErrWaitMma))
        return false;
      tc_fence_after();
      const uint32_t vs = v_smem + static_cast<uint32_t>(s) * KV_SLOT;
      // P(i) sits in the first BN/2 columns of S/P buffer b (16-bit pairs)
      const uint32_t pa = tmem + static_cast<uint32_t>(D + b * BN);
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        const uint64_t bdesc = make_smem_desc(vs + kk * 16 * SWV, BN * SWV, 8 * SWV, SWV);
        const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
        if constexpr (PAIR)
          mma_f16_ts_pair(tmem, pa + static_cast<uint32_t>(kk * 8), bdesc, IDESC_O, acc);
        else
          mma_f16_ts(tmem, pa + static_cast<uint32_t>(kk * 8), bdesc, IDESC_O, acc);
      }
      commit2(&sh.pv_done[b]);
      commit2(&sh.v_empty[s]);
      return true;
    };
    for (int j = 0; j < nblk && ok; ++j) {
      const int s = j % stages;
      const uint32_t r = static_cast<uint32_t>(j / stages);
      const int b = j % NB;
      if (!mbar_wait(smem_u32(&sh.k_full[s]), r & 1u, abort_flag, err, kErrWaitMma)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t ks = k_smem + static_cast<uint32_t>(s) * KV_SLOT;
      // Buffer b last held P(j - NB), whose PV MMA this thread issued
      // earlier; tcgen05 MMAs of one thread execute in issue order.
      const uint32_t s_tmem = tmem + static_cast<uint32_t>(D + b * BN);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t kbyte = static_cast<uint32_t>(kk) * 32u;
        const uint32_t aoff = (kbyte / SWQ) * (TM * SWQ) + (kbyte % SWQ);
        const uint32_t boff = (kbyte / SWQ) * (KROWS * SWQ) + (kbyte % SWQ);
        const uint64_t adesc = make_smem_desc(q_smem + aoff, 16, 8 * SWQ, SWQ);
        const uint64_t bdesc = make_smem_desc(ks + boff, 16, 8 * SWQ, SWQ);
        if constexpr (PAIR)
          mma_f16_ss_pair(s_tmem, adesc, bdesc, IDESC_S, kk > 0 ? 1u : 0u);
        else
          mma_f16_ss(s_tmem, adesc, bdesc, IDESC_S, kk > 0 ? 1u : 0u);
      }
      commit2(&sh.s_full[b]);
      commit2(&sh.k_empty[s]);
      if (j >= LAG && !pv_round(j - LAG)) {
        ok = false;
        break;
      }
    }
    for (int i = max(0, nblk - LAG); i < nblk && ok; ++i) ok = pv_round(i);
    if (!ok) {
      if constexpr (PAIR)
        mma_commit_pair(smem_u32(&sh.drain));
      else
        mma_commit(smem_u32(&sh.drain));
      mbar_wait_drain(smem_u32(&sh.drain), 0, err);
    }
  } else if (warp >= 4) {
    // ------------------------------------------- softmax / correction / epilogue
    const int wg = (warp - 4) >> 2;  // warpgroup: which half of the columns
    const int q = warp & 3;          // TMEM lane quarter of this warp
    // query row within the tile: TMEM lane 32q + lane (TM = 64: lanes
    // 32q + [0, 16) hold rows 16q + lane; the other lanes carry no row and
    // mask their whole S row, so their P is 0 and they store nothing)
    const int row = TM == 128 ? q * 32 + lane : q * 16 + lane;
    const bool active = TM == 128 || lane < 16;
    const int qrow = active ? q0 + row : S;
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t o_tmem = tmem + lane_addr + static_cast<uint32_t>(wg * OC);
    const int col0 = wg * SC;  // first S column of this warp
    const float2 scale2 = make_float2(scale_log2, scale_log2);
    float m_used = -INFINITY;
    float l = 0.f;
    bool ok = true;
    // A failed (timed-out) wait clears ok; the loop then still runs to the
    // end without touching TMEM so that both warps of a row pair meet at
    // every named barrier (the other waits fail fast once abort is raised).
    for (int j = 0; j < nblk; ++j) {
      const int b = j % NB;
      const uint32_t u = static_cast<uint32_t>(j / NB);
      const uint32_t sp = tmem + lane_addr + static_cast<uint32_t>(D + b * BN);
      if (ok && !mbar_wait(smem_u32(&sh.s_full[b]), u & 1u, abort_flag, err, kErrWaitSoftmax))
        ok = false;
      ok = __all_sync(0xffffffffu, ok);  // warp-uniform from here on
      tc_fence_after();
      uint32_t sv[SC];  // S scores (fp32 bits) as the TMEM loads leave them
      float mb = 0.f;
      // Mask padding / future keys only where the block needs it (block-
      // uniform test on the tile's first row); work on raw scores, with the
      // log2-domain scale folded into the exponent's FMA below.
      const int key0 = j * BN + col0;
      const bool need_mask = j * BN + BN > S || (CAUSAL && j * BN + BN - 1 > q0);
      auto f = [&](int i) { return __uint_as_float(sv[i]); };
      if (ok) {
        // this warp's share of S_j -> sv, all TMEM loads in flight before
        // one wait
#pragma unroll
        for (int c = 0; c < SC / SCH; ++c)
          tmem_ld_cols<SCH>(sp + static_cast<uint32_t>(col0 + c * SCH), sv + c * SCH);
        tmem_wait_ld();
        if (need_mask || !active) {
#pragma unroll
          for (int i = 0; i < SC; ++i) {
            const int key = key0 + i;
            if (!active || key >= S || (CAUSAL && key > qrow)) sv[i] = __float_as_uint(-INFINITY);
          }
        }
        // row max: four independent three-input max chains
        float mx[4] = {f(0), f(1), f(2), f(3)};
#pragma unroll
        for (int i = 4; i + 1 < SC; i += 2)
          mx[(i >> 1) & 3] = fmax3(mx[(i >> 1) & 3], f(i), f(i + 1));
        mb = fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]) * scale_log2;
      }
      if constexpr (WG == 2) {
        // combine with the other half of the row (warp pair q, q + 4); the
        // barrier also orders both warps' S loads before either P store
        xchg[((j & 1) * 2 + wg) * 128 + row] = mb;
        tc_fence_before();
        named_barrier(1 + q, 64);
        tc_fence_after();
        mb = fmaxf(mb, xchg[((j & 1) * 2 + (wg ^ 1)) * 128 + row]);
      }
      if (!ok) continue;
      if (j == 0) {
        m_used = mb;
      } else {
        const bool need = mb > m_used + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          const float m_new = need ? mb : m_used;
          const float alpha = ex2_approx(m_used - m_new);
          // O holds PV_0..PV_{j-1}; wait for PV_{j-1} before rescaling it
          const int pj = j - 1;
          ok = mbar_wait(smem_u32(&sh.pv_done[pj % NB]), static_cast<uint32_t>(pj / NB) & 1u,
                         abort_flag, err, kErrWaitSoftmax);
          if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            continue;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < OC / OCH; ++c) {
            uint32_t r[OCH];
            const uint32_t addr = o_tmem + static_cast<uint32_t>(c * OCH);
            tmem_ld_cols<OCH>(addr, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < OCH; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st_cols<OCH>(addr, r);
          }
          tmem_wait_st();
          l *= alpha;
          m_used = m_new;
        }
      }
      // P_j = exp2(s * scale - m_used) with packed fp32x2 FMAs, row sum in
      // four packed partial sums
      const float neg_m = (m_used == -INFINITY) ? 0.f : -m_used;
      const float2 shift2 = make_float2(neg_m, neg_m);
      float2 rs[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                      make_float2(0.f, 0.f)};
      // P_j -> TMEM over the first BN/2 columns of its own S buffer (this
      // warp: columns [col0/2, col0/2 + SC/2)), 16 columns as soon as they
      // are packed.  The MMA issuer writes S_{j+NB} into this buffer only
      // after issuing PV_j, and tcgen05 MMAs execute in issue order.
#pragma unroll
      for (int c = 0; c < (SC / 2) / 16; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int g2 = 0; g2 < 16; ++g2) {
          const int g = c * 16 + g2;
          const float2 x = __ffma2_rn(make_float2(f(2 * g), f(2 * g + 1)), scale2, shift2);
          const float2 p = make_float2(ex2_approx(x.x), ex2_approx(x.y));  // -inf -> 0
          rs[g & 3] = __fadd2_rn(rs[g & 3], p);
          pk[g2] = FMT == 1 ? pack_bf16(p.x, p.y) : pack_f16(p.x, p.y);
        }
        tmem_st16(sp + static_cast<uint32_t>(col0 / 2 + c * 16), pk);
      }
      const float2 rs01 = __fadd2_rn(rs[0], rs[1]), rs23 = __fadd2_rn(rs[2], rs[3]);
      const float2 rsum = __fadd2_rn(rs01, rs23);
      l += rsum.x + rsum.y;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_cluster(mapa_shared(smem_u32(&sh.p_full[b]), 0));  // even CTA's barrier
        else
          mbar_arrive(smem_u32(&sh.p_full[b]));
      }
    }
    // ------------------------------------------------------------ epilogue
    if (ok && nblk > 0) {
      const int pj = nblk - 1;
      ok = mbar_wait(smem_u32(&sh.pv_done[pj % NB]), static_cast<uint32_t>(pj / NB) & 1u,
                     abort_flag, err, kErrWaitSoftmax);
    }
    ok = __all_sync(0xffffffffu, ok);
    if constexpr (WG == 2) {
      // full row sum from both halves (both warps of the pair reach this
      // barrier whether or not their waits succeeded)
      xchg[((nblk & 1) * 2 + wg) * 128 + row] = l;
      named_barrier(1 + q, 64);
      l += xchg[((nblk & 1) * 2 + (wg ^ 1)) * 128 + row];
    }
    if (ok) {
      tc_fence_after();
      const float inv_l = l > 0.f ? 1.0f / l : 0.f;
      T* orow = O + (static_cast<int64_t>(bh) * S + qrow) * D + wg * OC;
#pragma unroll 1
      for (int c = 0; c < OC / OCH; ++c) {
        uint32_t r[OCH];
        tmem_ld_cols<OCH>(o_tmem + static_cast<uint32_t>(c * OCH), r);
        tmem_wait_ld();
        if (qrow < S) {
          uint32_t pk[OCH / 2];
#pragma unroll
          for (int i = 0; i < OCH / 2; ++i) {
            const float lo = __uint_as_float(r[2 * i]) * inv_l;
            const float hi = __uint_as_float(r[2 * i + 1]) * inv_l;
            pk[i] = FMT == 1 ? pack_bf16(lo, hi) : pack_f16(lo, hi);
          }
          uint4* d4 = reinterpret_cast<uint4*>(orow + c * OCH);
#pragma unroll
          for (int i = 0; i < OCH / 8; ++i)
            d4[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // no CTA leaves while its peer may still signal it
  tc_fence_after();
  if (warp == 2) {
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem, ALLOC);
    else
      tmem_dealloc(tmem, ALLOC);
  }
}

// ------------------------------------------------ two query tiles per CTA
// BLOCK_M 256 with num_warps 8: persistent CTAs, one per SM, each taking
// (256-row query span, head) work items from a counter; an item is two
// 128-row query tiles, t = 0 and 1, that share every K/V block.  The next
// item's Q load and first S MMAs run under the current item's epilogue (Q
// is reloaded once the item's last S MMAs are done, O_t is rewritten once
// the epilogue has read it), and the K/V rings run on across items.  TMEM
// holds O_t in columns [t*D, t*D + D) and one S/P buffer per tile in
// [2D + t*BN, 2D + (t+1)*BN).  The MMA thread alternates the tiles
//     ... PV_0(j), S_0(j+1), PV_1(j), S_1(j+1), PV_0(j+1), S_0(j+2) ...
// so while softmax warpgroup t turns S_t(j) into P_t(j), the tensor pipe
// runs the other tile's PV and S MMAs: each tile's chain S -> softmax -> PV
// overlaps the other's, and every SM sub-partition holds one softmax warp
// of each tile.  S_t(j+1) is written over P_t(j) only after PV_t(j) was
// issued (tcgen05 MMAs of one thread execute in issue order).
// Warps: 0 TMA of Q (both tiles, once) and the K ring, 3 TMA of the V ring,
// 1 MMA issuer, 2 TMEM owner, 4-7 softmax of tile 0 (TMEM lanes = rows),
// 8-11 softmax of tile 1.  The softmax is the one-tile kernel's: running
// max in the log2 domain moved (with the O rescale) only past the lazy
// threshold, P = exp2(s - m) as 16-bit pairs into TMEM, fp32 row sums;
// each softmax warpgroup writes its tile's output.
struct AttnDualShared {
  uint64_t q_full;
  uint64_t k_full[kAttnMaxStages];
  uint64_t k_empty[kAttnMaxStages];
  uint64_t v_full[kAttnMaxStages];
  uint64_t v_empty[kAttnMaxStages];
  uint64_t s_full[2];
  uint64_t p_full[2][2];  // [tile][half of the block's keys]
  uint64_t pv_done[2];
  uint64_t q_empty;    // the item's last S MMAs are done: Q may be reloaded
  uint64_t o_free[2];  // the epilogue has read O_t out of TMEM
  uint64_t item_full[2];   // the CTA's next work item is published in item[]
  uint64_t item_empty[2];  // every other role has read it: the slot is free
  int item[2];             // work item of the CTA's it-th turn at [it & 1]; -1: none
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

constexpr int kAttnDualThreads = 384;
constexpr int kAttnCausalGroup = 16;  // heads per longest-first group (causal grids)
// Register split: the kernel launches at 65536 / 384 = 168 registers per
// thread (64512 for the CTA); the warpgroup of producers, MMA issuer and
// TMEM owner gives back down to kAttnDualLowRegs and each softmax
// warpgroup (a 128-column S row per thread) grows to kAttnDualHighRegs:
// 128 * 88 + 256 * 208 = 64512, the launch's total, so every increase
// is covered (the persistent MMA thread spills below 88).
constexpr int kAttnDualLowRegs = 88;
constexpr int kAttnDualHighRegs = 208;
static_assert(128 * kAttnDualLowRegs + 256 * kAttnDualHighRegs <= 168 * kAttnDualThreads,
              "register split exceeds the launch's registers");

// Work items of the persistent two-tile kernel are handed out in order by
// an atomic counter: a CTA takes the next item when it starts one, so the
// causal spans of different lengths spread evenly over the SMs (a fixed
// round-robin of the same order left the busiest SM 10 % above the mean).
// Each launch uses one of kAttnWorkSlots counter pairs {next item, CTAs
// done}, chosen round-robin by the host; the last CTA to finish sets its
// pair back to zero for the next launch that gets the slot.  Launches that
// overlap on one device use different slots unless more than
// kAttnWorkSlots of them run at once.
constexpr int kAttnWorkSlots = 64;
__device__ unsigned int g_attn_work[kAttnWorkSlots][2];

// Work item i: the 256-row query span and head it covers.  Full attention
// walks the spans of one head after another, so the CTAs in flight share
// the K/V of a few heads in L2.  Causal spans go longest first across groups of
// kAttnCausalGroup heads: items are then handed out longest first over the
// whole GPU (a per-head order leaves short spans of the first heads and
// long spans of the last ones in the same wave), while the K/V of the heads
// in flight stay within L2.
template <bool CAUSAL>
__device__ __forceinline__ void attn_dual_item(int i, int spans, int BH, int& span, int& bh) {
  if constexpr (CAUSAL) {
    const int per_group = kAttnCausalGroup * spans;
    const int g = i / per_group;
    const int r = i - g * per_group;
    const int gh = min(kAttnCausalGroup, BH - g * kAttnCausalGroup);
    span = spans - 1 - r / gh;
    bh = g * kAttnCausalGroup + r % gh;
  } else {
    span = i % spans;
    bh = i / spans;
  }
}

// K/V blocks of query tile t (0 or 1) of the span starting at row q0.
template <int BN, bool CAUSAL>
__device__ __forceinline__ int attn_dual_blocks(int S, int q0, int t) {
  const int len = CAUSAL ? min(S, q0 + 128 * (t + 1)) : S;
  return (len + BN - 1) / BN;
}

// The item of the CTA's it-th turn, published by the K producer (-1: no
// more work); the caller's warp (all lanes, WARP) or thread has read it once
// it returns.  Returns false when the wait fails.
constexpr int kAttnItemReaders = 10;  // V producer, MMA thread, 8 softmax warps
template <bool WARP>
__device__ __forceinline__ bool attn_dual_next_item(AttnDualShared& sh, int it,
                                                    volatile int* abort_flag, unsigned int* err,
                                                    uint32_t site, int& item) {
  if (!mbar_wait(smem_u32(&sh.item_full[it & 1]), static_cast<uint32_t>(it >> 1) & 1u,
                 abort_flag, err, site))
    return false;
  item = *reinterpret_cast<volatile int*>(&sh.item[it & 1]);
  if (WARP) __syncwarp();
  if (!WARP || (threadIdx.x & 31) == 0) mbar_arrive(smem_u32(&sh.item_empty[it & 1]));
  return true;
}

// Position in a ring of `stages` slots: slot and the parity of its round.
struct RingPos {
  int slot = 0;
  uint32_t parity = 0;
  __device__ __forceinline__ void step(int stages) {
    if (++slot == stages) {
      slot = 0;
      parity ^= 1u;
    }
  }
};

template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

template <int D>
struct AttnDualGeom {
  static constexpr int ES = 2;
  static constexpr int SW = (D * ES) < 128 ? (D * ES) : 128;  // swizzle of Q/K/V rows
  static constexpr uint32_t Q_BYTES = 128u * D * ES;           // one query tile
};

// TMA producer of Q (both tiles of each item) and the K ring (is_k), or of
// the V ring.  The rings run on across items: every item loads the nb1
// blocks of its tile 1.
template <int BN, int D, bool CAUSAL>
__device__ __forceinline__ void attn_dual_producer(const CUtensorMap* tma_q,
                                                   const CUtensorMap* map, AttnDualShared& sh,
                                                   uint32_t q_smem, uint32_t ring, int S,
                                                   int BH, int stages, int work_slot, bool is_k,
                                                   volatile int* abort_flag, unsigned int* err) {
  using G = AttnDualGeom<D>;
  constexpr uint32_t KV_BYTES = static_cast<uint32_t>(BN) * D * G::ES;
  constexpr uint32_t KV_SLOT = (KV_BYTES + 1023u) & ~1023u;
  uint64_t* full = is_k ? sh.k_full : sh.v_full;
  uint64_t* empty = is_k ? sh.k_empty : sh.v_empty;
  const int spans = (S + 255) / 256;
  const int items = spans * BH;
  bool ok = true;
  int issued = 0;      // ring loads issued (over all items)
  int q_loads = 0;     // Q loads issued
  RingPos pos;
  for (int it = 0; ok; ++it) {
    int item;
    if (is_k) {
      // take the next item and publish it to the CTA's other roles, once
      // they have all read the item published two turns ago in this slot
      if (it >= 2 && !mbar_wait(smem_u32(&sh.item_empty[it & 1]),
                                static_cast<uint32_t>((it >> 1) - 1) & 1u, abort_flag, err,
                                kErrWaitProducer)) {
        ok = false;
        break;
      }
      const int next = static_cast<int>(atomicAdd(&g_attn_work[work_slot][0], 1u));
      item = next < items ? next : -1;
      sh.item[it & 1] = item;
      mbar_arrive(smem_u32(&sh.item_full[it & 1]));
    } else {
      ok = attn_dual_next_item<false>(sh, it, abort_flag, err, kErrWaitProducer, item);
    }
    if (!ok || item < 0) break;
    int span, bh;
    attn_dual_item<CAUSAL>(item, spans, BH, span, bh);
    const int q0 = span * 256;
    const int nblk = attn_dual_blocks<BN, CAUSAL>(S, q0, 1);
    if (is_k) {
      // Q of the previous item is free once its last S MMAs are done
      if (it > 0 && !mbar_wait(smem_u32(&sh.q_empty), static_cast<uint32_t>(it - 1) & 1u,
                               abort_flag, err, kErrWaitProducer)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(smem_u32(&sh.q_full), 2u * G::Q_BYTES);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int a = 0; a < (D * G::ES) / G::SW; ++a)
          tma_load_3d(q_smem + t * G::Q_BYTES + a * 128 * G::SW, tma_q, smem_u32(&sh.q_full),
                      a * (G::SW / G::ES), q0 + 128 * t, bh);
      ++q_loads;
    }
    for (int j = 0; j < nblk; ++j) {
      if (!mbar_wait(smem_u32(&empty[pos.slot]), pos.parity ^ 1u, abort_flag, err,
                     kErrWaitProducer)) {
        ok = false;
        break;
      }
      const uint32_t dst = ring + static_cast<uint32_t>(pos.slot) * KV_SLOT;
      mbar_arrive_expect_tx(smem_u32(&full[pos.slot]), KV_BYTES);
      // K: rows [j*BN, +BN) in K-major atoms; V: the same rows, MN-major
      // column chunks (the B operand of the PV MMA)
#pragma unroll
      for (int a = 0; a < (D * G::ES) / G::SW; ++a)
        tma_load_3d(dst + a * BN * G::SW, map, smem_u32(&full[pos.slot]), a * (G::SW / G::ES),
                    j * BN, bh);
      ++issued;
      pos.step(stages);
    }
  }
  if (!ok) {
    // let the copies in flight land before the CTA can exit
    if (q_loads > 0)
      mbar_wait_drain(smem_u32(&sh.q_full), static_cast<uint32_t>(q_loads - 1) & 1u, err);
    for (int g = max(0, issued - stages); g < issued; ++g)
      mbar_wait_drain(smem_u32(&full[g % stages]), static_cast<uint32_t>(g / stages) & 1u, err);
  }
}

// MMA issuer: S_t(j) = Q_t K_j^T and O_t += P_t(j) V_j, tiles alternating.
template <int FMT, int BN, int D, bool CAUSAL>
__device__ __forceinline__ void attn_dual_mma(AttnDualShared& sh, uint32_t tmem, uint32_t q_smem,
                                              uint32_t k_smem, uint32_t v_smem, int S, int BH,
                                              int stages, volatile int* abort_flag,
                                              unsigned int* err) {
  using G = AttnDualGeom<D>;
  constexpr int SW = G::SW;
  constexpr uint32_t KV_SLOT = ((static_cast<uint32_t>(BN) * D * G::ES) + 1023u) & ~1023u;
  constexpr uint32_t IDESC_S = make_idesc(FMT, 128, BN, false, false);
  constexpr uint32_t IDESC_O = make_idesc(FMT, 128, D, false, true);
  // The tensor pipe runs these MMAs back to back only while this thread
  // issues them faster than they execute, so the work between two groups
  // is kept short: descriptors are built once and advanced by constant
  // offsets (a descriptor's address field is the byte address >> 4, and
  // every shared-memory address stays below 256 KB), ring positions are
  // stepped without division, and each wait first tests the phase without
  // blocking, since the awaited phase has usually completed by then.
  auto wait = [&](const uint64_t* bar, uint32_t parity) {
    const uint32_t b = smem_u32(bar);
    return mbar_test_wait(b, parity) || mbar_wait(b, parity, abort_flag, err, kErrWaitMma);
  };
  constexpr uint64_t HI = smem_desc_hi(8 * SW, SW);  // Q, K (K-major) and V (MN-major)
  const uint32_t q_lo = smem_desc_lo(q_smem, 16);
  const uint32_t k_lo = smem_desc_lo(k_smem, 16);
  const uint32_t v_lo = smem_desc_lo(v_smem, BN * SW);
  auto s_mma = [&](int t, int k_slot) {
    const uint32_t qd = q_lo + static_cast<uint32_t>(t) * (G::Q_BYTES >> 4);
    const uint32_t kd = k_lo + static_cast<uint32_t>(k_slot) * (KV_SLOT >> 4);
    const uint32_t s_tmem = tmem + static_cast<uint32_t>(2 * D + t * BN);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const uint32_t kbyte = static_cast<uint32_t>(kk) * 32u;
      const uint32_t aoff = (kbyte / SW) * (128 * SW) + (kbyte % SW);
      const uint32_t boff = (kbyte / SW) * (BN * SW) + (kbyte % SW);
      mma_f16_ss(s_tmem, HI | (qd + (aoff >> 4)), HI | (kd + (boff >> 4)), IDESC_S,
                 kk > 0 ? 1u : 0u);
    }
    mma_commit(smem_u32(&sh.s_full[t]));
    // S_1 is the last reader of a K block (S_0 of it was issued before)
    if (t == 1) mma_commit(smem_u32(&sh.k_empty[k_slot]));
  };
  // P_t sits in the first BN/2 columns of tile t's S/P buffer
  auto pv_mma = [&](int t, int v_slot, int j, uint32_t par, bool last) {
    const uint32_t vd = v_lo + static_cast<uint32_t>(v_slot) * (KV_SLOT >> 4);
    const uint32_t pa = tmem + static_cast<uint32_t>(2 * D + t * BN);
    const uint32_t o_tmem = tmem + static_cast<uint32_t>(t * D);
    // keys [0, BN/2) as soon as their P is stored, then the rest; when the
    // second half is already released (every softmax warp releases the
    // first half before the second), one test replaces both waits
    const bool all_ready = mbar_test_wait(smem_u32(&sh.p_full[t][1]), par);
    if (all_ready) tc_fence_after();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (!all_ready) {
        if (!wait(&sh.p_full[t][h], par)) return false;
        tc_fence_after();
      }
#pragma unroll
      for (int kk = h * (BN / 32); kk < (h + 1) * (BN / 32); ++kk)
        mma_f16_ts(o_tmem, pa + static_cast<uint32_t>(kk * 8),
                   HI | (vd + static_cast<uint32_t>((kk * 16 * SW) >> 4)), IDESC_O,
                   (j > 0 || kk > 0) ? 1u : 0u);
    }
    if (last) mma_commit(smem_u32(&sh.pv_done[t]));  // for the epilogue
    // PV_1 is the last reader of a V block (PV_0 of it was issued before)
    if (t == 1) mma_commit(smem_u32(&sh.v_empty[v_slot]));
    return true;
  };
  const int spans = (S + 255) / 256;
  bool ok = true;
  RingPos kpos, vpos;         // next K and next V block of the rings
  uint32_t tile_blocks[2] = {0u, 0u};  // blocks of each tile so far: P phases
  for (int it = 0; ok; ++it) {
    int item;
    ok = attn_dual_next_item<false>(sh, it, abort_flag, err, kErrWaitMma, item);
    if (!ok || item < 0) break;
    int span, bh;
    attn_dual_item<CAUSAL>(item, spans, BH, span, bh);
    const int q0 = span * 256;
    const int nb0 = attn_dual_blocks<BN, CAUSAL>(S, q0, 0);
    const int nb1 = attn_dual_blocks<BN, CAUSAL>(S, q0, 1);  // nb0 <= nb1
    const uint32_t itp = static_cast<uint32_t>(it) & 1u;
    // S_t(0) overwrites the S/P buffer that PV_t(last) of the previous item
    // read; that PV was issued before, and MMAs execute in issue order
    ok = wait(&sh.q_full, itp) && wait(&sh.k_full[kpos.slot], kpos.parity);
    if (ok) {
      s_mma(0, kpos.slot);
      s_mma(1, kpos.slot);
      kpos.step(stages);
      if (nb1 == 1) mma_commit(smem_u32(&sh.q_empty));  // the item's last S MMAs
    }
    for (int j = 0; j < nb1 && ok; ++j) {
      if (!wait(&sh.v_full[vpos.slot], vpos.parity)) {
        ok = false;
        break;
      }
      bool k_ready = false;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int nbt = t == 0 ? nb0 : nb1;
        if (ok && j < nbt) {
          // PV_t(0) overwrites O_t: the previous item's epilogue must have
          // read it out
          if (j == 0 && it > 0) {
            ok = wait(&sh.o_free[t], itp ^ 1u);
            tc_fence_after();
          }
          if (ok) ok = pv_mma(t, vpos.slot, j, tile_blocks[t] & 1u, j + 1 == nbt);
          ++tile_blocks[t];
        }
        if (ok && j + 1 < nbt) {
          if (!k_ready) {
            // K arrives by TMA (async proxy, like the MMA's reads): the
            // barrier's phase alone orders it, no tcgen05 fence
            ok = wait(&sh.k_full[kpos.slot], kpos.parity);
            k_ready = true;
          }
          if (ok) {
            s_mma(t, kpos.slot);
            if (t == 1 && j + 2 == nb1) mma_commit(smem_u32(&sh.q_empty));
          }
        }
      }
      vpos.step(stages);
      if (k_ready) kpos.step(stages);
    }
  }
  if (!ok) {
    mma_commit(smem_u32(&sh.drain));
    mbar_wait_drain(smem_u32(&sh.drain), 0, err);
  }
}

// Softmax and epilogue of tile t = (warp - 4) / 4 for each work item of
// the CTA; thread = query row = TMEM lane.
template <typename T, int FMT, int BN, int D, bool CAUSAL>
__device__ __forceinline__ void attn_dual_softmax(AttnDualShared& sh, uint32_t tmem,
                                                  T* __restrict__ O, int S, int BH,
                                                  float scale_log2, int warp, int lane,
                                                  volatile int* abort_flag, unsigned int* err) {
  const int t = (warp - 4) >> 2;
  const int q = warp & 3;  // TMEM lane quarter
  const int row = q * 32 + lane;
  const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
  const uint32_t sp = tmem + lane_addr + static_cast<uint32_t>(2 * D + t * BN);
  const uint32_t o_tmem = tmem + lane_addr + static_cast<uint32_t>(t * D);
  const float2 scale2 = make_float2(scale_log2, scale_log2);
  const int spans = (S + 255) / 256;
  bool ok = true;
  uint32_t tb = 0;  // blocks of this tile so far (over all items): S and P phases
  for (int it = 0; ok; ++it) {
    int item;
    ok = attn_dual_next_item<true>(sh, it, abort_flag, err, kErrWaitSoftmax, item);
    if (!__all_sync(0xffffffffu, ok) || item < 0) break;
    int span, bh;
    attn_dual_item<CAUSAL>(item, spans, BH, span, bh);
    const int q0 = span * 256;
    const int tile_first = q0 + 128 * t;
    const int qrow = tile_first + row;
    const int nblk = attn_dual_blocks<BN, CAUSAL>(S, q0, t);
    float m_used = -INFINITY;
    float l = 0.f;
    for (int j = 0; j < nblk; ++j, ++tb) {
      if (!mbar_wait(smem_u32(&sh.s_full[t]), tb & 1u, abort_flag, err, kErrWaitSoftmax))
        ok = false;
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c)
        tmem_ld32(sp + static_cast<uint32_t>(c * 32), *reinterpret_cast<uint32_t(*)[32]>(sv + c * 32));
      tmem_wait_ld();
      auto f = [&](int i) { return __uint_as_float(sv[i]); };
      const int key0 = j * BN;
      if (key0 + BN > S || (CAUSAL && key0 + BN - 1 > tile_first)) {
        // keys key0 + i with i <= last are visible (i is a constant of the
        // unrolled loop: one compare and one select per score)
        const int last = CAUSAL ? min(S - 1, qrow) - key0 : S - 1 - key0;
#pragma unroll
        for (int i = 0; i < BN; ++i)
          if (i > last) sv[i] = __float_as_uint(-INFINITY);
      }
      float mx[4] = {f(0), f(1), f(2), f(3)};
#pragma unroll
      for (int i = 4; i + 1 < BN; i += 2) mx[(i >> 1) & 3] = fmax3(mx[(i >> 1) & 3], f(i), f(i + 1));
      const float mb = fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]) * scale_log2;
      if (j == 0) {
        m_used = mb;
      } else {
        const bool need = mb > m_used + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          const float m_new = need ? mb : m_used;
          const float alpha = ex2_approx(m_used - m_new);
          // O_t holds PV_t(0..j-1), complete: PV_t(j-1) was issued before
          // S_t(j), which is done, and PV_t(j) waits for this thread's P
#pragma unroll 1
          for (int c = 0; c < D / 16; ++c) {
            uint32_t r[16];
            const uint32_t addr = o_tmem + static_cast<uint32_t>(c * 16);
            tmem_ld16(addr, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st16(addr, r);
          }
          tmem_wait_st();
          l *= alpha;
          m_used = m_new;
        }
      }
      const float neg_m = (m_used == -INFINITY) ? 0.f : -m_used;
      const float2 shift2 = make_float2(neg_m, neg_m);
      float2 rs[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                      make_float2(0.f, 0.f)};
      // P_t(j) over the first BN/2 columns of the buffer, 16 columns as soon
      // as they are packed; the keys of each half of the block are released
      // to the PV MMA as soon as their P is stored, so the MMA on the first
      // half overlaps the exponentials of the second
      auto release = [&](int h) {
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&sh.p_full[t][h]));
      };
      constexpr int HALF_CHUNKS = BN / 64;  // 32-key chunks per half (0: BN 32)
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int g2 = 0; g2 < 16; ++g2) {
          const int g = c * 16 + g2;
          const float2 x = __ffma2_rn(make_float2(f(2 * g), f(2 * g + 1)), scale2, shift2);
          const float2 p = make_float2(ex2_approx(x.x), ex2_approx(x.y));  // -inf -> 0
          rs[g & 3] = __fadd2_rn(rs[g & 3], p);
          pk[g2] = FMT == 1 ? pack_bf16(p.x, p.y) : pack_f16(p.x, p.y);
        }
        tmem_st16(sp + static_cast<uint32_t>(c * 16), pk);
        if (c + 1 == HALF_CHUNKS) release(0);
      }
      const float2 rsum = __fadd2_rn(__fadd2_rn(rs[0], rs[1]), __fadd2_rn(rs[2], rs[3]));
      l += rsum.x + rsum.y;
      if (HALF_CHUNKS == 0) release(0);
      release(1);
    }
    // ------------------------------------------------------------ epilogue
    // pv_done[t] is committed once per item, after the tile's last PV MMA
    if (ok && nblk > 0)
      ok = mbar_wait(smem_u32(&sh.pv_done[t]), static_cast<uint32_t>(it) & 1u, abort_flag, err,
                     kErrWaitSoftmax);
    if (!__all_sync(0xffffffffu, ok)) {
      ok = false;
      break;
    }
    tc_fence_after();
    // O_t to registers, then hand O_t back to the MMA thread (the next item's
    // first PV overwrites it) before normalising and storing
    uint32_t ov[D];
#pragma unroll
    for (int c = 0; c < D / 32; ++c)
      tmem_ld32(o_tmem + static_cast<uint32_t>(c * 32),
                *reinterpret_cast<uint32_t(*)[32]>(ov + c * 32));
    tmem_wait_ld();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&sh.o_free[t]));
    if (qrow < S) {
      const float inv_l = l > 0.f ? 1.0f / l : 0.f;
      T* orow = O + (static_cast<int64_t>(bh) * S + qrow) * D;
#pragma unroll
      for (int c = 0; c < D / 16; ++c) {
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float lo = __uint_as_float(ov[c * 16 + 2 * i]) * inv_l;
          const float hi = __uint_as_float(ov[c * 16 + 2 * i + 1]) * inv_l;
          pk[i] = FMT == 1 ? pack_bf16(lo, hi) : pack_f16(lo, hi);
        }
        uint4* d4 = reinterpret_cast<uint4*>(orow + c * 16);
        d4[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        d4[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
    }
  }
}

template <typename T, int FMT, int BN, int D, bool CAUSAL>
__global__ void __launch_bounds__(kAttnDualThreads, 1)
    attn_tc_dual_kernel(const __grid_constant__ CUtensorMap tma_q,
                        const __grid_constant__ CUtensorMap tma_k,
                        const __grid_constant__ CUtensorMap tma_v, T* __restrict__ O, int BH,
                        int S, int stages, float scale_log2, int work_slot, unsigned int* err) {
  using G = AttnDualGeom<D>;
  constexpr uint32_t KV_SLOT = ((static_cast<uint32_t>(BN) * D * G::ES) + 1023u) & ~1023u;
  constexpr int COLS = 2 * D + 2 * BN;
  constexpr int ALLOC = attn_tmem_alloc(COLS);
  static_assert(COLS <= 512, "TMEM holds 512 columns");
  static_assert(BN % 32 == 0 && D % 32 == 0, "TMEM accesses of 32 columns");

  __shared__ AttnDualShared sh;
  extern __shared__ uint8_t dyn_smem[];
  const uint32_t base = (smem_u32(dyn_smem) + 1023u) & ~1023u;
  const uint32_t q_smem = base;  // tile t at q_smem + t * Q_BYTES
  const uint32_t k_smem = q_smem + 2u * G::Q_BYTES;
  const uint32_t v_smem = k_smem + static_cast<uint32_t>(stages) * KV_SLOT;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&sh.q_full), 1);
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&sh.k_full[s]), 1);
      mbar_init(smem_u32(&sh.k_empty[s]), 1);
      mbar_init(smem_u32(&sh.v_full[s]), 1);
      mbar_init(smem_u32(&sh.v_empty[s]), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&sh.s_full[t]), 1);
      mbar_init(smem_u32(&sh.p_full[t][0]), 4);
      mbar_init(smem_u32(&sh.p_full[t][1]), 4);
      mbar_init(smem_u32(&sh.pv_done[t]), 1);
      mbar_init(smem_u32(&sh.o_free[t]), 4);
    }
    mbar_init(smem_u32(&sh.q_empty), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&sh.item_full[i]), 1);
      mbar_init(smem_u32(&sh.item_empty[i]), kAttnItemReaders);
    }
    mbar_init(smem_u32(&sh.drain), 1);
    sh.abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tma_q);
    tma_prefetch_desc(&tma_k);
    tma_prefetch_desc(&tma_v);
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(&sh.tmem_base), ALLOC);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* abort_flag = &sh.abort;
  // Register split by whole warpgroups; each setmaxnreg heads its role's
  // branch so that the register allocator gives that code the new budget.
  if (warp < 4) {
    regs_dec<kAttnDualLowRegs>();
    if ((warp == 0 || warp == 3) && lane == 0)
      attn_dual_producer<BN, D, CAUSAL>(&tma_q, warp == 0 ? &tma_k : &tma_v, sh, q_smem,
                                        warp == 0 ? k_smem : v_smem, S, BH, stages, work_slot,
                                        warp == 0, abort_flag, err);
    else if (warp == 1 && lane == 0)
      attn_dual_mma<FMT, BN, D, CAUSAL>(sh, tmem, q_smem, k_smem, v_smem, S, BH, stages,
                                        abort_flag, err);
  } else {
    regs_inc<kAttnDualHighRegs>();
    attn_dual_softmax<T, FMT, BN, D, CAUSAL>(sh, tmem, O, S, BH, scale_log2, warp, lane,
                                             abort_flag, err);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, ALLOC);
  if (threadIdx.x == 0) {
    // every CTA has taken its last item before it counts itself done, so the
    // last one can clear the slot
    unsigned int* work = g_attn_work[work_slot];
    if (atomicAdd(&work[1], 1u) == gridDim.x - 1) {
      atomicExch(&work[0], 0u);
      atomicExch(&work[1], 0u);
    }
  }
}

// ------------------------------------------------------------------- host
typedef CUresult (*EncodeTiledFn3)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// (BH, S, D) tensor as a 3-D map {D, S, BH} with box {sw/es, rows, 1}.
static bool encode_bsd(CUtensorMap* map, CUtensorMapDataType dt, const void* ptr, uint64_t BH,
                       uint64_t S, uint64_t D, uint32_t rows, int sw) {
  EncodeTiledFn3 fn = reinterpret_cast<EncodeTiledFn3>(tensor_map_encoder());
  if (!fn) return false;
  const cuuint64_t dims[3] = {D, S, BH};
  const cuuint64_t strides[2] = {D * 2, S * D * 2};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(sw / 2), rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapSwizzle swz = sw == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : sw == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                            : CU_TENSOR_MAP_SWIZZLE_32B;
  return fn(map, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static uint32_t attn_tc_smem(int BN, int D, int stages, bool pair, int tm) {
  auto al = [](uint32_t x) { return (x + 1023u) & ~1023u; };
  const uint32_t q = static_cast<uint32_t>(tm) * D * 2;
  const uint32_t kv = static_cast<uint32_t>(pair ? BN / 2 : BN) * D * 2;  // a K (or V) slot
  return al(q) + static_cast<uint32_t>(stages) * 2 * al(kv) + 1024u;
}

// Plan: aux[0] = dynamic smem bytes, aux[1] = softmax warpgroups (WG),
// aux[2] = CTA pair, aux[3] = S/P buffers, aux[4] = query rows per CTA.
// BLOCK_M 64 -> one 64-row query tile per CTA (M=64 MMAs, one softmax
// warpgroup); 128 -> one 128-row query tile per CTA; 256 -> a cluster of two
// CTAs on two consecutive query tiles of a head, sharing each K/V block
// through M=256 cta_group::2 MMAs (each CTA stages half of K's rows and half
// of V's columns, halving the shared-memory and TMA bytes per tile).
// num_warps 4 -> one softmax warpgroup; 8 -> two splitting each row's
// columns (BLOCK_N >= 64; with BLOCK_N 32 a warp would hold fewer than the
// 32 columns of one TMEM access, so the kernel keeps one warpgroup).
static uint32_t attn_dual_smem(int BN, int D, int stages) {
  auto al = [](uint32_t x) { return (x + 1023u) & ~1023u; };
  const uint32_t q = 2u * 128u * static_cast<uint32_t>(D) * 2u;
  const uint32_t kv = static_cast<uint32_t>(BN) * D * 2u;
  return al(q) + static_cast<uint32_t>(stages) * 2 * al(kv) + 1024u;
}

// BLOCK_M 256 with num_warps 8: two 128-row query tiles per CTA
// (attn_tc_dual_kernel); aux[2] = 2 marks it.
static gpo_status plan_attention_dual(const gpo_key& k, Plan& p, std::string& log) {
  const int D = static_cast<int>(k.shape[2]);
  const int BN = k.block_n;
  if (k.num_stages < 1 || k.num_stages > kAttnMaxStages) {
    log = "num_stages must be in [1, 4]";
    return GPO_BAD_CONFIG;
  }
  const int cols = 2 * D + 2 * BN;
  if (cols > static_cast<int>(kTmemCols)) {
    log = "TMEM needs " + std::to_string(cols) + " columns (2 O tiles x " + std::to_string(D) +
          " + 2 S buffers x " + std::to_string(BN) + ") > 512";
    return GPO_COMPILE_ERROR;
  }
  const uint32_t dyn = attn_dual_smem(BN, D, k.num_stages);
  const uint32_t smem = dyn + static_cast<uint32_t>(sizeof(AttnDualShared));
  if (smem > kMaxSmemPerCta) {
    log = "shared memory " + std::to_string(smem) + " B (2 Q tiles + " +
          std::to_string(k.num_stages) + " K and V stages) exceeds the 232448 B per-CTA limit";
    return GPO_COMPILE_ERROR;
  }
  p.aux[0] = static_cast<int>(dyn);
  p.aux[1] = 1;
  p.aux[2] = 2;
  p.aux[3] = 1;
  p.aux[4] = 128;
  p.family = "attn_tc";
  p.res.smem_bytes = smem;
  p.res.tmem_cols = static_cast<uint32_t>(attn_tmem_alloc(cols));
  p.res.threads_per_cta = static_cast<uint32_t>(kAttnDualThreads);
  // persistent: one CTA per SM at launch, at most one per work item
  p.res.grid_x = static_cast<uint32_t>(cdiv(k.shape[1], 256) * k.shape[0]);
  p.res.grid_y = p.res.grid_z = 1;
  p.res.persistent = 1u;
  p.res.launches_per_call = 1;
  snprintf(p.res.kernel, sizeof(p.res.kernel), "attn_tc_dual_kernel<%s,BN=%d,D=%d,%s,two_tiles>",
           k.dtype == GPO_BFLOAT16 ? "bf16" : "f16", BN, D,
           k.task == GPO_TASK_ATTENTION_CAUSAL ? "causal" : "full");
  return GPO_OK;
}

gpo_status plan_attention_tc(const gpo_key& k, Plan& p, std::string& log) {
  if (k.block_m == 256 && k.num_warps == 8) return plan_attention_dual(k, p, log);
  const int D = static_cast<int>(k.shape[2]);
  const int BN = k.block_n;
  const bool pair = k.block_m == 256;
  const int tm = k.block_m == 64 ? 64 : 128;  // query rows per CTA
  const int wg = (k.num_warps == 8 && BN >= 64 && tm == 128) ? 2 : 1;
  if (k.num_stages < 1 || k.num_stages > kAttnMaxStages) {
    log = "num_stages must be in [1, 4]";
    return GPO_BAD_CONFIG;
  }
  const int min_cols = D + 2 * BN;
  if (min_cols > static_cast<int>(kTmemCols)) {
    log = "TMEM needs " + std::to_string(min_cols) + " columns (O " + std::to_string(D) +
          " + 2 S buffers x " + std::to_string(BN) + ") > 512";
    return GPO_COMPILE_ERROR;
  }
  const uint32_t dyn =
      attn_tc_smem(BN, D, k.num_stages, pair, tm) + (wg == 2 ? kAttnXchgBytes : 0u);
  const uint32_t smem = dyn + static_cast<uint32_t>(sizeof(AttnShared));
  // two CTAs per SM when two S/P buffers fit TMEM's half and shared memory
  // holds two CTAs (228 KB per SM, 1 KB reserved per CTA)
  const bool duo =
      !pair && wg == 1 && attn_duo_nb(D, BN) > 0 && 2u * (smem + 1024u) <= 233472u;
  const int nb = duo ? attn_duo_nb(D, BN) : attn_sbufs(D, BN);
  const int cols_needed = D + nb * BN;
  if (smem > kMaxSmemPerCta) {
    log = "shared memory " + std::to_string(smem) + " B (Q tile + " +
          std::to_string(k.num_stages) + " K and V stages) exceeds the 232448 B per-CTA limit";
    return GPO_COMPILE_ERROR;
  }
  p.aux[0] = static_cast<int>(dyn);
  p.aux[1] = wg;
  p.aux[2] = pair ? 1 : 0;
  p.aux[3] = nb;
  p.aux[4] = tm;
  p.family = "attn_tc";
  p.res.smem_bytes = smem;
  p.res.tmem_cols = static_cast<uint32_t>(attn_tmem_alloc(cols_needed));
  p.res.threads_per_cta = static_cast<uint32_t>(128 + 128 * wg);
  p.res.grid_x = static_cast<uint32_t>(pair ? 2 * cdiv(k.shape[1], 256) : cdiv(k.shape[1], tm));
  p.res.grid_y = static_cast<uint32_t>(k.shape[0]);
  p.res.grid_z = 1;
  p.res.launches_per_call = 1;
  snprintf(p.res.kernel, sizeof(p.res.kernel), "attn_tc_kernel<%s,%sBN=%d,D=%d,%s,wg=%d,sbufs=%d%s>",
           k.dtype == GPO_BFLOAT16 ? "bf16" : "f16", tm == 64 ? "BM=64," : "", BN, D,
           k.task == GPO_TASK_ATTENTION_CAUSAL ? "causal" : "full", wg, nb,
           pair ? ",cta_pair" : "");
  return GPO_OK;
}

template <typename T, int FMT, int BN, int D, bool CAUSAL, int WG, bool PAIR, int NB,
          int TM = 128>
static gpo_status run_attn_tc_wg(const gpo_key& k, const Plan& p, const gpo_args& a,
                                 const LaunchCtx& c, CUtensorMapDataType dt) {
  const uint64_t BH = static_cast<uint64_t>(k.shape[0]), S = static_cast<uint64_t>(k.shape[1]);
  constexpr int SW = (D * 2) < 128 ? (D * 2) : 128;
  constexpr int SWV = (PAIR ? D : D * 2) < 128 ? (PAIR ? D : D * 2) : 128;  // V half: D/2 columns
  CUtensorMap mq, mk, mv;
  if (!encode_bsd(&mq, dt, a.in[0], BH, S, D, TM, SW) ||
      !encode_bsd(&mk, dt, a.in[1], BH, S, D, PAIR ? BN / 2 : BN, SW) ||
      !encode_bsd(&mv, dt, a.in[2], BH, S, D, BN, SWV))
    return GPO_LAUNCH_ERROR;
  auto kern = attn_tc_kernel<T, FMT, BN, D, CAUSAL, WG, PAIR, NB, TM>;
  const uint32_t dyn = static_cast<uint32_t>(p.aux[0]);
  gpo_status s = ensure_smem_attr(reinterpret_cast<const void*>(kern), dyn);
  if (s != GPO_OK) return s;
  const dim3 grid(static_cast<unsigned>(PAIR ? 2 * cdiv(S, 256) : cdiv(S, TM)),
                  static_cast<unsigned>(BH));
  const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
  T* out = static_cast<T*>(a.out);
  const int Si = static_cast<int>(S), stages = k.num_stages;
  if constexpr (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(128 + 128 * WG, 1, 1);
    cfg.dynamicSmemBytes = dyn;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, out, Si, stages, scale_log2, c.err) !=
        cudaSuccess)
      return launch_status();
  } else {
    kern<<<grid, 128 + 128 * WG, dyn, c.stream>>>(mq, mk, mv, out, Si, stages, scale_log2,
                                                   c.err);
  }
  return launch_status();
}

template <typename T, int FMT, int BN, int D, bool CAUSAL>
static gpo_status run_attn_tc_dual(const gpo_key& k, const Plan& p, const gpo_args& a,
                                   const LaunchCtx& c, CUtensorMapDataType dt) {
  const uint64_t BH = static_cast<uint64_t>(k.shape[0]), S = static_cast<uint64_t>(k.shape[1]);
  constexpr int SW = (D * 2) < 128 ? (D * 2) : 128;
  CUtensorMap mq, mk, mv;
  if (!encode_bsd(&mq, dt, a.in[0], BH, S, D, 128, SW) ||
      !encode_bsd(&mk, dt, a.in[1], BH, S, D, BN, SW) ||
      !encode_bsd(&mv, dt, a.in[2], BH, S, D, BN, SW))
    return GPO_LAUNCH_ERROR;
  auto kern = attn_tc_dual_kernel<T, FMT, BN, D, CAUSAL>;
  const uint32_t dyn = static_cast<uint32_t>(p.aux[0]);
  gpo_status s = ensure_smem_attr(reinterpret_cast<const void*>(kern), dyn);
  if (s != GPO_OK) return s;
  // persistent CTAs (one per SM: shared memory and TMEM) taking (span,
  // head) items from the launch's work counter
  const uint64_t items = cdiv(S, 256) * BH;
  const dim3 grid(static_cast<unsigned>(
      std::min<uint64_t>(items, static_cast<uint64_t>(c.sm_count > 0 ? c.sm_count : 148))));
  const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
  static std::atomic<unsigned> launches{0};
  const int work_slot = static_cast<int>(launches.fetch_add(1u) % kAttnWorkSlots);
  kern<<<grid, kAttnDualThreads, dyn, c.stream>>>(mq, mk, mv, static_cast<T*>(a.out),
                                                  static_cast<int>(BH), static_cast<int>(S),
                                                  k.num_stages, scale_log2, work_slot, c.err);
  return launch_status();
}

template <typename T, int FMT, int BN, int D, bool CAUSAL>
static gpo_status run_attn_tc(const gpo_key& k, const Plan& p, const gpo_args& a,
                              const LaunchCtx& c, CUtensorMapDataType dt) {
  if (p.aux[2] == 2) {
    if constexpr (2 * D + 2 * BN <= 512) return run_attn_tc_dual<T, FMT, BN, D, CAUSAL>(k, p, a, c, dt);
    return GPO_INTERNAL;  // rejected by the plan (TMEM)
  }
  if constexpr (D + 2 * BN <= 512) {
    constexpr int NB = attn_sbufs(D, BN);
    const bool pair = p.aux[2] != 0;
    constexpr int NBD = attn_duo_nb(D, BN);
    if (p.aux[4] == 64) {  // 64-row query tiles: one warpgroup, no pair
      if (pair || p.aux[1] != 1) return GPO_INTERNAL;
      if constexpr (NBD > 0) {
        if (p.aux[3] == NBD) return run_attn_tc_wg<T, FMT, BN, D, CAUSAL, 1, false, NBD, 64>(k, p, a, c, dt);
      }
      if (p.aux[3] != NB) return GPO_INTERNAL;
      return run_attn_tc_wg<T, FMT, BN, D, CAUSAL, 1, false, NB, 64>(k, p, a, c, dt);
    }
    if constexpr (NBD > 0) {
      if (p.aux[3] == NBD) {
        if (pair || p.aux[1] != 1) return GPO_INTERNAL;
        return run_attn_tc_wg<T, FMT, BN, D, CAUSAL, 1, false, NBD>(k, p, a, c, dt);
      }
    }
    if (p.aux[3] != NB) return GPO_INTERNAL;
    if constexpr (BN >= 64) {
      // two softmax warpgroups: one 128-row tile per CTA (BLOCK_M 256 with
      // 8 warps is the two-tile kernel)
      if (p.aux[1] == 2) {
        if (pair) return GPO_INTERNAL;
        return run_attn_tc_wg<T, FMT, BN, D, CAUSAL, 2, false, NB>(k, p, a, c, dt);
      }
    }
    if (p.aux[1] != 1) return GPO_INTERNAL;
    return pair ? run_attn_tc_wg<T, FMT, BN, D, CAUSAL, 1, true, NB>(k, p, a, c, dt)
                : run_attn_tc_wg<T, FMT, BN, D, CAUSAL, 1, false, NB>(k, p, a, c, dt);
  } else {
    return GPO_INTERNAL;  // rejected by the plan (TMEM)
  }
}

template <typename T, int FMT, int BN, bool CAUSAL>
static gpo_status run_attn_tc_d(const gpo_key& k, const Plan& p, const gpo_args& a,
                                const LaunchCtx& c, CUtensorMapDataType dt) {
  switch (k.shape[2]) {
    case 32: return run_attn_tc<T, FMT, BN, 32, CAUSAL>(k, p, a, c, dt);
    case 64: return run_attn_tc<T, FMT, BN, 64, CAUSAL>(k, p, a, c, dt);
    case 128: return run_attn_tc<T, FMT, BN, 128, CAUSAL>(k, p, a, c, dt);
    case 256: return run_attn_tc<T, FMT, BN, 256, CAUSAL>(k, p, a, c, dt);
    default: return GPO_INTERNAL;
  }
}

template <typename T, int FMT, bool CAUSAL>
static gpo_status run_attn_tc_bn(const gpo_key& k, const Plan& p, const gpo_args& a,
                                 const LaunchCtx& c, CUtensorMapDataType dt) {
  switch (k.block_n) {
    case 32: return run_attn_tc_d<T, FMT, 32, CAUSAL>(k, p, a, c, dt);
    case 64: return run_attn_tc_d<T, FMT, 64, CAUSAL>(k, p, a, c, dt);
    case 128: return run_attn_tc_d<T, FMT, 128, CAUSAL>(k, p, a, c, dt);
    default: return GPO_INTERNAL;
  }
}

gpo_status launch_attention_tc(const gpo_key& k, const Plan& p, const gpo_args& a,
                               const LaunchCtx& c) {
  if (!a.in[0] || !a.in[1] || !a.in[2] || !a.out) return GPO_BAD_ARGS;
  if (!aligned16(a.in[0]) || !aligned16(a.in[1]) || !aligned16(a.in[2]) || !aligned16(a.out))
    return GPO_BAD_ARGS;
  if (k.shape[0] == 0 || k.shape[1] == 0) return GPO_OK;
  const bool causal = k.task == GPO_TASK_ATTENTION_CAUSAL;
  if (k.dtype == GPO_BFLOAT16)
    return causal ? run_attn_tc_bn<__nv_bfloat16, 1, true>(k, p, a, c,
                                                           CU_TENSOR_MAP_DATA_TYPE_BFLOAT16)
                  : run_attn_tc_bn<__nv_bfloat16, 1, false>(k, p, a, c,
                                                            CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
  if (k.dtype == GPO_FLOAT16)
    return causal ? run_attn_tc_bn<__half, 0, true>(k, p, a, c, CU_TENSOR_MAP_DATA_TYPE_FLOAT16)
                  : run_attn_tc_bn<__half, 0, false>(k, p, a, c, CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  return GPO_BAD_ARGS;
}

}  // namespace gpo

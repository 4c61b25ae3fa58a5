// CUDA-core matmul family and the matmul dispatcher.
//
// Serves the candidates the tensor-core family does not: dtype float32
// (IEEE fp32, ALLOW_TF32 off as in compiler/triton/runner.py:100) and tile
// shapes below tcgen05's minimum M (BLOCK_M 16 / 32 / 64) or N (16), plus
// shapes whose row pitch TMA cannot describe.  Each thread owns a TM x TN
// register micro-tile; A and B tiles pass through shared memory in K chunks
// of 32 (fp32), double-buffered.  The per-thread accumulator count BLOCK_M*BLOCK_N/threads is
// the register tile; above 128 fp32 values it cannot be held without
// spilling the whole accumulator, which this family reports as a compile
// error (the resource Triton would exhaust for the same config).
#include <algorithm>
#include <type_traits>

#include "gpo_common.cuh"
#include "gpo_internal.h"

namespace gpo {

constexpr int kSimtKC = 32;
constexpr int kSimtStage = 16;  // staged elements per thread per operand (register prefetch)

__device__ __forceinline__ float tf32_truncate(float x) {
  return __uint_as_float(__float_as_uint(x) & ~0x1FFFu);
}

// Two shared-memory stages: while the threads multiply K chunk k out of one
// stage, the next chunk's global loads are already in registers and land in
// the other stage after the chunk (one barrier per chunk).  A is read along
// its rows (coalesced) and staged transposed ([k][m], rows padded by 4
// floats against bank conflicts) so that a thread's TM operands are
// contiguous 16-byte vectors; B is staged as is ([k][n]) and a thread's TN
// columns are TN/4 strips of 4 spaced BN/(TN/4) apart, so that a warp's
// 16-byte reads are consecutive.  The outer product runs as packed fp32x2
// FMAs.  Configs whose tile needs more than kSimtStage staged elements per
// thread skip the prefetch (load, barrier, compute).
template <typename T, int TM, int TN>
__global__ void __launch_bounds__(256) matmul_simt_kernel(const T* __restrict__ A,
                                                          const T* __restrict__ B,
                                                          T* __restrict__ C, int M, int N, int K,
                                                          int BM, int BN, int group_m,
                                                          int tf32) {
  using E = Elem<T>;
  constexpr int KC = kSimtKC;
  extern __shared__ __align__(16) float sm[];
  const int LDA = BM + 4;  // padded row of the transposed A stage
  const int stage_floats = KC * (LDA + BN);
  // this thread's j-th column within the tile
  auto col_of = [&](int j, int tx) -> int {
    if constexpr (TN % 4 == 0)
      return (j / 4) * (BN / (TN / 4)) + tx * 4 + (j % 4);
    else
      return tx * TN + j;
  };
  const int num_pid_m = (M + BM - 1) / BM;
  const int num_pid_n = (N + BN - 1) / BN;
  // grouped raster, as kernels.py:38-46
  const int pid = blockIdx.x;
  const int in_group = group_m * num_pid_n;
  const int gid = pid / in_group;
  const int first_m = gid * group_m;
  const int gsize = min(num_pid_m - first_m, group_m);
  const int pm = first_m + (pid % gsize);
  const int pn = (pid % in_group) / gsize;
  const int row0 = pm * BM, col0 = pn * BN;

  const int threads = blockDim.x;
  const int tx_n = BN / TN;  // threads along N
  const int ty = threadIdx.x / tx_n, tx = threadIdx.x % tx_n;
  const int la = (BM * KC + threads - 1) / threads;  // A elements per thread per chunk
  const int lb = (BN * KC + threads - 1) / threads;
  const bool staged = la <= kSimtStage && lb <= kSimtStage;

  constexpr int TP = TN >= 2 ? TN / 2 : 1;  // fp32 pairs per row (TN = 1: one lane used)
  float2 acc[TM][TP];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TP; ++j) acc[i][j] = make_float2(0.f, 0.f);

  // element e of the A chunk: row e / KC, k e % KC (coalesced along K); of
  // the B chunk: k e / BN, col e % BN (coalesced along N)
  auto a_val = [&](int e, int k0) -> float {
    const int mm = e / KC, kk = e % KC;
    const int r = row0 + mm, kc = k0 + kk;
    float v = (r < M && kc < K) ? E::to_f(A[static_cast<int64_t>(r) * K + kc]) : 0.f;
    return tf32 ? tf32_truncate(v) : v;
  };
  auto b_val = [&](int e, int k0) -> float {
    const int kk = e / BN, nn = e % BN;
    const int cidx = col0 + nn, kc = k0 + kk;
    float v = (cidx < N && kc < K) ? E::to_f(B[static_cast<int64_t>(kc) * N + cidx]) : 0.f;
    return tf32 ? tf32_truncate(v) : v;
  };
  auto compute = [&](const float* As, const float* Bs) {
#pragma unroll
    for (int kk = 0; kk < KC; ++kk) {
      float a[TM], b[TN];
      const float* ap = As + kk * LDA + ty * TM;
      const float* bp = Bs + kk * BN;
      if constexpr (TM % 4 == 0) {
#pragma unroll
        for (int i = 0; i < TM; i += 4) {
          const float4 v = *reinterpret_cast<const float4*>(ap + i);
          a[i] = v.x; a[i + 1] = v.y; a[i + 2] = v.z; a[i + 3] = v.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < TM; ++i) a[i] = ap[i];
      }
      if constexpr (TN % 4 == 0) {
#pragma unroll
        for (int j = 0; j < TN; j += 4) {
          const float4 v = *reinterpret_cast<const float4*>(bp + col_of(j, tx));
          b[j] = v.x; b[j + 1] = v.y; b[j + 2] = v.z; b[j + 3] = v.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < TN; ++j) b[j] = bp[col_of(j, tx)];
      }
#pragma unroll
      for (int i = 0; i < TM; ++i) {
        if constexpr (TN >= 2) {
          const float2 ai = make_float2(a[i], a[i]);
#pragma unroll
          for (int j = 0; j < TP; ++j)
            acc[i][j] = __ffma2_rn(ai, make_float2(b[2 * j], b[2 * j + 1]), acc[i][j]);
        } else {
          acc[i][0].x = fmaf(a[i], b[0], acc[i][0].x);
        }
      }
    }
  };

  if (staged) {
    float ra[kSimtStage], rb[kSimtStage];
    auto gload = [&](int k0) {
#pragma unroll
      for (int i = 0; i < kSimtStage; ++i) {
        const int e = threadIdx.x + i * threads;
        if (i < la && e < BM * KC) ra[i] = a_val(e, k0);
        if (i < lb && e < BN * KC) rb[i] = b_val(e, k0);
      }
    };
    auto sstore = [&](float* As, float* Bs) {
#pragma unroll
      for (int i = 0; i < kSimtStage; ++i) {
        const int e = threadIdx.x + i * threads;
        if (i < la && e < BM * KC) As[(e % KC) * LDA + e / KC] = ra[i];
        if (i < lb && e < BN * KC) Bs[e] = rb[i];
      }
    };
    gload(0);
    sstore(sm, sm + KC * LDA);
    __syncthreads();
    int cur = 0;
    for (int k0 = 0; k0 < K; k0 += KC) {
      const bool more = k0 + KC < K;
      if (more) gload(k0 + KC);
      float* Ac = sm + cur * stage_floats;
      compute(Ac, Ac + KC * LDA);
      if (more) {
        float* An = sm + (cur ^ 1) * stage_floats;
        sstore(An, An + KC * LDA);
      }
      __syncthreads();
      cur ^= 1;
    }
  } else {
    for (int k0 = 0; k0 < K; k0 += KC) {
      for (int e = threadIdx.x; e < KC * BM; e += threads) sm[(e % KC) * LDA + e / KC] = a_val(e, k0);
      for (int e = threadIdx.x; e < KC * BN; e += threads) sm[KC * LDA + e] = b_val(e, k0);
      __syncthreads();
      compute(sm, sm + KC * LDA);
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int r = row0 + ty * TM + i;
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < TP; ++j) {
      const int cidx = col0 + col_of(2 * j, tx);  // pairs never straddle a strip
      if (cidx < N) C[static_cast<int64_t>(r) * N + cidx] = E::from_f(acc[i][j].x);
      if (TN >= 2 && cidx + 1 < N)
        C[static_cast<int64_t>(r) * N + cidx + 1] = E::from_f(acc[i][j].y);
    }
  }
}

// ----------------------------------------------- fp32, cp.async pipeline
// IEEE fp32 with K and N multiples of 4 and 16-byte aligned operands: the
// chunks go global -> shared memory with cp.async (16-byte pieces, zero
// fill past M, N and K), three stages deep, so the loads of chunk k+2 are in
// flight while chunk k is multiplied and no register holds them.  A is
// staged row-major (rows padded to KC+4 floats) and read as scalars — the
// threads of a warp share at most two rows, so the reads broadcast — and B
// as in matmul_simt_kernel.
constexpr int kSimtAsyncStages = 3;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int TM, int TN>
__global__ void __launch_bounds__(256) matmul_simt_async_kernel(const float* __restrict__ A,
                                                                const float* __restrict__ B,
                                                                float* __restrict__ C, int M,
                                                                int N, int K, int BM, int BN,
                                                                int group_m) {
  constexpr int KC = kSimtKC;
  constexpr int S = kSimtAsyncStages;
  constexpr int LDK = KC + 4;
  constexpr int TP = TN >= 2 ? TN / 2 : 1;
  extern __shared__ __align__(16) float sm[];
  const int stage = BM * LDK + KC * BN;
  const int num_pid_m = (M + BM - 1) / BM;
  const int num_pid_n = (N + BN - 1) / BN;
  const int pid = blockIdx.x;  // grouped raster, as kernels.py:38-46
  const int in_group = group_m * num_pid_n;
  const int gid = pid / in_group;
  const int first_m = gid * group_m;
  const int gsize = min(num_pid_m - first_m, group_m);
  const int pm = first_m + (pid % gsize);
  const int pn = (pid % in_group) / gsize;
  const int row0 = pm * BM, col0 = pn * BN;
  const int threads = blockDim.x;
  const int tx_n = BN / TN;
  const int ty = threadIdx.x / tx_n, tx = threadIdx.x % tx_n;
  auto col_of = [&](int j) -> int {
    if constexpr (TN % 4 == 0)
      return (j / 4) * (BN / (TN / 4)) + tx * 4 + (j % 4);
    else
      return tx * TN + j;
  };

  auto issue = [&](int chunk, int slot) {
    const int k0 = chunk * KC;
    float* As = sm + slot * stage;
    float* Bs = As + BM * LDK;
    for (int e = threadIdx.x; e < BM * (KC / 4); e += threads) {
      const int mm = e / (KC / 4), kq = e % (KC / 4);
      const int r = row0 + mm, kc = k0 + kq * 4;
      const bool in = r < M && kc < K;  // K % 4 == 0: a piece is wholly in or out
      cp_async16(smem_u32(As + mm * LDK + kq * 4),
                 in ? static_cast<const void*>(A + static_cast<int64_t>(r) * K + kc) : A,
                 in ? 16 : 0);
    }
    for (int e = threadIdx.x; e < KC * (BN / 4); e += threads) {
      const int kk = e / (BN / 4), nq = e % (BN / 4);
      const int kc = k0 + kk, cidx = col0 + nq * 4;
      const bool in = kc < K && cidx < N;  // N % 4 == 0
      cp_async16(smem_u32(Bs + kk * BN + nq * 4),
                 in ? static_cast<const void*>(B + static_cast<int64_t>(kc) * N + cidx) : B,
                 in ? 16 : 0);
    }
    cp_async_commit();
  };

  float2 acc[TM][TP];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TP; ++j) acc[i][j] = make_float2(0.f, 0.f);

  const int nch = (K + KC - 1) / KC;
#pragma unroll
  for (int c = 0; c < S - 1; ++c) {
    if (c < nch)
      issue(c, c);
    else
      cp_async_commit();
  }
  for (int ch = 0; ch < nch; ++ch) {
    cp_async_wait<S - 2>();  // this thread's pieces of chunk ch landed
    __syncthreads();         // everyone's; and slot (ch - 1) % S is no longer read
    if (ch + S - 1 < nch)
      issue(ch + S - 1, (ch + S - 1) % S);
    else
      cp_async_commit();
    const float* As = sm + (ch % S) * stage;
    const float* Bs = As + BM * LDK;
    // A rows hold K contiguously (LDK = KC + 4 floats, 16-byte aligned):
    // one 16-byte load gives a thread four K steps of one of its rows
#pragma unroll 2
    for (int k4 = 0; k4 < KC; k4 += 4) {
      float4 a4[TM];
#pragma unroll
      for (int i = 0; i < TM; ++i)
        a4[i] = *reinterpret_cast<const float4*>(As + (ty * TM + i) * LDK + k4);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int kk = k4 + u;
        float b[TN];
        if constexpr (TN % 4 == 0) {
#pragma unroll
          for (int j = 0; j < TN; j += 4) {
            const float4 v = *reinterpret_cast<const float4*>(Bs + kk * BN + col_of(j));
            b[j] = v.x; b[j + 1] = v.y; b[j + 2] = v.z; b[j + 3] = v.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < TN; ++j) b[j] = Bs[kk * BN + col_of(j)];
        }
#pragma unroll
        for (int i = 0; i < TM; ++i) {
          const float ai = u == 0 ? a4[i].x : u == 1 ? a4[i].y : u == 2 ? a4[i].z : a4[i].w;
          if constexpr (TN >= 2) {
            const float2 ai2 = make_float2(ai, ai);
#pragma unroll
            for (int j = 0; j < TP; ++j)
              acc[i][j] = __ffma2_rn(ai2, make_float2(b[2 * j], b[2 * j + 1]), acc[i][j]);
          } else {
            acc[i][0].x = fmaf(ai, b[0], acc[i][0].x);
          }
        }
      }
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int r = row0 + ty * TM + i;
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < TP; ++j) {
      const int cidx = col0 + col_of(2 * j);
      if (cidx < N) C[static_cast<int64_t>(r) * N + cidx] = acc[i][j].x;
      if (TN >= 2 && cidx + 1 < N) C[static_cast<int64_t>(r) * N + cidx + 1] = acc[i][j].y;
    }
  }
}

// (TM, TN) per accumulator count.
static bool simt_micro(int acc, int& tm, int& tn) {
  switch (acc) {
    case 1: tm = 1; tn = 1; return true;
    case 2: tm = 1; tn = 2; return true;
    case 4: tm = 2; tn = 2; return true;
    case 8: tm = 2; tn = 4; return true;
    case 16: tm = 4; tn = 4; return true;
    case 32: tm = 4; tn = 8; return true;
    case 64: tm = 8; tn = 8; return true;
    case 128: tm = 8; tn = 16; return true;
    default: return false;
  }
}

static bool pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }

// Plan: aux[0] = per-thread accumulators, aux[1] = dynamic smem.
gpo_status plan_matmul_simt(const gpo_key& k, Plan& p, std::string& log) {
  const int BM = k.block_m, BN = k.block_n;
  if (!pow2(BM) || !pow2(BN) || BM < 16 || BN < 16 || BM > 256 || BN > 256) {
    log = "BLOCK_M / BLOCK_N must be powers of two in [16, 256]";
    return GPO_BAD_CONFIG;
  }
  if (!pow2(k.block_k) || k.block_k > 256) {
    log = "BLOCK_K must be a power of two <= 256";
    return GPO_BAD_CONFIG;
  }
  if (k.num_warps < 1 || k.num_warps > 8 || !pow2(k.num_warps)) {
    log = "num_warps must be 1, 2, 4 or 8";
    return GPO_BAD_CONFIG;
  }
  if (k.group_m < 1) {
    log = "GROUP_M must be >= 1";
    return GPO_BAD_CONFIG;
  }
  const int threads = k.num_warps * 32;
  if (BM * BN < threads) {
    log = "tile has fewer outputs than threads";
    return GPO_BAD_CONFIG;
  }
  const int acc = BM * BN / threads;
  int tm, tn;
  if (!simt_micro(acc, tm, tn) || tm > BM || tn > BN) {
    log = "register tile of " + std::to_string(acc) +
          " fp32 accumulators per thread exceeds the 128-register budget";
    return GPO_COMPILE_ERROR;
  }
  const uint32_t dyn = static_cast<uint32_t>(2 * kSimtKC * (BM + 4 + BN) * 4);  // two stages
  if (dyn > kMaxSmemPerCta) {
    log = "shared memory " + std::to_string(dyn) + " B for two K stages exceeds 232448 B";
    return GPO_COMPILE_ERROR;
  }
  p.aux[0] = acc;
  p.aux[1] = static_cast<int>(dyn);
  // IEEE fp32 with K, N multiples of 4: the cp.async pipeline (chosen at
  // launch when the operands are 16-byte aligned)
  const uint32_t adyn = static_cast<uint32_t>(
      kSimtAsyncStages * (BM * (kSimtKC + 4) + kSimtKC * BN) * 4);
  const bool async_ok = k.dtype == GPO_FLOAT32 && k.shape[2] % 4 == 0 && k.shape[1] % 4 == 0 &&
                        adyn <= kMaxSmemPerCta;
  p.aux[2] = async_ok ? static_cast<int>(adyn) : 0;
  p.family = "matmul_simt";
  p.res.smem_bytes = async_ok ? adyn : dyn;
  p.res.threads_per_cta = static_cast<uint32_t>(threads);
  p.res.grid_x = static_cast<uint32_t>(cdiv(k.shape[0], BM) * cdiv(k.shape[1], BN));
  p.res.grid_y = p.res.grid_z = 1;
  p.res.launches_per_call = 1;
  snprintf(p.res.kernel, sizeof(p.res.kernel), "%s<%dx%d per thread>",
           async_ok ? "matmul_simt_async_kernel" : "matmul_simt_kernel", tm, tn);
  return GPO_OK;
}

template <typename T, int TM, int TN>
static gpo_status run_simt(const gpo_key& k, const Plan& p, const gpo_args& a,
                           const LaunchCtx& c) {
  const unsigned grid = static_cast<unsigned>(cdiv(k.shape[0], k.block_m) *
                                              cdiv(k.shape[1], k.block_n));
  if constexpr (std::is_same<T, float>::value) {
    if (p.aux[2] > 0 && aligned16(a.in[0]) && aligned16(a.in[1])) {
      auto kern = matmul_simt_async_kernel<TM, TN>;
      gpo_status st = ensure_smem_attr(reinterpret_cast<const void*>(kern),
                                       static_cast<uint32_t>(p.aux[2]));
      if (st != GPO_OK) return st;
      kern<<<grid, k.num_warps * 32, p.aux[2], c.stream>>>(
          static_cast<const float*>(a.in[0]), static_cast<const float*>(a.in[1]),
          static_cast<float*>(a.out), static_cast<int>(k.shape[0]), static_cast<int>(k.shape[1]),
          static_cast<int>(k.shape[2]), k.block_m, k.block_n, k.group_m);
      return launch_status();
    }
  }
  gpo_status st = ensure_smem_attr(reinterpret_cast<const void*>(&matmul_simt_kernel<T, TM, TN>),
                                   static_cast<uint32_t>(p.aux[1]));
  if (st != GPO_OK) return st;
  matmul_simt_kernel<T, TM, TN><<<grid, k.num_warps * 32, p.aux[1], c.stream>>>(
      static_cast<const T*>(a.in[0]), static_cast<const T*>(a.in[1]), static_cast<T*>(a.out),
      static_cast<int>(k.shape[0]), static_cast<int>(k.shape[1]), static_cast<int>(k.shape[2]),
      k.block_m, k.block_n, k.group_m, k.dtype == GPO_TF32 ? 1 : 0);
  return launch_status();
}

template <typename T>
static gpo_status run_simt_dt(const gpo_key& k, const Plan& p, const gpo_args& a,
                              const LaunchCtx& c) {
  switch (p.aux[0]) {
    case 1: return run_simt<T, 1, 1>(k, p, a, c);
    case 2: return run_simt<T, 1, 2>(k, p, a, c);
    case 4: return run_simt<T, 2, 2>(k, p, a, c);
    case 8: return run_simt<T, 2, 4>(k, p, a, c);
    case 16: return run_simt<T, 4, 4>(k, p, a, c);
    case 32: return run_simt<T, 4, 8>(k, p, a, c);
    case 64: return run_simt<T, 8, 8>(k, p, a, c);
    case 128: return run_simt<T, 8, 16>(k, p, a, c);
    default: return GPO_INTERNAL;
  }
}

gpo_status launch_matmul_simt(const gpo_key& k, const Plan& p, const gpo_args& a,
                              const LaunchCtx& c) {
  if (!a.in[0] || !a.in[1] || !a.out) return GPO_BAD_ARGS;
  if (k.shape[0] == 0 || k.shape[1] == 0) return GPO_OK;
  switch (k.dtype) {
    case GPO_FLOAT32:
    case GPO_TF32: return run_simt_dt<float>(k, p, a, c);
    case GPO_FLOAT16: return run_simt_dt<__half>(k, p, a, c);
    case GPO_BFLOAT16: return run_simt_dt<__nv_bfloat16>(k, p, a, c);
    default: return GPO_BAD_ARGS;
  }
}

// ------------------------------------------------------------- dispatcher
// Tensor cores for 16-bit / tf32 with BLOCK_M in {64, 128, 256} and
// BLOCK_N in {32..256} when TMA can describe the operands; CUDA cores
// otherwise.
// aux[7] records the choice (1 = tcgen05).
gpo_status plan_matmul(const gpo_key& k, Plan& p, std::string& log) {
  if (k.ndim != 3 || k.shape[0] < 0 || k.shape[1] < 0 || k.shape[2] < 0) {
    log = "expected shape (M, N, K)";
    return GPO_BAD_CONFIG;
  }
  const int es = dtype_bytes(k.dtype);
  const bool tc_dtype = k.dtype != GPO_FLOAT32;
  const bool tc_tile =
      (k.block_m == 32 || k.block_m == 64 || k.block_m == 128 || k.block_m == 256) &&
      k.block_n >= 32 && k.block_k * es >= 32 && (k.num_warps == 4 || k.num_warps == 8);
  const bool tc_shape = (k.shape[2] * es) % 16 == 0 && (k.shape[1] * es) % 16 == 0;
  if (tc_dtype && tc_tile && tc_shape) {
    gpo_status s = plan_matmul_tc(k, p, log);
    // BLOCK_M 32 stages A in 64-row atoms on the tensor cores; where that
    // does not fit, the CUDA-core tile (32-row A) still may
    if (!(k.block_m == 32 && s == GPO_COMPILE_ERROR)) {
      p.aux[7] = 1;
      return s;
    }
    p = Plan{};
    log.clear();
  }
  p.aux[7] = 0;
  return plan_matmul_simt(k, p, log);
}

gpo_status launch_matmul(const gpo_key& k, const Plan& p, const gpo_args& a, const LaunchCtx& c) {
  if (!a.out) return GPO_BAD_ARGS;
  if (k.shape[2] == 0 && k.shape[0] > 0 && k.shape[1] > 0) {
    // empty contraction: C = 0
    const size_t bytes = static_cast<size_t>(k.shape[0]) * k.shape[1] * dtype_bytes(k.dtype);
    return cudaMemsetAsync(a.out, 0, bytes, c.stream) == cudaSuccess ? GPO_OK : GPO_LAUNCH_ERROR;
  }
  return p.aux[7] ? launch_matmul_tc(k, p, a, c) : launch_matmul_simt(k, p, a, c);
}

}  // namespace gpo

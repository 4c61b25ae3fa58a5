// CUDA-core matmul family and the matmul dispatcher.
//
// Serves the candidates the tensor-core family does not: dtype float32
// (IEEE fp32, ALLOW_TF32 off as in compiler/triton/runner.py:100) and tile
// shapes below tcgen05's minimum M (BLOCK_M 16 / 32 / 64) or N (16), plus
// shapes whose row pitch TMA cannot describe.  Each thread owns a TM x TN
// register micro-tile; A and B tiles pass through shared memory in K chunks
// of 16 (fp32).  The per-thread accumulator count BLOCK_M*BLOCK_N/threads is
// the register tile; above 128 fp32 values it cannot be held without
// spilling the whole accumulator, which this family reports as a compile
// error (the resource Triton would exhaust for the same config).
#include <algorithm>

#include "gpo_common.cuh"
#include "gpo_internal.h"

namespace gpo {

constexpr int kSimtKC = 16;

__device__ __forceinline__ float tf32_truncate(float x) {
  return __uint_as_float(__float_as_uint(x) & ~0x1FFFu);
}

template <typename T, int TM, int TN>
__global__ void __launch_bounds__(256) matmul_simt_kernel(const T* __restrict__ A,
                                                          const T* __restrict__ B,
                                                          T* __restrict__ C, int M, int N, int K,
                                                          int BM, int BN, int group_m,
                                                          int tf32) {
  using E = Elem<T>;
  extern __shared__ float sm[];
  float* As = sm;                 // [KC][BM]
  float* Bs = sm + kSimtKC * BM;  // [KC][BN]
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

  const int tx_n = BN / TN;  // threads along N
  const int ty = threadIdx.x / tx_n, tx = threadIdx.x % tx_n;
  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < K; k0 += kSimtKC) {
    for (int e = threadIdx.x; e < kSimtKC * BM; e += blockDim.x) {
      const int kk = e / BM, mm = e % BM;
      const int r = row0 + mm, kc = k0 + kk;
      float v = (r < M && kc < K) ? E::to_f(A[static_cast<int64_t>(r) * K + kc]) : 0.f;
      As[kk * BM + mm] = tf32 ? tf32_truncate(v) : v;
    }
    for (int e = threadIdx.x; e < kSimtKC * BN; e += blockDim.x) {
      const int kk = e / BN, nn = e % BN;
      const int cidx = col0 + nn, kc = k0 + kk;
      float v = (cidx < N && kc < K) ? E::to_f(B[static_cast<int64_t>(kc) * N + cidx]) : 0.f;
      Bs[kk * BN + nn] = tf32 ? tf32_truncate(v) : v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kSimtKC; ++kk) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = As[kk * BM + ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; ++j) b[j] = Bs[kk * BN + tx * TN + j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int r = row0 + ty * TM + i;
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int cidx = col0 + tx * TN + j;
      if (cidx < N) C[static_cast<int64_t>(r) * N + cidx] = E::from_f(acc[i][j]);
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
  const uint32_t dyn = static_cast<uint32_t>(kSimtKC * (BM + BN) * 4);
  p.aux[0] = acc;
  p.aux[1] = static_cast<int>(dyn);
  p.family = "matmul_simt";
  p.res.smem_bytes = dyn;
  p.res.threads_per_cta = static_cast<uint32_t>(threads);
  p.res.grid_x = static_cast<uint32_t>(cdiv(k.shape[0], BM) * cdiv(k.shape[1], BN));
  p.res.grid_y = p.res.grid_z = 1;
  p.res.launches_per_call = 1;
  snprintf(p.res.kernel, sizeof(p.res.kernel), "matmul_simt_kernel<%dx%d per thread>", tm, tn);
  return GPO_OK;
}

template <typename T, int TM, int TN>
static gpo_status run_simt(const gpo_key& k, const Plan& p, const gpo_args& a,
                           const LaunchCtx& c) {
  const unsigned grid = static_cast<unsigned>(cdiv(k.shape[0], k.block_m) *
                                              cdiv(k.shape[1], k.block_n));
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
// Tensor cores for 16-bit / tf32 with BLOCK_M in {128, 256} and BLOCK_N in
// {32..256} when TMA can describe the operands; CUDA cores otherwise.
// aux[7] records the choice (1 = tcgen05).
gpo_status plan_matmul(const gpo_key& k, Plan& p, std::string& log) {
  if (k.ndim != 3 || k.shape[0] < 0 || k.shape[1] < 0 || k.shape[2] < 0) {
    log = "expected shape (M, N, K)";
    return GPO_BAD_CONFIG;
  }
  const int es = dtype_bytes(k.dtype);
  const bool tc_dtype = k.dtype != GPO_FLOAT32;
  const bool tc_tile = (k.block_m == 128 || k.block_m == 256) && k.block_n >= 32 &&
                       k.block_k * es >= 32 && (k.num_warps == 4 || k.num_warps == 8);
  const bool tc_shape = (k.shape[2] * es) % 16 == 0 && (k.shape[1] * es) % 16 == 0;
  if (tc_dtype && tc_tile && tc_shape) {
    gpo_status s = plan_matmul_tc(k, p, log);
    p.aux[7] = 1;
    return s;
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

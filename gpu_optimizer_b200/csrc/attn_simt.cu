// CUDA-core flash-attention forward family and the attention dispatcher.
//
// Serves candidates the tensor-core family does not: dtype float32 (IEEE
// fp32; the reference keeps ALLOW_TF32 off for attention,
// compiler/triton/runner.py:237) and tiles other than BLOCK_M 64 / 128 /
// 256 (BLOCK_M 16 or 32, BLOCK_N 16, head dims below 32, 2 warps).
// Algorithm per (query tile, batch*head), as attention_kernel
// (compiler/triton/kernels.py:212-270): stream K/V tiles of BLOCK_N keys,
// online softmax with fp32 running max / sum, P cast to V's dtype before the
// PV product (kernels.py:264), O divided by the running sum at the end.
// Q, K, V, S and O tiles live in shared memory as fp32; a config whose tiles
// exceed 227 KB is a compile error of this family.
#include <algorithm>

#include "gpo_common.cuh"
#include "gpo_internal.h"

namespace gpo {

template <typename T, int D, bool CAUSAL>
__global__ void __launch_bounds__(512) attn_simt_kernel(const T* __restrict__ q,
                                                        const T* __restrict__ k,
                                                        const T* __restrict__ v,
                                                        T* __restrict__ o, int S, int BM, int BN,
                                                        float sm_scale) {
  using E = Elem<T>;
  extern __shared__ float sm[];
  float* Qs = sm;                 // [BM][D]
  float* Ks = Qs + BM * D;        // [BN][D+1]
  float* Vs = Ks + BN * (D + 1);  // [BN][D]
  float* Ss = Vs + BN * D;        // [BM][BN]
  float* Os = Ss + BM * BN;       // [BM][D]
  float* mrow = Os + BM * D;      // [BM]
  float* lrow = mrow + BM;        // [BM]
  float* arow = lrow + BM;        // [BM] rescale factor of the current block

  const int bh = blockIdx.y;
  const int q0 = blockIdx.x * BM;
  const int64_t head = static_cast<int64_t>(bh) * S * D;
  const int T_ = blockDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = T_ >> 5;

  for (int e = threadIdx.x; e < BM * D; e += T_) {
    const int r = e / D, d = e % D;
    Qs[e] = (q0 + r < S) ? E::to_f(q[head + static_cast<int64_t>(q0 + r) * D + d]) : 0.f;
    Os[e] = 0.f;
  }
  for (int r = threadIdx.x; r < BM; r += T_) {
    mrow[r] = -INFINITY;
    lrow[r] = 0.f;
  }
  const int kend = CAUSAL ? min(S, q0 + BM) : S;
  for (int n0 = 0; n0 < kend; n0 += BN) {
    __syncthreads();
    for (int e = threadIdx.x; e < BN * D; e += T_) {
      const int n = e / D, d = e % D;
      const bool ok = n0 + n < S;
      const int64_t g = head + static_cast<int64_t>(n0 + n) * D + d;
      Ks[n * (D + 1) + d] = ok ? E::to_f(k[g]) : 0.f;
      Vs[n * D + d] = ok ? E::to_f(v[g]) : 0.f;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < BM * BN; e += T_) {
      const int r = e / BN, n = e % BN;
      const int key = n0 + n;
      float acc = 0.f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) acc = fmaf(Qs[r * D + d], Ks[n * (D + 1) + d], acc);
      const bool masked = key >= S || (CAUSAL && key > q0 + r);
      Ss[e] = masked ? -INFINITY : acc * sm_scale;
    }
    __syncthreads();
    // one warp per row: online max / sum, P cast to V's dtype
    for (int r = warp; r < BM; r += nw) {
      float mx = -INFINITY;
      for (int n = lane; n < BN; n += 32) mx = fmaxf(mx, Ss[r * BN + n]);
      mx = warp_max(mx);
      const float m_old = mrow[r];
      const float m_new = fmaxf(m_old, mx);
      const bool live = m_new != -INFINITY;
      const float alpha = live ? expf(m_old - m_new) : 1.f;
      float sum = 0.f;
      for (int n = lane; n < BN; n += 32) {
        const float p = live ? expf(Ss[r * BN + n] - m_new) : 0.f;
        sum += p;
        Ss[r * BN + n] = E::to_f(E::from_f(p));
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        lrow[r] = lrow[r] * alpha + sum;
        mrow[r] = m_new;
        arow[r] = alpha;
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < BM * D; e += T_) {
      const int r = e / D, d = e % D;
      float acc = Os[e] * arow[r];
      for (int n = 0; n < BN; ++n) acc = fmaf(Ss[r * BN + n], Vs[n * D + d], acc);
      Os[e] = acc;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < BM * D; e += T_) {
    const int r = e / D, d = e % D;
    if (q0 + r < S) o[head + static_cast<int64_t>(q0 + r) * D + d] = E::from_f(Os[e] / lrow[r]);
  }
}

static bool pow2i(int v) { return v > 0 && (v & (v - 1)) == 0; }

static uint32_t simt_smem(int BM, int BN, int D) {
  return static_cast<uint32_t>(4 * (BM * D + BN * (D + 1) + BN * D + BM * BN + BM * D + 3 * BM));
}

gpo_status plan_attention_simt(const gpo_key& k, Plan& p, std::string& log) {
  const int D = static_cast<int>(k.shape[2]);
  const int BM = k.block_m, BN = k.block_n;
  if (!pow2i(BM) || !pow2i(BN) || BM < 16 || BN < 16 || BM > 256 || BN > 256) {
    log = "BLOCK_M / BLOCK_N must be powers of two in [16, 256]";
    return GPO_BAD_CONFIG;
  }
  if (k.num_warps < 1 || k.num_warps > 16 || !pow2i(k.num_warps)) {
    log = "num_warps must be a power of two in [1, 16]";
    return GPO_BAD_CONFIG;
  }
  if (D != 16 && D != 32 && D != 64 && D != 128 && D != 256) {
    log = "head dim must be 16, 32, 64, 128 or 256";
    return GPO_BAD_CONFIG;
  }
  const uint32_t dyn = simt_smem(BM, BN, D);
  if (dyn > kMaxSmemPerCta) {
    log = "fp32 Q/K/V/S/O tiles need " + std::to_string(dyn) + " B > 232448 B shared memory";
    return GPO_COMPILE_ERROR;
  }
  p.aux[0] = static_cast<int>(dyn);
  p.family = "attn_simt";
  p.res.smem_bytes = dyn;
  p.res.threads_per_cta = static_cast<uint32_t>(k.num_warps * 32);
  p.res.grid_x = static_cast<uint32_t>(cdiv(k.shape[1], BM));
  p.res.grid_y = static_cast<uint32_t>(k.shape[0]);
  p.res.grid_z = 1;
  p.res.launches_per_call = 1;
  snprintf(p.res.kernel, sizeof(p.res.kernel), "attn_simt_kernel<D=%d,%s>", D,
           k.task == GPO_TASK_ATTENTION_CAUSAL ? "causal" : "full");
  return GPO_OK;
}

template <typename T, int D, bool CAUSAL>
static gpo_status run_attn_simt(const gpo_key& k, const Plan& p, const gpo_args& a,
                                const LaunchCtx& c) {
  auto kern = attn_simt_kernel<T, D, CAUSAL>;
  const uint32_t dyn = static_cast<uint32_t>(p.aux[0]);
  gpo_status s = ensure_smem_attr(reinterpret_cast<const void*>(kern), dyn);
  if (s != GPO_OK) return s;
  const dim3 grid(static_cast<unsigned>(cdiv(k.shape[1], k.block_m)),
                  static_cast<unsigned>(k.shape[0]));
  kern<<<grid, k.num_warps * 32, dyn, c.stream>>>(
      static_cast<const T*>(a.in[0]), static_cast<const T*>(a.in[1]),
      static_cast<const T*>(a.in[2]), static_cast<T*>(a.out), static_cast<int>(k.shape[1]),
      k.block_m, k.block_n, 1.0f / sqrtf(static_cast<float>(D)));
  return launch_status();
}

template <typename T, bool CAUSAL>
static gpo_status run_attn_simt_d(const gpo_key& k, const Plan& p, const gpo_args& a,
                                  const LaunchCtx& c) {
  switch (k.shape[2]) {
    case 16: return run_attn_simt<T, 16, CAUSAL>(k, p, a, c);
    case 32: return run_attn_simt<T, 32, CAUSAL>(k, p, a, c);
    case 64: return run_attn_simt<T, 64, CAUSAL>(k, p, a, c);
    case 128: return run_attn_simt<T, 128, CAUSAL>(k, p, a, c);
    case 256: return run_attn_simt<T, 256, CAUSAL>(k, p, a, c);
    default: return GPO_INTERNAL;
  }
}

template <typename T>
static gpo_status run_attn_simt_c(const gpo_key& k, const Plan& p, const gpo_args& a,
                                  const LaunchCtx& c) {
  return k.task == GPO_TASK_ATTENTION_CAUSAL ? run_attn_simt_d<T, true>(k, p, a, c)
                                             : run_attn_simt_d<T, false>(k, p, a, c);
}

gpo_status launch_attention_simt(const gpo_key& k, const Plan& p, const gpo_args& a,
                                 const LaunchCtx& c) {
  if (!a.in[0] || !a.in[1] || !a.in[2] || !a.out) return GPO_BAD_ARGS;
  if (k.shape[0] == 0 || k.shape[1] == 0) return GPO_OK;
  switch (k.dtype) {
    case GPO_FLOAT32: return run_attn_simt_c<float>(k, p, a, c);
    case GPO_FLOAT16: return run_attn_simt_c<__half>(k, p, a, c);
    case GPO_BFLOAT16: return run_attn_simt_c<__nv_bfloat16>(k, p, a, c);
    default: return GPO_BAD_ARGS;
  }
}

// ------------------------------------------------------------- dispatcher
// Tensor cores for 16-bit inputs with BLOCK_M = 64 (64-row query tiles,
// M=64 MMAs), 128 (one CTA per query tile) or 256 (a CTA pair on two query
// tiles), BLOCK_N in {32, 64, 128},
// head dim in {32, 64, 128, 256} and num_warps 4 (one softmax warpgroup) or
// 8 (two); CUDA cores otherwise.  aux[7] records the choice (1 = tcgen05).
gpo_status plan_attention(const gpo_key& k, Plan& p, std::string& log) {
  if (k.ndim != 3 || k.shape[0] < 0 || k.shape[1] < 0 || k.shape[2] < 1) {
    log = "expected shape (BH, S, D)";
    return GPO_BAD_CONFIG;
  }
  const int64_t D = k.shape[2];
  if (D & (D - 1) || D < 16) {
    // same rule and message as compiler/triton/runner.py:233-234
    log = "head dim " + std::to_string(D) + " must be a power of two >= 16";
    return GPO_BAD_CONFIG;
  }
  const bool tc = (k.dtype == GPO_BFLOAT16 || k.dtype == GPO_FLOAT16) &&
                  (k.block_m == 64 || k.block_m == 128 || k.block_m == 256) &&
                  (k.block_n == 32 || k.block_n == 64 || k.block_n == 128) && D >= 32 &&
                  D <= 256 && (k.num_warps == 4 || k.num_warps == 8);
  if (tc) {
    gpo_status s = plan_attention_tc(k, p, log);
    p.aux[7] = 1;
    return s;
  }
  p.aux[7] = 0;
  return plan_attention_simt(k, p, log);
}

gpo_status launch_attention(const gpo_key& k, const Plan& p, const gpo_args& a,
                            const LaunchCtx& c) {
  return p.aux[7] ? launch_attention_tc(k, p, a, c) : launch_attention_simt(k, p, a, c);
}

}  // namespace gpo

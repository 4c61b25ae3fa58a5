// Row-wise kernel families: softmax and layernorm over the last dimension.
//
// One CTA of num_warps*32 threads per row (grid (M,), as
// compiler/triton/runner.py:175,194 launch).  BLOCK_N selects the strategy
// exactly as the reference does (runner.py:170,189):
//   BLOCK_N >= N : single tile — the row is read from HBM once, held in
//                  registers (or, when the per-thread share exceeds 64
//                  values, staged in shared memory), reduced, and written.
//   BLOCK_N <  N : online / two-pass — statistics pass over BLOCK_N tiles,
//                  then a normalise pass that re-reads the row (which on
//                  B200 mostly hits the 126 MB L2).
// With num_stages >= 2 a single-tile row kernel runs persistent, prefetching
// its next row while it reduces the current one (rows_pipe).
// Thread t owns V consecutive elements (one 16-byte vector) per vector slot
// and slots are strided by the CTA width, so every warp access is a
// contiguous 512-byte segment.  Statistics are fp32.
#include <algorithm>

#include "gpo_common.cuh"
#include "gpo_internal.h"

namespace gpo {

template <typename T>
struct RowVec {
  static constexpr int V = 16 / sizeof(T);
};

// Load vector slot j (V consecutive elements) of tile [tile0, tile0+bn)
// owned by this thread; out-of-range elements read as `fill`.
template <typename T>
__device__ __forceinline__ void row_load_slot(const T* __restrict__ row, int64_t n, int64_t tile0,
                                              int64_t bn, bool vec, float fill, int j,
                                              float* x) {
  using E = Elem<T>;
  constexpr int V = RowVec<T>::V;
  const int64_t vi = threadIdx.x + static_cast<int64_t>(j) * blockDim.x;
  const int64_t e0 = tile0 + vi * V;
  const bool in_tile = vi * V < bn;
  if (vec && in_tile && e0 + V <= n) {
    uint4 r = __ldcs(reinterpret_cast<const uint4*>(row + e0));
    const T* er = reinterpret_cast<const T*>(&r);
#pragma unroll
    for (int u = 0; u < V; ++u) x[u] = E::to_f(er[u]);
  } else {
#pragma unroll
    for (int u = 0; u < V; ++u) {
      const int64_t e = e0 + u;
      x[u] = (in_tile && vi * V + u < bn && e < n) ? E::to_f(row[e]) : fill;
    }
  }
}

// Load the VPT vector slots of tile [tile0, tile0+bn) owned by this thread.
template <typename T, int VPT>
__device__ __forceinline__ void row_load(const T* __restrict__ row, int64_t n, int64_t tile0,
                                         int64_t bn, bool vec, float fill,
                                         float (&x)[VPT * RowVec<T>::V]) {
#pragma unroll
  for (int j = 0; j < VPT; ++j) row_load_slot<T>(row, n, tile0, bn, vec, fill, j, x + j * RowVec<T>::V);
}

// y = (x - mean) * rstd * w + b over this thread's slots of one tile.
template <typename T, int VPT>
__device__ __forceinline__ void ln_affine(const T* __restrict__ w, const T* __restrict__ b,
                                          int64_t n, int64_t tile0, int64_t bn, bool vec,
                                          float mean, float rstd,
                                          float (&v)[VPT * RowVec<T>::V]) {
  constexpr int V = RowVec<T>::V;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    float wv[V], bv[V];
    row_load_slot<T>(w, n, tile0, bn, vec, 0.f, j, wv);
    row_load_slot<T>(b, n, tile0, bn, vec, 0.f, j, bv);
#pragma unroll
    for (int u = 0; u < V; ++u) v[j * V + u] = (v[j * V + u] - mean) * rstd * wv[u] + bv[u];
  }
}

template <typename T, int VPT>
__device__ __forceinline__ void row_store(T* __restrict__ row, int64_t n, int64_t tile0,
                                          int64_t bn, bool vec,
                                          const float (&y)[VPT * RowVec<T>::V]) {
  using E = Elem<T>;
  constexpr int V = RowVec<T>::V;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t vi = threadIdx.x + static_cast<int64_t>(j) * blockDim.x;
    const int64_t e0 = tile0 + vi * V;
    const bool in_tile = vi * V < bn;
    if (vec && in_tile && e0 + V <= n) {
      uint4 r;
      T* er = reinterpret_cast<T*>(&r);
#pragma unroll
      for (int u = 0; u < V; ++u) er[u] = E::from_f(y[j * V + u]);
      __stcs(reinterpret_cast<uint4*>(row + e0), r);
    } else {
#pragma unroll
      for (int u = 0; u < V; ++u) {
        const int64_t e = e0 + u;
        if (in_tile && vi * V + u < bn && e < n) row[e] = E::from_f(y[j * V + u]);
      }
    }
  }
}

// exp(x - m) as 2^((x - m) * log2 e): one FFMA + one MUFU ex2 per element
// (x = -inf gives 0).  neg_m_log2e = -m * log2(e).
__device__ __forceinline__ float exp_shifted(float x, float neg_m_log2e) {
  return ex2_approx(fmaf(x, 1.4426950408889634f, neg_m_log2e));
}

// Max / sum of a register array with 8 independent accumulators.
template <int N>
__device__ __forceinline__ float tree_max(const float (&v)[N]) {
  float a[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) a[t] = t < N ? v[t] : -INFINITY;
#pragma unroll
  for (int i = 8; i < N; ++i) a[i & 7] = fmaxf(a[i & 7], v[i]);
  return fmaxf(fmaxf(fmaxf(a[0], a[1]), fmaxf(a[2], a[3])),
               fmaxf(fmaxf(a[4], a[5]), fmaxf(a[6], a[7])));
}
template <int N>
__device__ __forceinline__ float tree_sum(const float (&v)[N]) {
  float a[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) a[t] = t < N ? v[t] : 0.f;
#pragma unroll
  for (int i = 8; i < N; ++i) a[i & 7] += v[i];
  return ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
}

// Block reductions; every thread receives the result.
__device__ __forceinline__ float block_allreduce_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = l < nw ? red[l] : -INFINITY;
  return warp_max(r);
}
__device__ __forceinline__ float block_allreduce_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = l < nw ? red[l] : 0.f;
  return warp_sum(r);
}

// ---------------------------------------------------------------- softmax
// Single tile held in registers (softmax_kernel SINGLE_TILE branch,
// compiler/triton/kernels.py:113-120).
template <typename T, int VPT>
__global__ void __launch_bounds__(1024) softmax_tile_regs(const T* __restrict__ x,
                                                          T* __restrict__ y, int64_t n,
                                                          int64_t bn, int vec) {
  constexpr int V = RowVec<T>::V;
  __shared__ float red[32];
  const T* xr = x + static_cast<int64_t>(blockIdx.x) * n;
  T* yr = y + static_cast<int64_t>(blockIdx.x) * n;
  float v[VPT * V];
  row_load<T, VPT>(xr, n, 0, bn, vec, -INFINITY, v);
  const float m = block_allreduce_max(tree_max(v), red);
  const float nm = -m * 1.4426950408889634f;
#pragma unroll
  for (int i = 0; i < VPT * V; ++i) v[i] = exp_shifted(v[i], nm);  // masked slots -> 0
  const float inv = 1.0f / block_allreduce_sum(tree_sum(v), red);
#pragma unroll
  for (int i = 0; i < VPT * V; ++i) v[i] *= inv;
  row_store<T, VPT>(yr, n, 0, bn, vec, v);
}

// Single tile staged in shared memory (fp32 copy of the row) when the
// per-thread share is too large for registers.
template <typename T>
__global__ void __launch_bounds__(1024) softmax_tile_smem(const T* __restrict__ x,
                                                          T* __restrict__ y, int64_t n) {
  using E = Elem<T>;
  extern __shared__ float srow[];
  __shared__ float red[32];
  const T* xr = x + static_cast<int64_t>(blockIdx.x) * n;
  T* yr = y + static_cast<int64_t>(blockIdx.x) * n;
  float m = -INFINITY;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float f = E::to_f(xr[i]);
    srow[i] = f;
    m = fmaxf(m, f);
  }
  m = block_allreduce_max(m, red);
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float e = exp_shifted(srow[i], -m * 1.4426950408889634f);
    srow[i] = e;
    s += e;
  }
  const float inv = 1.0f / block_allreduce_sum(s, red);
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) yr[i] = E::from_f(srow[i] * inv);
}

// Online two-pass softmax over BLOCK_N tiles (kernels.py:121-136): running
// (max, sum) per thread merged across the CTA, then a normalise pass.
template <typename T, int VPT>
__global__ void __launch_bounds__(1024) softmax_online(const T* __restrict__ x,
                                                       T* __restrict__ y, int64_t n, int64_t bn,
                                                       int vec) {
  constexpr int V = RowVec<T>::V;
  __shared__ float red[32];
  const T* xr = x + static_cast<int64_t>(blockIdx.x) * n;
  T* yr = y + static_cast<int64_t>(blockIdx.x) * n;
  float m = -INFINITY, s = 0.f;
  float v[VPT * V];
  for (int64_t t0 = 0; t0 < n; t0 += bn) {
    row_load<T, VPT>(xr, n, t0, bn, vec, -INFINITY, v);
    float tm = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPT * V; ++i) tm = fmaxf(tm, v[i]);
    const float nm = fmaxf(m, tm);
    if (nm != -INFINITY) {
      float ts = 0.f;
#pragma unroll
      for (int i = 0; i < VPT * V; ++i) ts += exp_shifted(v[i], -nm * 1.4426950408889634f);
      s = s * exp_shifted(m, -nm * 1.4426950408889634f) + ts;
      m = nm;
    }
  }
  const float M = block_allreduce_max(m, red);
  const float S = block_allreduce_sum(
      m == -INFINITY ? 0.f : s * exp_shifted(m, -M * 1.4426950408889634f), red);
  const float invS = 1.0f / S, nM = -M * 1.4426950408889634f;
  for (int64_t t0 = 0; t0 < n; t0 += bn) {
    row_load<T, VPT>(xr, n, t0, bn, vec, -INFINITY, v);
#pragma unroll
    for (int i = 0; i < VPT * V; ++i) v[i] = exp_shifted(v[i], nM) * invS;
    row_store<T, VPT>(yr, n, t0, bn, vec, v);
  }
}

// -------------------------------------------------------------- layernorm
// Single tile, centred variance (layernorm_kernel SINGLE_TILE branch,
// kernels.py:148-159).
template <typename T, int VPT>
__global__ void __launch_bounds__(1024) layernorm_tile_regs(const T* __restrict__ x,
                                                            const T* __restrict__ w,
                                                            const T* __restrict__ b,
                                                            T* __restrict__ y, int64_t n,
                                                            int64_t bn, float eps, int vec) {
  constexpr int V = RowVec<T>::V;
  __shared__ float red[32];
  const T* xr = x + static_cast<int64_t>(blockIdx.x) * n;
  T* yr = y + static_cast<int64_t>(blockIdx.x) * n;
  float v[VPT * V];
  row_load<T, VPT>(xr, n, 0, bn, vec, 0.f, v);
  const float mean = block_allreduce_sum(tree_sum(v), red) / static_cast<float>(n);
  float dq[VPT * V];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t e0 = (threadIdx.x + static_cast<int64_t>(j) * blockDim.x) * V;
#pragma unroll
    for (int u = 0; u < V; ++u) {
      const float d = (e0 + u < n) ? v[j * V + u] - mean : 0.f;
      dq[j * V + u] = d * d;
    }
  }
  const float var = block_allreduce_sum(tree_sum(dq), red) / static_cast<float>(n);
  const float rstd = 1.0f / sqrtf(var + eps);
  ln_affine<T, VPT>(w, b, n, 0, bn, vec, mean, rstd, v);
  row_store<T, VPT>(yr, n, 0, bn, vec, v);
}

template <typename T>
__global__ void __launch_bounds__(1024) layernorm_tile_smem(const T* __restrict__ x,
                                                            const T* __restrict__ w,
                                                            const T* __restrict__ b,
                                                            T* __restrict__ y, int64_t n,
                                                            float eps) {
  using E = Elem<T>;
  extern __shared__ float srow[];
  __shared__ float red[32];
  const T* xr = x + static_cast<int64_t>(blockIdx.x) * n;
  T* yr = y + static_cast<int64_t>(blockIdx.x) * n;
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float f = E::to_f(xr[i]);
    srow[i] = f;
    s += f;
  }
  const float mean = block_allreduce_sum(s, red) / static_cast<float>(n);
  float q = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float d = srow[i] - mean;
    q += d * d;
  }
  const float var = block_allreduce_sum(q, red) / static_cast<float>(n);
  const float rstd = 1.0f / sqrtf(var + eps);
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
    yr[i] = E::from_f((srow[i] - mean) * rstd * E::to_f(w[i]) + E::to_f(b[i]));
}

// Tiled two-pass layernorm with var = E[x^2] - E[x]^2 clamped at 0
// (kernels.py:160-179).
template <typename T, int VPT>
__global__ void __launch_bounds__(1024) layernorm_twopass(const T* __restrict__ x,
                                                          const T* __restrict__ w,
                                                          const T* __restrict__ b,
                                                          T* __restrict__ y, int64_t n,
                                                          int64_t bn, float eps, int vec) {
  constexpr int V = RowVec<T>::V;
  __shared__ float red[32];
  const T* xr = x + static_cast<int64_t>(blockIdx.x) * n;
  T* yr = y + static_cast<int64_t>(blockIdx.x) * n;
  float v[VPT * V];
  float s = 0.f, q = 0.f;
  for (int64_t t0 = 0; t0 < n; t0 += bn) {
    row_load<T, VPT>(xr, n, t0, bn, vec, 0.f, v);
#pragma unroll
    for (int i = 0; i < VPT * V; ++i) {
      s += v[i];
      q += v[i] * v[i];
    }
  }
  const float total = block_allreduce_sum(s, red);
  const float total_sq = block_allreduce_sum(q, red);
  const float mean = total / static_cast<float>(n);
  const float var = fmaxf(total_sq / static_cast<float>(n) - mean * mean, 0.f);
  const float rstd = 1.0f / sqrtf(var + eps);
  for (int64_t t0 = 0; t0 < n; t0 += bn) {
    row_load<T, VPT>(xr, n, t0, bn, vec, 0.f, v);
    ln_affine<T, VPT>(w, b, n, t0, bn, vec, mean, rstd, v);
    row_store<T, VPT>(yr, n, t0, bn, vec, v);
  }
}

// ------------------------------------------------- persistent, pipelined
// num_stages >= 2 with a single register tile and 16-byte aligned rows:
// gridDim.x persistent CTAs (SM count x resident CTAs) walk rows
// blockIdx.x, blockIdx.x + gridDim.x, ...; while a CTA reduces and writes
// row r it already has the raw 16-byte vectors of its next row in flight,
// so HBM reads never wait on the block reductions.

// Largest CTA of the persistent row kernels for VPT vector slots per thread:
// four or more slots (32+ values in registers, plus the next row's vectors)
// need more than the 64 registers a 1024-thread bound leaves, so those
// instantiations are bounded to 256 threads and plan_rows sends wider CTAs
// to the per-row kernels.
__host__ __device__ constexpr int row_pipe_max_threads(int vpt) { return vpt >= 4 ? 256 : 1024; }

// Raw vector slots of one row (vec path: n*sizeof(T) % 16 == 0, so a slot
// is either fully inside the row or fully outside; outside slots read 0).
template <typename T, int VPT>
__device__ __forceinline__ void raw_row_load(const T* __restrict__ row, int64_t n,
                                             uint4 (&r)[VPT]) {
  constexpr int V = RowVec<T>::V;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t e0 = (threadIdx.x + static_cast<int64_t>(j) * blockDim.x) * V;
    r[j] = e0 < n ? __ldcs(reinterpret_cast<const uint4*>(row + e0)) : make_uint4(0, 0, 0, 0);
  }
}

template <typename T, int VPT>
__device__ __forceinline__ void raw_unpack(const uint4 (&r)[VPT], int64_t n, float fill,
                                           float (&v)[VPT * RowVec<T>::V]) {
  using E = Elem<T>;
  constexpr int V = RowVec<T>::V;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const bool in = (threadIdx.x + static_cast<int64_t>(j) * blockDim.x) * V < n;
    const T* e = reinterpret_cast<const T*>(&r[j]);
#pragma unroll
    for (int u = 0; u < V; ++u) v[j * V + u] = in ? E::to_f(e[u]) : fill;
  }
}

template <typename T, int VPT>
__device__ __forceinline__ void raw_row_store(T* __restrict__ row, int64_t n,
                                              const float (&v)[VPT * RowVec<T>::V]) {
  using E = Elem<T>;
  constexpr int V = RowVec<T>::V;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t e0 = (threadIdx.x + static_cast<int64_t>(j) * blockDim.x) * V;
    if (e0 < n) {
      uint4 r;
      T* e = reinterpret_cast<T*>(&r);
#pragma unroll
      for (int u = 0; u < V; ++u) e[u] = E::from_f(v[j * V + u]);
      __stcs(reinterpret_cast<uint4*>(row + e0), r);
    }
  }
}

template <typename T, int VPT>
__global__ void __launch_bounds__(row_pipe_max_threads(VPT)) softmax_rows_pipe(const T* __restrict__ x,
                                                          T* __restrict__ y, int64_t m,
                                                          int64_t n) {
  constexpr int V = RowVec<T>::V;
  __shared__ float red[32];
  int64_t row = blockIdx.x;
  if (row >= m) return;
  uint4 cur[VPT], nxt[VPT];
  raw_row_load<T, VPT>(x + row * n, n, cur);
  for (; row < m; row += gridDim.x) {
    const int64_t nr = row + gridDim.x;
    if (nr < m) raw_row_load<T, VPT>(x + nr * n, n, nxt);
    float v[VPT * V];
    raw_unpack<T, VPT>(cur, n, -INFINITY, v);
    const float mx = block_allreduce_max(tree_max(v), red);
    const float nm = -mx * 1.4426950408889634f;
#pragma unroll
    for (int i = 0; i < VPT * V; ++i) v[i] = exp_shifted(v[i], nm);
    const float inv = 1.0f / block_allreduce_sum(tree_sum(v), red);
#pragma unroll
    for (int i = 0; i < VPT * V; ++i) v[i] *= inv;
    raw_row_store<T, VPT>(y + row * n, n, v);
#pragma unroll
    for (int j = 0; j < VPT; ++j) cur[j] = nxt[j];
  }
}

template <typename T, int VPT>
__global__ void __launch_bounds__(row_pipe_max_threads(VPT)) layernorm_rows_pipe(const T* __restrict__ x,
                                                            const T* __restrict__ w,
                                                            const T* __restrict__ b,
                                                            T* __restrict__ y, int64_t m,
                                                            int64_t n, float eps) {
  constexpr int V = RowVec<T>::V;
  __shared__ float red[32];
  int64_t row = blockIdx.x;
  if (row >= m) return;
  uint4 cur[VPT], nxt[VPT];
  raw_row_load<T, VPT>(x + row * n, n, cur);
  for (; row < m; row += gridDim.x) {
    const int64_t nr = row + gridDim.x;
    if (nr < m) raw_row_load<T, VPT>(x + nr * n, n, nxt);
    float v[VPT * V];
    raw_unpack<T, VPT>(cur, n, 0.f, v);
    const float mean = block_allreduce_sum(tree_sum(v), red) / static_cast<float>(n);
    float dq[VPT * V];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const bool in = (threadIdx.x + static_cast<int64_t>(j) * blockDim.x) * V < n;
#pragma unroll
      for (int u = 0; u < V; ++u) {
        const float d = in ? v[j * V + u] - mean : 0.f;
        dq[j * V + u] = d * d;
      }
    }
    const float var = block_allreduce_sum(tree_sum(dq), red) / static_cast<float>(n);
    const float rstd = 1.0f / sqrtf(var + eps);
    ln_affine<T, VPT>(w, b, n, 0, n, true, mean, rstd, v);
    raw_row_store<T, VPT>(y + row * n, n, v);
#pragma unroll
    for (int j = 0; j < VPT; ++j) cur[j] = nxt[j];
  }
}

// Element pair p (elements 2p and 2p+1) of a 16-byte vector, as fp32.  A
// bf16 value is the upper half of the fp32 with the same bits, so each
// unpacks with one shift or mask.
template <typename T>
__device__ __forceinline__ float2 unpack2(const uint4& r, int p);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(const uint4& r, int p) {
  const uint32_t w = (&r.x)[p];
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(const uint4& r, int p) {
  const uint32_t w = (&r.x)[p];
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
template <>
__device__ __forceinline__ float2 unpack2<float>(const uint4& r, int p) {
  return make_float2(__uint_as_float((&r.x)[2 * p]), __uint_as_float((&r.x)[2 * p + 1]));
}

// Round an fp32 pair to T and place it as elements 2p, 2p+1 of a vector.
template <typename T>
__device__ __forceinline__ void pack2(uint4& r, int p, float2 y);
template <>
__device__ __forceinline__ void pack2<__nv_bfloat16>(uint4& r, int p, float2 y) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(y.x, y.y);
  (&r.x)[p] = *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ void pack2<__half>(uint4& r, int p, float2 y) {
  const __half2 h = __floats2half2_rn(y.x, y.y);
  (&r.x)[p] = *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ void pack2<float>(uint4& r, int p, float2 y) {
  (&r.x)[2 * p] = __float_as_uint(y.x);
  (&r.x)[2 * p + 1] = __float_as_uint(y.y);
}

// Sums of two values over the block in one exchange; every thread receives
// both.
__device__ __forceinline__ float2 block_allreduce_sum2(float2 v, float2* red2) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
    v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red2[w] = v;
  __syncthreads();
  float2 r = l < nw ? red2[l] : make_float2(0.f, 0.f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    r.x += __shfl_xor_sync(0xffffffffu, r.x, o);
    r.y += __shfl_xor_sync(0xffffffffu, r.y, o);
  }
  return r;
}

// ------------------------------------------- persistent, bulk-copy ring
// num_stages = R >= 2 with a single register tile, 16-byte aligned rows and
// R (+ gamma, beta) rows of shared memory: thread 0 streams whole rows into
// an R-slot shared-memory ring with cp.async.bulk (one mbarrier per slot),
// so R rows per CTA are in flight without holding registers, and every
// thread reads its vector slots of the row from shared memory.  The first
// block reduction of a row also proves that every thread has read its slot,
// so thread 0 refills the slot with row + R * gridDim.x right after it.
// Layernorm keeps gamma and beta in shared memory for the CTA's lifetime
// and takes the row statistics in one pass: sums of d = x - x0 and d^2
// with x0 the row's first element (the shifted-data variance, exact in
// real arithmetic and free of the E[x^2] - E[x]^2 cancellation as long as
// x0 lies within a few standard deviations of the mean), so a row needs
// one block reduction of two values instead of the two dependent
// reductions of the centred form.  When the shift is far from the mean,
// (mean - x0)^2 > kShiftGuard * var, the shifted variance has lost up to
// kShiftGuard + 1 times fp32 rounding of its value, so the row takes a
// second reduction of e = x - mean and e^2 over the values still in
// registers: the mean gains the small correction sum(e) / n and the
// variance is the centred one, the reference's single-tile formula
// (compiler/triton/kernels.py:148-159).  For rows of
// i.i.d. values that is the chance that the first element lies four
// standard deviations out (6e-5).  The math runs on packed fp32x2
// instructions.
constexpr int kRowRing = 4;
constexpr float kShiftGuard = 16.0f;

template <typename T, int VPT, bool LN>
__global__ void __launch_bounds__(row_pipe_max_threads(VPT)) rows_ring(const T* __restrict__ x,
                                                  const T* __restrict__ w,
                                                  const T* __restrict__ b, T* __restrict__ y,
                                                  int64_t m, int64_t n, float eps, int R,
                                                  unsigned int* err) {
  constexpr int V = RowVec<T>::V;
  extern __shared__ uint8_t dsm[];
  __shared__ uint64_t full[kRowRing];
  __shared__ float red[32];
  __shared__ float2 red2[32];
  __shared__ int abort_word;
  const uint32_t rowbytes = static_cast<uint32_t>(n) * sizeof(T);
  const uint32_t slot = (rowbytes + 127u) & ~127u;
  const uint32_t base = (smem_u32(dsm) + 127u) & ~127u;
  const uint8_t* basep = dsm + (base - smem_u32(dsm));
  if (threadIdx.x == 0) {
    for (int s = 0; s < R; ++s) mbar_init(smem_u32(&full[s]), 1);
    abort_word = 0;
    fence_barrier_init();
  }
  if constexpr (LN) {
    uint4* ws = reinterpret_cast<uint4*>(const_cast<uint8_t*>(basep) + R * slot);
    uint4* bs = reinterpret_cast<uint4*>(const_cast<uint8_t*>(basep) + (R + 1) * slot);
    for (int64_t i = threadIdx.x; i < n / V; i += blockDim.x) {
      ws[i] = __ldg(reinterpret_cast<const uint4*>(w) + i);
      bs[i] = __ldg(reinterpret_cast<const uint4*>(b) + i);
    }
  }
  __syncthreads();
  volatile int* abort_flag = &abort_word;
  int64_t row = blockIdx.x;
  int64_t issued = 0, consumed = 0;  // rows streamed / rows taken (thread 0's view)
  if (threadIdx.x == 0) {
    for (int k = 0; k < R; ++k) {
      const int64_t r = row + static_cast<int64_t>(k) * gridDim.x;
      if (r >= m) break;
      mbar_arrive_expect_tx(smem_u32(&full[k]), rowbytes);
      bulk_load(base + k * slot, x + r * n, rowbytes, smem_u32(&full[k]));
      ++issued;
    }
  }
  int s = 0;
  uint32_t ph = 0;
  // thread 0 streams row + R * gridDim.x into the slot just read by all
  auto refill = [&]() {
    if (threadIdx.x == 0) {
      const int64_t r2 = row + static_cast<int64_t>(R) * gridDim.x;
      if (r2 < m) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(smem_u32(&full[s]), rowbytes);
        bulk_load(base + s * slot, x + r2 * n, rowbytes, smem_u32(&full[s]));
        ++issued;
      }
    }
  };
  for (; row < m; row += gridDim.x) {
    const bool ok = mbar_wait(smem_u32(&full[s]), ph, abort_flag, err, kErrWaitProducer);
    if (!__syncthreads_and(ok)) break;
    ++consumed;
    uint4 raw[VPT];
    const uint8_t* src = basep + s * slot;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int64_t e0 = (threadIdx.x + static_cast<int64_t>(j) * blockDim.x) * V;
      raw[j] = e0 < n ? *reinterpret_cast<const uint4*>(src + e0 * sizeof(T))
                      : make_uint4(0, 0, 0, 0);
    }
    if constexpr (LN) {
      constexpr int P = V / 2;  // fp32 pairs per vector slot
      const float x0 = Elem<T>::to_f(*reinterpret_cast<const T*>(src));
      const float2 nx0 = make_float2(-x0, -x0);
      float2 xv[VPT * P];
      float2 sacc[4], qacc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) sacc[i] = qacc[i] = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const bool in = (threadIdx.x + static_cast<int64_t>(j) * blockDim.x) * V < n;
#pragma unroll
        for (int u = 0; u < P; ++u) {
          xv[j * P + u] = unpack2<T>(raw[j], u);
          if (in) {
            const float2 d = __fadd2_rn(xv[j * P + u], nx0);
            sacc[(j * P + u) & 3] = __fadd2_rn(sacc[(j * P + u) & 3], d);
            qacc[(j * P + u) & 3] = __ffma2_rn(d, d, qacc[(j * P + u) & 3]);
          }
        }
      }
      const float2 s01 = __fadd2_rn(sacc[0], sacc[1]), s23 = __fadd2_rn(sacc[2], sacc[3]);
      const float2 q01 = __fadd2_rn(qacc[0], qacc[1]), q23 = __fadd2_rn(qacc[2], qacc[3]);
      const float2 ss = __fadd2_rn(s01, s23), qq = __fadd2_rn(q01, q23);
      // the reduction's barriers order every thread's slot read before the
      // refill below
      const float2 sq = block_allreduce_sum2(make_float2(ss.x + ss.y, qq.x + qq.y), red2);
      refill();
      const float inv_n = 1.0f / static_cast<float>(n);
      const float dm = sq.x * inv_n;  // mean of d
      float mean = x0 + dm;
      float var = fmaxf(fmaf(-dm, dm, sq.y * inv_n), 0.f);
      // x0 far from the row mean (an outlying first element): the shifted
      // sums then cancel, so take the centred sum of squares over the row
      // values still in registers.  The vote keeps the branch (and its
      // block reduction) uniform even where the lanes' reduced sums differ
      // in their last bit.
      if (__syncthreads_or(dm * dm > kShiftGuard * var)) {
        // sums of e = x - mean and e^2: the mean takes the (now small)
        // correction sum(e) / n and the variance is the centred one
        const float2 nm2 = make_float2(-mean, -mean);
        float2 eacc[4], cacc[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) eacc[i] = cacc[i] = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          const bool in = (threadIdx.x + static_cast<int64_t>(j) * blockDim.x) * V < n;
#pragma unroll
          for (int u = 0; u < P; ++u) {
            if (in) {
              const float2 e = __fadd2_rn(xv[j * P + u], nm2);
              eacc[(j * P + u) & 3] = __fadd2_rn(eacc[(j * P + u) & 3], e);
              cacc[(j * P + u) & 3] = __ffma2_rn(e, e, cacc[(j * P + u) & 3]);
            }
          }
        }
        const float2 e2 = __fadd2_rn(__fadd2_rn(eacc[0], eacc[1]), __fadd2_rn(eacc[2], eacc[3]));
        const float2 c2 = __fadd2_rn(__fadd2_rn(cacc[0], cacc[1]), __fadd2_rn(cacc[2], cacc[3]));
        const float2 ec = block_allreduce_sum2(make_float2(e2.x + e2.y, c2.x + c2.y), red2);
        const float de = ec.x * inv_n;
        mean += de;
        var = fmaxf(fmaf(-de, de, ec.y * inv_n), 0.f);
      }
      const float rstd = 1.0f / sqrtf(var + eps);
      const float2 nmean = make_float2(-mean, -mean), rstd2 = make_float2(rstd, rstd);
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int64_t e0 = (threadIdx.x + static_cast<int64_t>(j) * blockDim.x) * V;
        if (e0 < n) {
          const uint4 wr = *reinterpret_cast<const uint4*>(basep + R * slot + e0 * sizeof(T));
          const uint4 br = *reinterpret_cast<const uint4*>(basep + (R + 1) * slot + e0 * sizeof(T));
          uint4 o;
#pragma unroll
          for (int u = 0; u < P; ++u) {
            const float2 t = __fmul2_rn(__fadd2_rn(xv[j * P + u], nmean), rstd2);
            pack2<T>(o, u, __ffma2_rn(t, unpack2<T>(wr, u), unpack2<T>(br, u)));
          }
          __stcs(reinterpret_cast<uint4*>(y + row * n + e0), o);
        }
      }
    } else {
      constexpr int P = V / 2;
      float2 xv[VPT * P];
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const bool in = (threadIdx.x + static_cast<int64_t>(j) * blockDim.x) * V < n;
#pragma unroll
        for (int u = 0; u < P; ++u) {
          xv[j * P + u] = unpack2<T>(raw[j], u);
          if (in) mx4[(j * P + u) & 3] = fmax3(mx4[(j * P + u) & 3], xv[j * P + u].x, xv[j * P + u].y);
        }
      }
      // first reduction: its barriers also order every thread's slot read
      // before the refill below
      const float mx = block_allreduce_max(fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])), red);
      refill();
      // exp(x - mx) = 2^(x * log2 e - mx * log2 e): one packed FMA per pair
      // and one ex2 per element
      const float2 l2e = make_float2(1.4426950408889634f, 1.4426950408889634f);
      const float2 nm = make_float2(-mx * 1.4426950408889634f, -mx * 1.4426950408889634f);
      float2 sacc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) sacc[i] = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const bool in = (threadIdx.x + static_cast<int64_t>(j) * blockDim.x) * V < n;
#pragma unroll
        for (int u = 0; u < P; ++u) {
          const float2 t = __ffma2_rn(xv[j * P + u], l2e, nm);
          xv[j * P + u] = make_float2(ex2_approx(t.x), ex2_approx(t.y));
          if (in) sacc[(j * P + u) & 3] = __fadd2_rn(sacc[(j * P + u) & 3], xv[j * P + u]);
        }
      }
      const float2 s2 = __fadd2_rn(__fadd2_rn(sacc[0], sacc[1]), __fadd2_rn(sacc[2], sacc[3]));
      const float inv = 1.0f / block_allreduce_sum(s2.x + s2.y, red);
      const float2 inv2 = make_float2(inv, inv);
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int64_t e0 = (threadIdx.x + static_cast<int64_t>(j) * blockDim.x) * V;
        if (e0 < n) {
          uint4 o;
#pragma unroll
          for (int u = 0; u < P; ++u) pack2<T>(o, u, __fmul2_rn(xv[j * P + u], inv2));
          __stcs(reinterpret_cast<uint4*>(y + row * n + e0), o);
        }
      }
    }
    if (++s == R) {
      s = 0;
      ph ^= 1u;
    }
  }
  // after an abort: let every streamed row land before the CTA exits
  if (threadIdx.x == 0) {
    for (int64_t i = consumed; i < issued; ++i)
      mbar_wait_drain(smem_u32(&full[i % R]), static_cast<uint32_t>(i / R) & 1u, err);
  }
}

// Shared memory a ring of R rows (+ gamma and beta for layernorm) needs.
static uint32_t ring_smem(int64_t n, int es, int R, bool ln) {
  const uint64_t slot = (static_cast<uint64_t>(n) * es + 127u) & ~uint64_t{127};
  const uint64_t total = slot * static_cast<uint64_t>(R + (ln ? 2 : 0)) + 128u;
  return total > kMaxSmemPerCta ? 0u : static_cast<uint32_t>(total);
}

// ------------------------------------------------------------------- host
// Plan: aux[0] = VPT (vector slots per thread, 0 = smem-staged single tile),
// aux[1] = single-tile flag, aux[2] = dynamic smem bytes.
static gpo_status plan_rows(const gpo_key& k, Plan& p, std::string& log, const char* what) {
  if (k.ndim != 2 || k.shape[0] < 0 || k.shape[1] < 1) {
    log = "expected a 2-D shape (M, N) with N >= 1";
    return GPO_BAD_CONFIG;
  }
  if (k.dtype == GPO_TF32) {
    log = "row kernels have no tf32 variant";
    return GPO_BAD_CONFIG;
  }
  if (k.num_warps < 1 || k.num_warps > 32 || k.block_n < 1 || k.block_n > (1 << 16)) {
    log = "num_warps must be in [1, 32] and BLOCK_N in [1, 65536]";
    return GPO_BAD_CONFIG;
  }
  const int64_t n = k.shape[1];
  const int threads = k.num_warps * 32;
  const int V = 16 / dtype_bytes(k.dtype);
  const bool single = k.block_n >= n;
  const int64_t slots = static_cast<int64_t>(cdiv(k.block_n, static_cast<uint64_t>(threads) * V));
  int vpt = 1;
  while (vpt < slots) vpt *= 2;
  const int vpt_max = 64 / V;  // at most 64 fp32 values per thread in registers
  uint32_t dyn = 0;
  if (vpt > vpt_max) {
    if (!single) {
      // tiles larger than the register budget cannot be processed in one
      // sweep per thread; Triton's equivalent spills.  Report honestly.
      log = "BLOCK_N tile needs " + std::to_string(slots * V) +
            " fp32 values per thread (> 64-register tile budget) in the tiled variant";
      return GPO_COMPILE_ERROR;
    }
    vpt = 0;
    dyn = static_cast<uint32_t>(n) * 4u;
    if (dyn + 128 > kMaxSmemPerCta) {
      log = "row of " + std::to_string(n) + " fp32 values exceeds 227 KB shared memory";
      return GPO_COMPILE_ERROR;
    }
  }
  p.aux[0] = vpt;
  p.aux[1] = single ? 1 : 0;
  p.aux[2] = static_cast<int>(dyn);
  // persistent row pipeline: register tile, single tile, aligned rows;
  // a shared-memory ring of num_stages rows when it fits (aux[3] = 2),
  // else one row prefetched into registers (aux[3] = 1)
  const bool pipe = single && vpt > 0 && k.num_stages >= 2 &&
                    (n * dtype_bytes(k.dtype)) % 16 == 0 && threads <= row_pipe_max_threads(vpt);
  const int ring_r = std::min(k.num_stages, kRowRing);
  const uint32_t ring_dyn =
      pipe ? ring_smem(n, dtype_bytes(k.dtype), ring_r, k.task == GPO_TASK_LAYERNORM) : 0u;
  p.aux[3] = pipe ? (ring_dyn ? 2 : 1) : 0;
  p.aux[4] = ring_r;
  if (ring_dyn) {
    dyn = ring_dyn;
    p.aux[2] = static_cast<int>(dyn);
  }
  p.family = "row_kernels";
  p.res.threads_per_cta = static_cast<uint32_t>(threads);
  p.res.grid_x = static_cast<uint32_t>(std::max<int64_t>(1, k.shape[0]));
  p.res.grid_y = p.res.grid_z = 1;
  p.res.launches_per_call = 1;
  p.res.smem_bytes = dyn + 128;
  if (ring_dyn)
    snprintf(p.res.kernel, sizeof(p.res.kernel), "%s_rows_ring<vpt=%d,rows=%d>", what, vpt,
             ring_r);
  else
    snprintf(p.res.kernel, sizeof(p.res.kernel), "%s_%s<vpt=%d>", what,
             pipe ? "rows_pipe"
                  : single ? (vpt ? "tile_regs" : "tile_smem")
                           : (k.task == GPO_TASK_SOFTMAX ? "online" : "twopass"),
             vpt);
  if (pipe) p.res.persistent = 1;
  return GPO_OK;
}

gpo_status plan_softmax(const gpo_key& k, Plan& p, std::string& log) {
  return plan_rows(k, p, log, "softmax");
}
gpo_status plan_layernorm(const gpo_key& k, Plan& p, std::string& log) {
  return plan_rows(k, p, log, "layernorm");
}

template <typename T, int VPT>
static gpo_status softmax_vpt(const gpo_key& k, const Plan& p, const gpo_args& a,
                              const LaunchCtx& c, int vec) {
  const unsigned grid = static_cast<unsigned>(k.shape[0]);
  const int threads = k.num_warps * 32;
  const T* x = static_cast<const T*>(a.in[0]);
  T* y = static_cast<T*>(a.out);
  if (p.aux[3] == 2 && vec) {
    auto kern = rows_ring<T, VPT, false>;
    const uint32_t dyn = static_cast<uint32_t>(p.aux[2]);
    gpo_status s = ensure_smem_attr(reinterpret_cast<const void*>(kern), dyn);
    if (s != GPO_OK) return s;
    const unsigned pg = persistent_grid(reinterpret_cast<const void*>(kern), threads, dyn,
                                        c.sm_count, k.shape[0]);
    kern<<<pg, threads, dyn, c.stream>>>(x, nullptr, nullptr, y, k.shape[0], k.shape[1], 0.f,
                                         p.aux[4], c.err);
  } else if (p.aux[3] && vec) {
    auto kern = softmax_rows_pipe<T, VPT>;
    const unsigned pg = persistent_grid(reinterpret_cast<const void*>(kern), threads, 0,
                                        c.sm_count, k.shape[0]);
    kern<<<pg, threads, 0, c.stream>>>(x, y, k.shape[0], k.shape[1]);
  } else if (p.aux[1])
    softmax_tile_regs<T, VPT><<<grid, threads, 0, c.stream>>>(x, y, k.shape[1], k.block_n, vec);
  else
    softmax_online<T, VPT><<<grid, threads, 0, c.stream>>>(x, y, k.shape[1], k.block_n, vec);
  return launch_status();
}

template <typename T>
static gpo_status softmax_dt(const gpo_key& k, const Plan& p, const gpo_args& a,
                             const LaunchCtx& c) {
  const int vec = (aligned16(a.in[0]) && aligned16(a.out) &&
                   (k.shape[1] * static_cast<int64_t>(sizeof(T))) % 16 == 0)
                      ? 1
                      : 0;
  switch (p.aux[0]) {
    case 0: {
      const uint32_t dyn = static_cast<uint32_t>(p.aux[2]);
      gpo_status s = ensure_smem_attr(reinterpret_cast<const void*>(&softmax_tile_smem<T>), dyn);
      if (s != GPO_OK) return s;
      softmax_tile_smem<T><<<static_cast<unsigned>(k.shape[0]), k.num_warps * 32, dyn, c.stream>>>(
          static_cast<const T*>(a.in[0]), static_cast<T*>(a.out), k.shape[1]);
      return launch_status();
    }
    case 1: return softmax_vpt<T, 1>(k, p, a, c, vec);
    case 2: return softmax_vpt<T, 2>(k, p, a, c, vec);
    case 4: return softmax_vpt<T, 4>(k, p, a, c, vec);
    case 8: return softmax_vpt<T, 8>(k, p, a, c, vec);
    case 16: return softmax_vpt<T, 16>(k, p, a, c, vec);
    default: return GPO_INTERNAL;
  }
}

gpo_status launch_softmax(const gpo_key& k, const Plan& p, const gpo_args& a, const LaunchCtx& c) {
  if (!a.in[0] || !a.out) return GPO_BAD_ARGS;
  if (k.shape[0] == 0) return GPO_OK;
  switch (k.dtype) {
    case GPO_FLOAT32: return softmax_dt<float>(k, p, a, c);
    case GPO_FLOAT16: return softmax_dt<__half>(k, p, a, c);
    case GPO_BFLOAT16: return softmax_dt<__nv_bfloat16>(k, p, a, c);
    default: return GPO_BAD_ARGS;
  }
}

template <typename T, int VPT>
static gpo_status layernorm_vpt(const gpo_key& k, const Plan& p, const gpo_args& a,
                                const LaunchCtx& c, int vec, float eps) {
  const unsigned grid = static_cast<unsigned>(k.shape[0]);
  const int threads = k.num_warps * 32;
  const T* x = static_cast<const T*>(a.in[0]);
  const T* w = static_cast<const T*>(a.in[1]);
  const T* b = static_cast<const T*>(a.in[2]);
  T* y = static_cast<T*>(a.out);
  if (p.aux[3] == 2 && vec) {
    auto kern = rows_ring<T, VPT, true>;
    const uint32_t dyn = static_cast<uint32_t>(p.aux[2]);
    gpo_status s = ensure_smem_attr(reinterpret_cast<const void*>(kern), dyn);
    if (s != GPO_OK) return s;
    const unsigned pg = persistent_grid(reinterpret_cast<const void*>(kern), threads, dyn,
                                        c.sm_count, k.shape[0]);
    kern<<<pg, threads, dyn, c.stream>>>(x, w, b, y, k.shape[0], k.shape[1], eps, p.aux[4],
                                         c.err);
  } else if (p.aux[3] && vec) {
    auto kern = layernorm_rows_pipe<T, VPT>;
    const unsigned pg = persistent_grid(reinterpret_cast<const void*>(kern), threads, 0,
                                        c.sm_count, k.shape[0]);
    kern<<<pg, threads, 0, c.stream>>>(x, w, b, y, k.shape[0], k.shape[1], eps);
  } else if (p.aux[1])
    layernorm_tile_regs<T, VPT>
        <<<grid, threads, 0, c.stream>>>(x, w, b, y, k.shape[1], k.block_n, eps, vec);
  else
    layernorm_twopass<T, VPT>
        <<<grid, threads, 0, c.stream>>>(x, w, b, y, k.shape[1], k.block_n, eps, vec);
  return launch_status();
}

template <typename T>
static gpo_status layernorm_dt(const gpo_key& k, const Plan& p, const gpo_args& a,
                               const LaunchCtx& c) {
  const float eps = a.eps > 0.f ? a.eps : 1e-5f;
  const int vec = (aligned16(a.in[0]) && aligned16(a.in[1]) && aligned16(a.in[2]) &&
                   aligned16(a.out) &&
                   (k.shape[1] * static_cast<int64_t>(sizeof(T))) % 16 == 0)
                      ? 1
                      : 0;
  switch (p.aux[0]) {
    case 0: {
      const uint32_t dyn = static_cast<uint32_t>(p.aux[2]);
      gpo_status s =
          ensure_smem_attr(reinterpret_cast<const void*>(&layernorm_tile_smem<T>), dyn);
      if (s != GPO_OK) return s;
      layernorm_tile_smem<T>
          <<<static_cast<unsigned>(k.shape[0]), k.num_warps * 32, dyn, c.stream>>>(
              static_cast<const T*>(a.in[0]), static_cast<const T*>(a.in[1]),
              static_cast<const T*>(a.in[2]), static_cast<T*>(a.out), k.shape[1], eps);
      return launch_status();
    }
    case 1: return layernorm_vpt<T, 1>(k, p, a, c, vec, eps);
    case 2: return layernorm_vpt<T, 2>(k, p, a, c, vec, eps);
    case 4: return layernorm_vpt<T, 4>(k, p, a, c, vec, eps);
    case 8: return layernorm_vpt<T, 8>(k, p, a, c, vec, eps);
    case 16: return layernorm_vpt<T, 16>(k, p, a, c, vec, eps);
    default: return GPO_INTERNAL;
  }
}

gpo_status launch_layernorm(const gpo_key& k, const Plan& p, const gpo_args& a,
                            const LaunchCtx& c) {
  if (!a.in[0] || !a.in[1] || !a.in[2] || !a.out) return GPO_BAD_ARGS;
  if (k.shape[0] == 0) return GPO_OK;
  switch (k.dtype) {
    case GPO_FLOAT32: return layernorm_dt<float>(k, p, a, c);
    case GPO_FLOAT16: return layernorm_dt<__half>(k, p, a, c);
    case GPO_BFLOAT16: return layernorm_dt<__nv_bfloat16>(k, p, a, c);
    default: return GPO_BAD_ARGS;
  }
}

}  // namespace gpo

// Bandwidth-bound kernel families: vecadd, fused / unfused elementwise
// (relu and gelu variants) and fp32 sum reduction (loop / atomic / two_pass).
//
// Launch geometry follows the reference's program model so that every
// config is a distinct, meaningful instantiation: one CTA of num_warps*32
// threads per BLOCK_SIZE slice (compiler/triton/runner.py:123,146,150,210),
// except the `loop` reduction which is a single CTA (runner.py:141,156).
// Inside a CTA the slice is moved with 16-byte vector accesses whenever the
// slice start and the three base pointers are 16-byte aligned; a scalar path
// covers the ragged tail and unaligned views.
#include <algorithm>
#include <mutex>

#include "gpo_common.cuh"
#include "gpo_internal.h"

namespace gpo {

// ---------------------------------------------------------------- op codes
enum EwOp : int {
  kOpAdd = 0,        // a + b                        (vecadd_kernel, kernels.py:68-75)
  kOpScale = 1,      // a * s                        (scale_kernel, kernels.py:195-201)
  kOpRelu = 2,       // max(a, 0)                    (relu_kernel, kernels.py:203-209)
  kOpFusedRelu = 3,  // max(a*s + b, 0) in fp32      (kernels.py:182-193)
  kOpGelu = 4,       // gelu(a), erf form (erf per A&S 7.1.26)
  kOpFusedGelu = 5,  // gelu(a*s + b) in fp32
};

// erf(x) by Abramowitz & Stegun, Handbook of Mathematical Functions,
// formula 7.1.26: erf(x) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5)
// exp(-x^2), t = 1 / (1 + p x), x >= 0, |error| <= 1.5e-7; odd extension
// for x < 0.  One reciprocal, one exp2 and a 5-term Horner chain.
__device__ __forceinline__ float erf_as7126(float x) {
  const float ax = fabsf(x);
  float t;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(0.3275911f, ax, 1.0f)));
  float poly = fmaf(1.061405429f, t, -1.453152027f);
  poly = fmaf(poly, t, 1.421413741f);
  poly = fmaf(poly, t, -0.284496736f);
  poly = fmaf(poly, t, 0.254829592f);
  poly *= t;
  const float e = ex2_approx(-ax * ax * 1.4426950408889634f);  // exp(-x^2)
  return copysignf(fmaf(-poly, e, 1.0f), x);
}

// gelu(z) = z * Phi(z) = 0.5 z (1 + erf(z / sqrt 2))
__device__ __forceinline__ float gelu_erf(float z) {
  return 0.5f * z * (1.0f + erf_as7126(z * 0.70710678118654752f));
}

template <int OP>
__device__ __forceinline__ float ew_apply(float a, float b, float s) {
  if constexpr (OP == kOpAdd) {
    return __fadd_rn(a, b);
  } else if constexpr (OP == kOpScale) {
    return __fmul_rn(a, s);
  } else if constexpr (OP == kOpRelu) {
    return a > 0.f ? a : 0.f;
  } else if constexpr (OP == kOpFusedRelu) {
    // two roundings (mul, add), as the fp32 torch expression computes it
    const float z = __fadd_rn(__fmul_rn(a, s), b);
    return z > 0.f ? z : 0.f;
  } else if constexpr (OP == kOpGelu) {
    return gelu_erf(a);
  } else {
    return gelu_erf(__fadd_rn(__fmul_rn(a, s), b));
  }
}

template <int OP>
constexpr bool ew_binary() {
  return OP == kOpAdd || OP == kOpFusedRelu || OP == kOpFusedGelu;
}

// One CTA per BLOCK_SIZE slice.  Vector path when `vec` (alignment checked
// on the host: pointers 16-byte aligned and BLOCK_SIZE*sizeof(T) % 16 == 0).
template <typename T, int OP>
__global__ void __launch_bounds__(1024) ew_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                                  T* __restrict__ out, int64_t n,
                                                  int64_t block_size, float s, int vec) {
  using E = Elem<T>;
  constexpr int V = 16 / sizeof(T);
  const int64_t base = static_cast<int64_t>(blockIdx.x) * block_size;
  if (base >= n) return;
  const int64_t lim = (n - base) < block_size ? (n - base) : block_size;
  int64_t done = 0;
  if (vec) {
    const int64_t nvec = lim / V;
    const uint4* av = reinterpret_cast<const uint4*>(a + base);
    const uint4* bv = reinterpret_cast<const uint4*>(ew_binary<OP>() ? b + base : a + base);
    uint4* ov = reinterpret_cast<uint4*>(out + base);
    // Batches of EW_BATCH vectors per thread: every load of a batch is
    // issued before the first store, so each thread keeps up to
    // 2 * EW_BATCH 16-byte loads in flight.
    constexpr int EW_BATCH = 4;
    const int64_t T_ = blockDim.x;
    for (int64_t i0 = threadIdx.x; i0 < nvec; i0 += EW_BATCH * T_) {
      uint4 ra[EW_BATCH], rb[EW_BATCH];
#pragma unroll
      for (int u = 0; u < EW_BATCH; ++u) {
        const int64_t i = i0 + u * T_;
        if (i < nvec) {
          ra[u] = __ldcs(av + i);
          if constexpr (ew_binary<OP>()) rb[u] = __ldcs(bv + i);
        }
      }
#pragma unroll
      for (int u = 0; u < EW_BATCH; ++u) {
        const int64_t i = i0 + u * T_;
        if (i < nvec) {
          const T* ea = reinterpret_cast<const T*>(&ra[u]);
          const T* eb = reinterpret_cast<const T*>(&rb[u]);
          uint4 ro;
          T* eo = reinterpret_cast<T*>(&ro);
#pragma unroll
          for (int j = 0; j < V; ++j) {
            const float fb = ew_binary<OP>() ? E::to_f(eb[j]) : 0.f;
            eo[j] = E::from_f(ew_apply<OP>(E::to_f(ea[j]), fb, s));
          }
          __stcs(ov + i, ro);
        }
      }
    }
    done = nvec * V;
  }
  for (int64_t i = done + threadIdx.x; i < lim; i += blockDim.x) {
    const float fb = ew_binary<OP>() ? E::to_f(b[base + i]) : 0.f;
    out[base + i] = E::from_f(ew_apply<OP>(E::to_f(a[base + i]), fb, s));
  }
}

// ------------------------------------------------------------ host helpers
static gpo_status check_1d_key(const gpo_key& k, std::string& log) {
  if (k.ndim != 1 || k.shape[0] < 0) {
    log = "expected a 1-D shape (n,)";
    return GPO_BAD_CONFIG;
  }
  if (k.block_size < 1 || k.block_size > (1 << 20)) {
    log = "BLOCK_SIZE must be in [1, 2^20]";
    return GPO_BAD_CONFIG;
  }
  if (k.num_warps < 1 || k.num_warps > 32) {
    log = "num_warps must be in [1, 32]";
    return GPO_BAD_CONFIG;
  }
  return GPO_OK;
}

static void fill_1d_res(const gpo_key& k, Plan& p, const char* name, uint32_t launches) {
  const uint64_t n = static_cast<uint64_t>(k.shape[0]);
  p.res.threads_per_cta = static_cast<uint32_t>(k.num_warps) * 32u;
  p.res.grid_x = static_cast<uint32_t>(std::max<uint64_t>(1, cdiv(n, k.block_size)));
  p.res.grid_y = p.res.grid_z = 1;
  p.res.launches_per_call = launches;
  p.res.smem_bytes = static_cast<uint32_t>(k.num_warps) * 4u;
  snprintf(p.res.kernel, sizeof(p.res.kernel), "%s", name);
}

template <typename T, int OP>
static gpo_status run_ew(const void* a, const void* b, void* out, int64_t n, int64_t bs,
                         int warps, float s, cudaStream_t st) {
  if (n == 0) return GPO_OK;
  const bool vec = aligned16(a) && aligned16(out) && (!ew_binary<OP>() || aligned16(b)) &&
                   ((bs * static_cast<int64_t>(sizeof(T))) % 16 == 0);
  const unsigned grid = static_cast<unsigned>(cdiv(n, bs));
  ew_kernel<T, OP><<<grid, warps * 32, 0, st>>>(static_cast<const T*>(a),
                                                static_cast<const T*>(b), static_cast<T*>(out),
                                                n, bs, s, vec ? 1 : 0);
  return launch_status();
}

template <int OP>
static gpo_status run_ew_dt(int dt, const void* a, const void* b, void* out, int64_t n,
                            int64_t bs, int warps, float s, cudaStream_t st) {
  switch (dt) {
    case GPO_FLOAT32:
      return run_ew<float, OP>(a, b, out, n, bs, warps, s, st);
    case GPO_FLOAT16:
      return run_ew<__half, OP>(a, b, out, n, bs, warps, s, st);
    case GPO_BFLOAT16:
      return run_ew<__nv_bfloat16, OP>(a, b, out, n, bs, warps, s, st);
    default:
      return GPO_BAD_ARGS;
  }
}

// ------------------------------------------------------------------ vecadd
gpo_status plan_vecadd(const gpo_key& k, Plan& p, std::string& log) {
  gpo_status s = check_1d_key(k, log);
  if (s != GPO_OK) return s;
  if (k.dtype == GPO_TF32) {
    log = "vecadd has no tf32 variant";
    return GPO_BAD_CONFIG;
  }
  p.family = "bw_kernels";
  fill_1d_res(k, p, "ew_kernel<add>", 1);
  return GPO_OK;
}

gpo_status launch_vecadd(const gpo_key& k, const Plan&, const gpo_args& a, const LaunchCtx& c) {
  if (!a.in[0] || !a.in[1] || !a.out) return GPO_BAD_ARGS;
  return run_ew_dt<kOpAdd>(k.dtype, a.in[0], a.in[1], a.out, k.shape[0], k.block_size,
                           k.num_warps, 0.f, c.stream);
}

// ------------------------------------------------------------- elementwise
// fused: one kernel, 3 streams.  unfused: scale -> add -> activation, each a
// separate launch through storage-dtype temporaries (runner.py:217-225), so
// the intermediates round exactly as the reference's three kernels do.
gpo_status plan_elementwise(const gpo_key& k, Plan& p, std::string& log) {
  gpo_status s = check_1d_key(k, log);
  if (s != GPO_OK) return s;
  if (k.dtype == GPO_TF32) {
    log = "elementwise has no tf32 variant";
    return GPO_BAD_CONFIG;
  }
  const bool gelu = k.task == GPO_TASK_FUSED_GELU;
  p.family = "bw_kernels";
  if (k.strategy == GPO_STRATEGY_FUSED) {
    fill_1d_res(k, p, gelu ? "ew_kernel<fused_gelu>" : "ew_kernel<fused_relu>", 1);
  } else if (k.strategy == GPO_STRATEGY_UNFUSED) {
    fill_1d_res(k, p, gelu ? "ew_kernel<scale,add,gelu>" : "ew_kernel<scale,add,relu>", 3);
    const uint64_t bytes = static_cast<uint64_t>(k.shape[0]) * dtype_bytes(k.dtype);
    p.res.scratch_bytes[0] = bytes;  // t1
    p.res.scratch_bytes[1] = bytes;  // t2
  } else {
    log = "strategy must be fused or unfused";
    return GPO_BAD_CONFIG;
  }
  return GPO_OK;
}

gpo_status launch_elementwise(const gpo_key& k, const Plan&, const gpo_args& a,
                              const LaunchCtx& c) {
  if (!a.in[0] || !a.in[1] || !a.out) return GPO_BAD_ARGS;
  const bool gelu = k.task == GPO_TASK_FUSED_GELU;
  const float sc = a.scale;
  const int64_t n = k.shape[0];
  if (k.strategy == GPO_STRATEGY_FUSED) {
    return gelu ? run_ew_dt<kOpFusedGelu>(k.dtype, a.in[0], a.in[1], a.out, n, k.block_size,
                                          k.num_warps, sc, c.stream)
                : run_ew_dt<kOpFusedRelu>(k.dtype, a.in[0], a.in[1], a.out, n, k.block_size,
                                          k.num_warps, sc, c.stream);
  }
  if (!a.scratch[0] || !a.scratch[1]) return GPO_BAD_ARGS;
  gpo_status s = run_ew_dt<kOpScale>(k.dtype, a.in[0], nullptr, a.scratch[0], n, k.block_size,
                                     k.num_warps, sc, c.stream);
  if (s != GPO_OK) return s;
  s = run_ew_dt<kOpAdd>(k.dtype, a.scratch[0], a.in[1], a.scratch[1], n, k.block_size,
                        k.num_warps, 0.f, c.stream);
  if (s != GPO_OK) return s;
  return gelu ? run_ew_dt<kOpGelu>(k.dtype, a.scratch[1], nullptr, a.out, n, k.block_size,
                                   k.num_warps, 0.f, c.stream)
              : run_ew_dt<kOpRelu>(k.dtype, a.scratch[1], nullptr, a.out, n, k.block_size,
                                   k.num_warps, 0.f, c.stream);
}

// --------------------------------------------------------------- reduction
// Block-level sum of per-thread fp32 partials; result valid in thread 0.
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = (blockDim.x + 31) >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < nw ? red[lane] : 0.f;
    v = warp_sum(v);
  }
  return v;
}

// Sum of one BLOCK_SIZE slice per CTA (reduce_partial_kernel /
// reduce_atomic_kernel, kernels.py:78-92).  ATOMIC: atomicAdd into dst[0];
// otherwise store into dst[blockIdx.x].
template <bool ATOMIC>
__global__ void __launch_bounds__(1024) reduce_slice_kernel(const float* __restrict__ x,
                                                            float* __restrict__ dst, int64_t n,
                                                            int64_t block_size, int vec) {
  __shared__ float red[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * block_size;
  const int64_t lim = (n - base) < block_size ? (n - base) : block_size;
  float acc = 0.f;
  int64_t done = 0;
  if (vec) {
    const int64_t nvec = lim / 4;
    const float4* xv = reinterpret_cast<const float4*>(x + base);
#pragma unroll 4
    for (int64_t i = threadIdx.x; i < nvec; i += blockDim.x) {
      const float4 v = __ldcs(xv + i);
      acc += (v.x + v.y) + (v.z + v.w);
    }
    done = nvec * 4;
  }
  for (int64_t i = done + threadIdx.x; i < lim; i += blockDim.x) acc += x[base + i];
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) {
    if constexpr (ATOMIC) {
      atomicAdd(dst, acc);
    } else {
      dst[blockIdx.x] = acc;
    }
  }
}

// Single-CTA strided accumulation over the whole array (reduce_loop_kernel,
// kernels.py:94-101).  Each thread keeps UNROLL independent float4 loads in
// flight per trip; UNROLL is BLOCK_SIZE / (threads * 4), the per-thread share
// of one BLOCK_SIZE chunk.
template <int UNROLL>
__global__ void __launch_bounds__(1024) reduce_loop_kernel(const float* __restrict__ x,
                                                           float* __restrict__ out, int64_t n,
                                                           int vec) {
  __shared__ float red[32];
  float acc[UNROLL];
#pragma unroll
  for (int u = 0; u < UNROLL; ++u) acc[u] = 0.f;
  int64_t done = 0;
  if (vec) {
    const int64_t nvec = n / 4;
    const float4* xv = reinterpret_cast<const float4*>(x);
    const int64_t T = blockDim.x;
    int64_t i = threadIdx.x;
    for (; i + (UNROLL - 1) * T < nvec; i += UNROLL * T) {
      float4 v[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) v[u] = __ldcs(xv + i + u * T);
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) acc[u] += (v[u].x + v[u].y) + (v[u].z + v[u].w);
    }
    for (; i < nvec; i += T) {
      const float4 v = __ldcs(xv + i);
      acc[0] += (v.x + v.y) + (v.z + v.w);
    }
    done = nvec * 4;
  }
  for (int64_t i = done + threadIdx.x; i < n; i += blockDim.x) acc[0] += x[i];
  float t = 0.f;
#pragma unroll
  for (int u = 0; u < UNROLL; ++u) t += acc[u];
  t = block_sum(t, red);
  if (threadIdx.x == 0) out[0] = t;
}

static int loop_unroll(int64_t bs, int threads) {
  const int64_t u = bs / (static_cast<int64_t>(threads) * 4);
  if (u >= 8) return 8;
  if (u >= 4) return 4;
  if (u >= 2) return 2;
  return 1;
}

static gpo_status run_loop(const float* x, float* out, int64_t n, int64_t bs, int warps,
                           cudaStream_t st) {
  const int threads = warps * 32;
  const int vec = aligned16(x) ? 1 : 0;
  switch (loop_unroll(bs, threads)) {
    case 8:
      reduce_loop_kernel<8><<<1, threads, 0, st>>>(x, out, n, vec);
      break;
    case 4:
      reduce_loop_kernel<4><<<1, threads, 0, st>>>(x, out, n, vec);
      break;
    case 2:
      reduce_loop_kernel<2><<<1, threads, 0, st>>>(x, out, n, vec);
      break;
    default:
      reduce_loop_kernel<1><<<1, threads, 0, st>>>(x, out, n, vec);
      break;
  }
  return launch_status();
}

gpo_status plan_reduction(const gpo_key& k, Plan& p, std::string& log) {
  gpo_status s = check_1d_key(k, log);
  if (s != GPO_OK) return s;
  if (k.dtype != GPO_FLOAT32) {
    log = "reduction is fp32 only (benchmarks/reduction/task.py:20)";
    return GPO_BAD_CONFIG;
  }
  p.family = "bw_kernels";
  const uint64_t n = static_cast<uint64_t>(k.shape[0]);
  const uint64_t nblocks = std::max<uint64_t>(1, cdiv(n, k.block_size));
  if (k.strategy == GPO_STRATEGY_LOOP) {
    fill_1d_res(k, p, "reduce_loop_kernel", 1);
    p.res.grid_x = 1;
  } else if (k.strategy == GPO_STRATEGY_ATOMIC) {
    fill_1d_res(k, p, "reduce_slice_kernel<atomic>", 2);  // memset + kernel
  } else if (k.strategy == GPO_STRATEGY_TWO_PASS) {
    fill_1d_res(k, p, "reduce_slice_kernel<partial>+reduce_loop_kernel", 2);
    p.res.scratch_bytes[0] = nblocks * sizeof(float);  // partial sums
  } else {
    log = "strategy must be loop, atomic or two_pass";
    return GPO_BAD_CONFIG;
  }
  return GPO_OK;
}

gpo_status launch_reduction(const gpo_key& k, const Plan&, const gpo_args& a,
                            const LaunchCtx& c) {
  if (!a.in[0] || !a.out) return GPO_BAD_ARGS;
  const float* x = static_cast<const float*>(a.in[0]);
  float* out = static_cast<float*>(a.out);
  const int64_t n = k.shape[0];
  const int64_t bs = k.block_size;
  const int threads = k.num_warps * 32;
  const int vec = (aligned16(x) && bs % 4 == 0) ? 1 : 0;
  if (k.strategy == GPO_STRATEGY_LOOP) return run_loop(x, out, n, bs, k.num_warps, c.stream);
  if (k.strategy == GPO_STRATEGY_ATOMIC) {
    if (cudaMemsetAsync(out, 0, sizeof(float), c.stream) != cudaSuccess) return GPO_LAUNCH_ERROR;
    if (n == 0) return GPO_OK;
    reduce_slice_kernel<true>
        <<<static_cast<unsigned>(cdiv(n, bs)), threads, 0, c.stream>>>(x, out, n, bs, vec);
    return launch_status();
  }
  // two_pass: partial sums per slice, then the loop kernel over the partials
  float* partial = static_cast<float*>(a.scratch[0]);
  if (!partial) return GPO_BAD_ARGS;
  if (n == 0) {
    if (cudaMemsetAsync(out, 0, sizeof(float), c.stream) != cudaSuccess) return GPO_LAUNCH_ERROR;
    return GPO_OK;
  }
  const int64_t nblocks = static_cast<int64_t>(cdiv(n, bs));
  reduce_slice_kernel<false>
      <<<static_cast<unsigned>(nblocks), threads, 0, c.stream>>>(x, partial, n, bs, vec);
  gpo_status s = launch_status();
  if (s != GPO_OK) return s;
  return run_loop(partial, out, nblocks, bs, k.num_warps, c.stream);
}

// ------------------------------------------------------------- self-test
// One thread waits, with a short bounded limit, on an mbarrier that nothing
// arrives on; the wait gives up, records kErrSelfTest in the error word and
// the kernel returns.  Exercises the device-timeout reporting path without
// any fault.
__global__ void selftest_timeout_kernel(unsigned int* err, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    fence_barrier_init();
    mbar_wait_for(smem_u32(&bar), 0, err, kErrSelfTest, limit_ns);
  }
}

gpo_status launch_selftest_timeout(const LaunchCtx& c, unsigned long long limit_ns) {
  selftest_timeout_kernel<<<1, 32, 0, c.stream>>>(c.err, limit_ns);
  return launch_status();
}

// ------------------------------------------------- allocation-free two_pass
// Some callers cannot allocate device memory at the point where they need a
// sum: plug-in hosts that own all device memory and hand this library only
// input and output buffers (an allocation would escape the host's
// accounting and can fail under its memory cap), and latency-critical
// callers that cannot take the device synchronisation a cudaMalloc /
// cudaFree pair can cause.  For them gpo_reduction_sum_noalloc runs the
// two_pass reduction with its partial sums in the fixed array below instead
// of a caller buffer.
//
// The array is part of the library image: every GPU that loads the library
// holds it (256 KiB) until the process exits.  All calls on a device share
// it, so calls whose kernels overlap on the GPU (different streams, no
// ordering between them) race on it; calls on one stream are ordered.
// Each call writes every partial it later reads, so nothing needs clearing;
// the array keeps whatever the last call left.
constexpr int64_t kNoAllocMaxPartials = 65536;
static __device__ __align__(256) float g_noalloc_partials[kNoAllocMaxPartials];

namespace {
constexpr int kNoAllocDevices = 64;
// The array's address belongs to one context of the device: the cache
// entry records that context and is looked up again when the device's
// current context differs (a context recreated after cudaDeviceReset maps
// the library image afresh).
struct NoAllocSlot {
  void* ctx;
  float* ptr;
};
std::mutex g_noalloc_mu;
NoAllocSlot g_noalloc[kNoAllocDevices] = {};

using CtxGetCurrentFn = int (*)(void**);  // cuCtxGetCurrent(CUcontext*)

// The calling thread's current context, or nullptr when none is current or
// the driver entry point is unavailable (the address is then looked up on
// every call).
void* current_context() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    void* f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(f);
  });
  void* ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != 0) return nullptr;
  return ctx;
}
}  // namespace

// Device address of g_noalloc_partials on the current device.  In host code
// the array's name is only a host-side stand-in, so the address is resolved
// with the device current: once per device and context.
static gpo_status noalloc_scratch(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return GPO_NO_DEVICE;
  }
  if (dev < 0 || dev >= kNoAllocDevices) return GPO_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocSlot& slot = g_noalloc[dev];
  void* ctx = current_context();
  if (slot.ptr == nullptr || ctx == nullptr || ctx != slot.ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_partials);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      return GPO_LAUNCH_ERROR;
    }
    slot.ptr = static_cast<float*>(p);
    slot.ctx = current_context();  // current now, if it was not before
  }
  *out = slot.ptr;
  return GPO_OK;
}

}  // namespace gpo

extern "C" gpo_status gpo_reduction_sum_noalloc(const float* x, int64_t n, float* out,
                                                int32_t block_size, int32_t num_warps,
                                                void* stream) {
  using namespace gpo;
  if (!x || !out || n < 0 || block_size < 1 || block_size > (1 << 20) || num_warps < 1 ||
      num_warps > 32)
    return GPO_BAD_ARGS;
  const int64_t nblocks = n == 0 ? 0 : static_cast<int64_t>(cdiv(n, block_size));
  if (nblocks > kNoAllocMaxPartials) return GPO_BAD_ARGS;  // n > 65536 * block_size
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    return cudaMemsetAsync(out, 0, sizeof(float), st) == cudaSuccess ? GPO_OK
                                                                       : GPO_LAUNCH_ERROR;
  }
  float* partial = nullptr;
  gpo_status s = noalloc_scratch(&partial);
  if (s != GPO_OK) return s;
  const int vec = (aligned16(x) && block_size % 4 == 0) ? 1 : 0;
  reduce_slice_kernel<false><<<static_cast<unsigned>(nblocks), num_warps * 32, 0, st>>>(
      x, partial, n, block_size, vec);
  s = launch_status();
  if (s != GPO_OK) return s;
  return run_loop(partial, out, nblocks, block_size, num_warps, st);
}

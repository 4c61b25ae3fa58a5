/*
 * gpo.h — C ABI of the B200 (sm_100a) kernel backend for the gpu-optimizer
 * autotuning agent.
 *
 * The reference launches every candidate as a parameterised Triton kernel
 * through compiler/triton/runner.py.  This library replaces the layer below
 * that Python API: one candidate configuration (task, shape, BLOCK_*,
 * GROUP_M, num_warps, num_stages, dtype, strategy) selects one template
 * instantiation of a hand-written CUDA kernel family, and resource overflow
 * (shared memory, TMEM columns, register tile) is reported as a compile
 * failure exactly where Triton would raise OutOfResources.
 *
 * Conventions
 *  - Plain C types only: device pointers as void*, sizes as int64_t, the CUDA
 *    stream as an opaque void* (a cudaStream_t / CUstream handle, or NULL for
 *    the legacy default stream).
 *  - Nothing throws across the ABI; every function returns a gpo_status.
 *  - gpo_compile is pure host logic (no CUDA call), so configuration
 *    validation works on machines without a GPU.
 *  - gpo_launch never allocates device memory for the caller's data: outputs
 *    and scratch buffers (sizes from gpo_query) are passed in by the caller,
 *    as the reference runner allocates them at build time
 *    (compiler/triton/runner.py:101,122,137,151,172,191,209,218-219,239).
 *    The library keeps one 256-byte device error word per device, allocated
 *    on the first launch on that device.
 *  - Modules are immutable after gpo_compile and may be shared by host
 *    threads; launches on different streams may run concurrently.  The
 *    persistent two-tile attention kernel (BLOCK_M 256, num_warps 8) takes
 *    its work items from one of 64 counters in the library, chosen per
 *    launch in turn: at most 64 of its launches may overlap on one device,
 *    and replays of one captured graph must not overlap each other.
 */
#ifndef GPO_H_
#define GPO_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GPO_ABI_VERSION 1

#if defined(__GNUC__)
#define GPO_API __attribute__((visibility("default")))
#else
#define GPO_API
#endif

/* Status codes.  GPO_COMPILE_ERROR maps to the reference's compile_error
 * status (benchmarks/harness.py:34,169-173).  GPO_LAUNCH_ERROR on a
 * candidate's first launch (warm_compile) is compile_error too, as the
 * reference's first-launch failures are (compiler/triton/runner.py:75-89);
 * after it, runtime_error.  GPO_TIMEOUT is always runtime_error
 * (benchmarks/harness.py:35,182-184): a wait that gave up says nothing about
 * whether the candidate compiles. */
typedef enum gpo_status {
  GPO_OK = 0,
  GPO_COMPILE_ERROR = 1, /* a real resource limit is exceeded; log says which */
  GPO_BAD_CONFIG = 2,    /* parameter value outside every template family     */
  GPO_BAD_ARGS = 3,      /* null/misaligned pointer, bad shape or stride      */
  GPO_LAUNCH_ERROR = 4,  /* the CUDA runtime rejected the launch              */
  GPO_TIMEOUT = 5,       /* a bounded device-side wait gave up                */
  GPO_NO_DEVICE = 6,     /* no sm_100 device visible                          */
  GPO_INTERNAL = 7
} gpo_status;

/* Task ids: the reference task registry (benchmarks/__init__.py:14-25) plus
 * the two B200 workload variants registered as separate tasks so that the
 * reference tasks' candidate ids stay stable. */
typedef enum gpo_task {
  GPO_TASK_MATMUL = 0,            /* benchmarks/matmul/task.py:16            */
  GPO_TASK_VECADD = 1,            /* benchmarks/vecadd/task.py:16            */
  GPO_TASK_REDUCTION = 2,         /* benchmarks/reduction/task.py:18         */
  GPO_TASK_SOFTMAX = 3,           /* benchmarks/softmax/task.py:16           */
  GPO_TASK_LAYERNORM = 4,         /* benchmarks/layernorm/task.py:18         */
  GPO_TASK_FUSED_ELEMENTWISE = 5, /* benchmarks/fused_elementwise/task.py:22 */
  GPO_TASK_ATTENTION = 6,         /* benchmarks/attention/task.py:24         */
  GPO_TASK_ATTENTION_CAUSAL = 7,  /* causal variant of the attention task    */
  GPO_TASK_FUSED_GELU = 8         /* y = gelu(x*w + b), fused_elementwise layout */
} gpo_task;

/* Storage/compute dtype: benchmarks/base.py:24-29. */
typedef enum gpo_dtype {
  GPO_FLOAT32 = 0,
  GPO_TF32 = 1, /* fp32 storage, tf32 tensor-core math */
  GPO_FLOAT16 = 2,
  GPO_BFLOAT16 = 3
} gpo_dtype;

/* Strategy parameter: reduction (benchmarks/reduction/task.py:44) and
 * fused_elementwise (benchmarks/fused_elementwise/task.py:53). */
typedef enum gpo_strategy {
  GPO_STRATEGY_NONE = 0,
  GPO_STRATEGY_LOOP = 1,
  GPO_STRATEGY_ATOMIC = 2,
  GPO_STRATEGY_TWO_PASS = 3,
  GPO_STRATEGY_FUSED = 4,
  GPO_STRATEGY_UNFUSED = 5
} gpo_strategy;

/* One candidate = one instantiation key.  Mirrors the config dict of
 * compiler/transformations/space.py:23-24 (Config) for the task and shape of
 * a Candidate (space.py:171-191).  Parameters a task does not use are 0.
 * shape: matmul (M, N, K); vecadd / reduction / fused (n); softmax and
 * layernorm (M, N); attention (BH, S, D). */
typedef struct gpo_key {
  int32_t task;     /* gpo_task */
  int32_t dtype;    /* gpo_dtype */
  int32_t strategy; /* gpo_strategy */
  int32_t block_m, block_n, block_k, block_size;
  int32_t group_m, num_warps, num_stages;
  int32_t ndim;
  int64_t shape[4];
} gpo_key;

/* What a compiled module needs; filled by gpo_query. */
typedef struct gpo_resources {
  uint32_t smem_bytes;        /* dynamic + static shared memory per CTA     */
  uint32_t tmem_cols;         /* TMEM columns allocated per CTA (0: none)   */
  uint32_t threads_per_cta;
  uint32_t grid_x, grid_y, grid_z; /* grid of the main kernel             */
  uint32_t launches_per_call; /* kernels (+ memsets) one gpo_launch issues  */
  uint32_t persistent;        /* 1: grid sized to the SM count              */
  uint64_t scratch_bytes[2];  /* caller-allocated scratch buffers           */
  char kernel[96];            /* kernel family / instantiation name         */
} gpo_resources;

/* Launch arguments: device pointers.  `in` in task order (matmul a,b;
 * vecadd x,y; reduction x; softmax x; layernorm x,w,b; fused x,bias;
 * attention q,k,v).  All tensors are dense row-major (contiguous). */
typedef struct gpo_args {
  const void* in[4];
  void* out;
  void* scratch[2];
  float scale; /* fused elementwise scale; 0 selects the task default */
  float eps;   /* layernorm epsilon; 0 selects the task default 1e-5  */
} gpo_args;

typedef struct gpo_module gpo_module;

/* ABI version of the loaded library (GPO_ABI_VERSION at build time). */
GPO_API int gpo_abi_version(void);

/* Select and validate the template instantiation for `key`.
 * Replaces Triton's JIT compile step, surfaced by the reference at
 * compiler/triton/runner.py:75-89 (warm_compile) and :52-72
 * (build_callable's KernelBuildError).  On GPO_COMPILE_ERROR /
 * GPO_BAD_CONFIG a human-readable reason is written to `log`.  No CUDA
 * call is made. */
GPO_API gpo_status gpo_compile(const gpo_key* key, gpo_module** out, char* log, size_t log_cap);

/* Resources of a compiled module (replaces the launch dict of
 * compiler/triton/runner.py:31-37, 115 and the smem estimate of
 * compiler/transformations/constraints.py:21-38). */
GPO_API gpo_status gpo_query(const gpo_module* mod, gpo_resources* res);

/* Enqueue one execution of the candidate on `stream` (the call the
 * reference makes as K.<kernel>[grid](...) inside fn(),
 * compiler/triton/runner.py:104-113,125-127,139-158,174-178,193-197,
 * 212-225,242-254).  Asynchronous; device-side timeouts are reported by
 * gpo_device_status. */
GPO_API gpo_status gpo_launch(gpo_module* mod, const gpo_args* args, void* stream);

/* Read and clear the error word of the current device after synchronising
 * `stream`.  *flags receives the site bits of any bounded wait that gave up
 * (0 when none).  Returns GPO_TIMEOUT when flags != 0. */
GPO_API gpo_status gpo_device_status(void* stream, uint32_t* flags);

/* Diagnostics for the failure-detection path: launch one CTA whose thread
 * waits, with a bounded limit of `limit_ms` (1..2000), on an mbarrier that
 * nothing arrives on, then read the error word as gpo_device_status does.
 * Expected result: GPO_TIMEOUT with the self-test bit (1 << 6) in *flags.
 * No counterpart in the reference, whose harness has no device timeouts
 * (benchmarks/harness.py:144-203). */
GPO_API gpo_status gpo_selftest_timeout(void* stream, uint32_t limit_ms, uint32_t* flags);

/* Sum of n fp32 values with the two_pass algorithm (per-slice partial sums,
 * then one CTA summing the partials), without allocating anything: the
 * partial sums live in a fixed 65536-float array inside the library, so a
 * caller that cannot allocate device memory passes just x (device, n
 * floats), out (device, one float), BLOCK_SIZE and num_warps.  Such callers
 * are plug-in hosts that own all device memory and give a kernel library
 * only its input and output buffers (an allocation escapes the host's
 * accounting and can fail under its memory cap), and latency-critical
 * callers that cannot accept the device synchronisation a cudaMalloc /
 * cudaFree pair can cause.  Same kernels and numerics as the two_pass
 * strategy of gpo_launch.
 *  - Limit: cdiv(n, block_size) <= 65536, i.e. n <= 65536 * block_size;
 *    larger n returns GPO_BAD_ARGS before anything is launched.
 *  - The first call on a device (and the first after that device's context
 *    is recreated, e.g. by cudaDeviceReset) looks up the array's device
 *    address; make that first call before any stream capture.
 *  - All calls on a device share the array: calls whose kernels may overlap
 *    on the GPU (unordered streams) race; calls on one stream do not.
 *  - No cudaMalloc, cudaFree or other allocation is made by this call.
 * No counterpart in the reference, whose runner allocates the partials with
 * torch at build time. */
GPO_API gpo_status gpo_reduction_sum_noalloc(const float* x, int64_t n, float* out,
                                             int32_t block_size, int32_t num_warps,
                                             void* stream);

/* Free a module. */
GPO_API void gpo_destroy(gpo_module* mod);

/* CUDA source of the kernel family a module instantiates, followed by the
 * resolved configuration (replaces compiler/triton/runner.py:275-297,
 * render_source).  Works without a GPU.  The returned string lives as long
 * as the module. */
GPO_API const char* gpo_source(const gpo_module* mod);

/* Name of a status code. */
GPO_API const char* gpo_status_name(gpo_status s);

#ifdef __cplusplus
}
#endif

#endif /* GPO_H_ */

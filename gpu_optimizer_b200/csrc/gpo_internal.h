// Internal interface between the C-ABI front end (abi.cu) and the kernel
// families.  Each family exposes a `plan_*` function (pure host logic: picks
// the instantiation and fills the resource record, or reports why the config
// cannot be built) and a `launch_*` function (enqueues the kernels).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/gpo.h"

namespace gpo {

constexpr uint32_t kMaxSmemPerCta = 227 * 1024;  // sm_100 opt-in limit
constexpr uint32_t kTmemCols = 512;

// Everything a family needs at launch time.
struct LaunchCtx {
  cudaStream_t stream;
  unsigned int* err;  // per-device error word
  int device;
  int sm_count;
};

// Host-side plan of one instantiation.
struct Plan {
  gpo_resources res{};
  int variant = 0;       // family-specific instantiation index
  int aux[8] = {0};      // family-specific resolved parameters
  std::string family;    // source family name (for gpo_source)
};

// Returns GPO_OK or GPO_COMPILE_ERROR / GPO_BAD_CONFIG with a reason in *log.
typedef gpo_status (*PlanFn)(const gpo_key&, Plan&, std::string& log);
typedef gpo_status (*LaunchFn)(const gpo_key&, const Plan&, const gpo_args&, const LaunchCtx&);

// bandwidth-bound families (bw_kernels.cu)
gpo_status plan_vecadd(const gpo_key&, Plan&, std::string&);
gpo_status launch_vecadd(const gpo_key&, const Plan&, const gpo_args&, const LaunchCtx&);
gpo_status plan_elementwise(const gpo_key&, Plan&, std::string&);
gpo_status launch_elementwise(const gpo_key&, const Plan&, const gpo_args&, const LaunchCtx&);
gpo_status plan_reduction(const gpo_key&, Plan&, std::string&);
gpo_status launch_reduction(const gpo_key&, const Plan&, const gpo_args&, const LaunchCtx&);

gpo_status launch_selftest_timeout(const LaunchCtx&, unsigned long long limit_ns);

// row-wise families (row_kernels.cu)
gpo_status plan_softmax(const gpo_key&, Plan&, std::string&);
gpo_status launch_softmax(const gpo_key&, const Plan&, const gpo_args&, const LaunchCtx&);
gpo_status plan_layernorm(const gpo_key&, Plan&, std::string&);
gpo_status launch_layernorm(const gpo_key&, const Plan&, const gpo_args&, const LaunchCtx&);

// contractions (matmul_tc.cu, matmul_simt.cu, attn_tc.cu, attn_simt.cu)
gpo_status plan_matmul(const gpo_key&, Plan&, std::string&);
gpo_status launch_matmul(const gpo_key&, const Plan&, const gpo_args&, const LaunchCtx&);
gpo_status plan_matmul_tc(const gpo_key&, Plan&, std::string&);
gpo_status launch_matmul_tc(const gpo_key&, const Plan&, const gpo_args&, const LaunchCtx&);
gpo_status plan_matmul_simt(const gpo_key&, Plan&, std::string&);
gpo_status launch_matmul_simt(const gpo_key&, const Plan&, const gpo_args&, const LaunchCtx&);
gpo_status plan_attention(const gpo_key&, Plan&, std::string&);
gpo_status launch_attention(const gpo_key&, const Plan&, const gpo_args&, const LaunchCtx&);
gpo_status plan_attention_tc(const gpo_key&, Plan&, std::string&);
gpo_status launch_attention_tc(const gpo_key&, const Plan&, const gpo_args&, const LaunchCtx&);
gpo_status plan_attention_simt(const gpo_key&, Plan&, std::string&);
gpo_status launch_attention_simt(const gpo_key&, const Plan&, const gpo_args&, const LaunchCtx&);

// Element size of a storage dtype.
inline int dtype_bytes(int dt) { return (dt == GPO_FLOAT16 || dt == GPO_BFLOAT16) ? 2 : 4; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline uint64_t cdiv(uint64_t a, uint64_t b) { return (a + b - 1) / b; }

// Map a CUDA runtime error after a launch to a status.
inline gpo_status launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GPO_OK : GPO_LAUNCH_ERROR;
}

// Set the dynamic shared memory opt-in of a kernel once per device.
gpo_status ensure_smem_attr(const void* func, uint32_t dyn_smem);

// Grid of a persistent kernel: SM count x resident CTAs per SM (occupancy
// of `func` at `threads` / `dyn_smem`, cached), at most `work_items`.
unsigned persistent_grid(const void* func, int threads, size_t dyn_smem, int sm_count,
                         int64_t work_items);

// Driver entry point for cuTensorMapEncodeTiled, resolved once.
void* tensor_map_encoder();

}  // namespace gpo

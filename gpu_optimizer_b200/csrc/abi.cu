// C-ABI front end of libgpo.so: configuration -> plan (pure host logic),
// launch dispatch, per-device error word, embedded kernel sources.
// Declarations and the reference interface each entry point replaces are in
// include/gpo.h.
#include <algorithm>
#include <cstring>
#include <map>
#include <tuple>
#include <mutex>
#include <string>
#include <utility>

#include "gpo_internal.h"

struct gpo_module {
  gpo_key key;
  gpo::Plan plan;
  std::string source;
};

namespace gpo {

namespace {

// Embedded CUDA sources, one entry per kernel family (generated at build
// time from the .cu files of this directory).
#include "gpo_sources.inc"

constexpr int kMaxDevices = 64;

struct DeviceState {
  bool ready = false;
  unsigned int* err = nullptr;
  int sm_count = 0;
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];
std::map<std::pair<const void*, int>, uint32_t> g_smem_attr;

gpo_status device_state(int dev, DeviceState** out) {
  if (dev < 0 || dev >= kMaxDevices) return GPO_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& d = g_dev[dev];
  if (!d.ready) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        major != 10)
      return GPO_NO_DEVICE;
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return GPO_NO_DEVICE;
    void* p = nullptr;
    if (cudaMalloc(&p, 256) != cudaSuccess) return GPO_INTERNAL;
    if (cudaMemset(p, 0, 256) != cudaSuccess) return GPO_INTERNAL;
    d.err = static_cast<unsigned int*>(p);
    d.ready = true;
  }
  *out = &d;
  return GPO_OK;
}

PlanFn plan_for(int task) {
  switch (task) {
    case GPO_TASK_MATMUL: return plan_matmul;
    case GPO_TASK_VECADD: return plan_vecadd;
    case GPO_TASK_REDUCTION: return plan_reduction;
    case GPO_TASK_SOFTMAX: return plan_softmax;
    case GPO_TASK_LAYERNORM: return plan_layernorm;
    case GPO_TASK_FUSED_ELEMENTWISE:
    case GPO_TASK_FUSED_GELU: return plan_elementwise;
    case GPO_TASK_ATTENTION:
    case GPO_TASK_ATTENTION_CAUSAL: return plan_attention;
    default: return nullptr;
  }
}

LaunchFn launch_for(int task) {
  switch (task) {
    case GPO_TASK_MATMUL: return launch_matmul;
    case GPO_TASK_VECADD: return launch_vecadd;
    case GPO_TASK_REDUCTION: return launch_reduction;
    case GPO_TASK_SOFTMAX: return launch_softmax;
    case GPO_TASK_LAYERNORM: return launch_layernorm;
    case GPO_TASK_FUSED_ELEMENTWISE:
    case GPO_TASK_FUSED_GELU: return launch_elementwise;
    case GPO_TASK_ATTENTION:
    case GPO_TASK_ATTENTION_CAUSAL: return launch_attention;
    default: return nullptr;
  }
}

const char* family_source(const std::string& family) {
  for (const auto& e : kSources)
    if (family == e.name) return e.text;
  return nullptr;
}

void write_log(char* log, size_t cap, const std::string& msg) {
  if (!log || cap == 0) return;
  const size_t n = msg.size() < cap - 1 ? msg.size() : cap - 1;
  std::memcpy(log, msg.data(), n);
  log[n] = '\0';
}

}  // namespace

gpo_status ensure_smem_attr(const void* func, uint32_t dyn_smem) {
  if (dyn_smem <= 48u * 1024u) return GPO_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GPO_NO_DEVICE;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_smem_attr.find({func, dev});
    if (it != g_smem_attr.end() && it->second >= dyn_smem) return GPO_OK;
  }
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(dyn_smem)) != cudaSuccess) {
    cudaGetLastError();
    return GPO_LAUNCH_ERROR;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  uint32_t& v = g_smem_attr[{func, dev}];
  if (v < dyn_smem) v = dyn_smem;
  return GPO_OK;
}

unsigned persistent_grid(const void* func, int threads, size_t dyn_smem, int sm_count,
                         int64_t work_items) {
  static std::mutex mu;
  // keyed by shared memory too: one kernel runs with different stage counts
  static std::map<std::tuple<const void*, int, size_t>, int> occ;
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = occ.find({func, threads, dyn_smem});
    if (it != occ.end()) per_sm = it->second;
  }
  if (per_sm == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, func, threads, dyn_smem) !=
            cudaSuccess ||
        per_sm < 1) {
      cudaGetLastError();
      per_sm = 1;
    }
    std::lock_guard<std::mutex> lk(mu);
    occ[{func, threads, dyn_smem}] = per_sm;
  }
  const int64_t g = static_cast<int64_t>(per_sm) * (sm_count > 0 ? sm_count : 148);
  return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(g, work_items)));
}

void* tensor_map_encoder() {
  static void* fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    void* f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = f;
  });
  return fn;
}

}  // namespace gpo

extern "C" {

int gpo_abi_version(void) { return GPO_ABI_VERSION; }

const char* gpo_status_name(gpo_status s) {
  switch (s) {
    case GPO_OK: return "GPO_OK";
    case GPO_COMPILE_ERROR: return "GPO_COMPILE_ERROR";
    case GPO_BAD_CONFIG: return "GPO_BAD_CONFIG";
    case GPO_BAD_ARGS: return "GPO_BAD_ARGS";
    case GPO_LAUNCH_ERROR: return "GPO_LAUNCH_ERROR";
    case GPO_TIMEOUT: return "GPO_TIMEOUT";
    case GPO_NO_DEVICE: return "GPO_NO_DEVICE";
    case GPO_INTERNAL: return "GPO_INTERNAL";
  }
  return "GPO_UNKNOWN";
}

gpo_status gpo_compile(const gpo_key* key, gpo_module** out, char* log, size_t log_cap) {
  if (!key || !out) return GPO_BAD_ARGS;
  *out = nullptr;
  gpo::PlanFn plan = gpo::plan_for(key->task);
  if (!plan) {
    gpo::write_log(log, log_cap, "no kernel family for task id " + std::to_string(key->task));
    return GPO_BAD_CONFIG;
  }
  if (key->dtype < GPO_FLOAT32 || key->dtype > GPO_BFLOAT16) {
    gpo::write_log(log, log_cap, "unknown dtype id " + std::to_string(key->dtype));
    return GPO_BAD_CONFIG;
  }
  gpo_module* m = new (std::nothrow) gpo_module();
  if (!m) return GPO_INTERNAL;
  m->key = *key;
  std::string msg;
  gpo_status s;
  try {
    s = plan(*key, m->plan, msg);
  } catch (...) {
    s = GPO_INTERNAL;
    msg = "internal error while planning";
  }
  if (s != GPO_OK) {
    gpo::write_log(log, log_cap, msg);
    delete m;
    return s;
  }
  gpo::write_log(log, log_cap, "");
  *out = m;
  return GPO_OK;
}

gpo_status gpo_query(const gpo_module* mod, gpo_resources* res) {
  if (!mod || !res) return GPO_BAD_ARGS;
  *res = mod->plan.res;
  return GPO_OK;
}

gpo_status gpo_launch(gpo_module* mod, const gpo_args* args, void* stream) {
  if (!mod || !args) return GPO_BAD_ARGS;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return GPO_NO_DEVICE;
  }
  gpo::DeviceState* ds = nullptr;
  gpo_status s = gpo::device_state(dev, &ds);
  if (s != GPO_OK) return s;
  gpo::LaunchCtx ctx{static_cast<cudaStream_t>(stream), ds->err, dev, ds->sm_count};
  gpo_args a = *args;
  if (a.scale == 0.f) a.scale = 0.7071f;  // benchmarks/fused_elementwise/task.py:19
  if (a.eps == 0.f) a.eps = 1e-5f;        // benchmarks/layernorm/task.py:15
  gpo::LaunchFn fn = gpo::launch_for(mod->key.task);
  if (!fn) return GPO_BAD_CONFIG;
  try {
    return fn(mod->key, mod->plan, a, ctx);
  } catch (...) {
    return GPO_INTERNAL;
  }
}

gpo_status gpo_device_status(void* stream, uint32_t* flags) {
  if (flags) *flags = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GPO_NO_DEVICE;
  gpo::DeviceState* ds = nullptr;
  gpo_status s = gpo::device_state(dev, &ds);
  if (s != GPO_OK) return s;
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) {
    cudaGetLastError();
    return GPO_LAUNCH_ERROR;
  }
  uint32_t v = 0;
  if (cudaMemcpy(&v, ds->err, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess)
    return GPO_LAUNCH_ERROR;
  if (v != 0) cudaMemset(ds->err, 0, sizeof(v));
  if (flags) *flags = v;
  return v ? GPO_TIMEOUT : GPO_OK;
}

gpo_status gpo_selftest_timeout(void* stream, uint32_t limit_ms, uint32_t* flags) {
  if (flags) *flags = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GPO_NO_DEVICE;
  gpo::DeviceState* ds = nullptr;
  gpo_status s = gpo::device_state(dev, &ds);
  if (s != GPO_OK) return s;
  if (limit_ms == 0 || limit_ms > 2000) return GPO_BAD_ARGS;
  gpo::LaunchCtx ctx{static_cast<cudaStream_t>(stream), ds->err, dev, ds->sm_count};
  s = gpo::launch_selftest_timeout(ctx, static_cast<unsigned long long>(limit_ms) * 1000000ull);
  if (s != GPO_OK) return s;
  return gpo_device_status(stream, flags);
}

void gpo_destroy(gpo_module* mod) { delete mod; }

const char* gpo_source(const gpo_module* mod) {
  if (!mod) return nullptr;
  gpo_module* m = const_cast<gpo_module*>(mod);
  if (m->source.empty()) {
    const gpo_key& k = m->key;
    std::string hdr = "// kernel family: " + m->plan.family + "\n";
    hdr += "// instantiation: " + std::string(m->plan.res.kernel) + "\n";
    hdr += "// resolved configuration:\n";
    hdr += "//   task = " + std::to_string(k.task) + ", dtype = " + std::to_string(k.dtype) +
           ", strategy = " + std::to_string(k.strategy) + "\n";
    hdr += "//   BLOCK_M = " + std::to_string(k.block_m) +
           ", BLOCK_N = " + std::to_string(k.block_n) +
           ", BLOCK_K = " + std::to_string(k.block_k) +
           ", BLOCK_SIZE = " + std::to_string(k.block_size) + "\n";
    hdr += "//   GROUP_M = " + std::to_string(k.group_m) +
           ", num_warps = " + std::to_string(k.num_warps) +
           ", num_stages = " + std::to_string(k.num_stages) + "\n";
    hdr += "//   smem = " + std::to_string(m->plan.res.smem_bytes) +
           " B, tmem_cols = " + std::to_string(m->plan.res.tmem_cols) +
           ", threads = " + std::to_string(m->plan.res.threads_per_cta) + "\n\n";
    const char* src = gpo::family_source(m->plan.family);
    m->source = hdr + (src ? src : "// source not embedded\n");
    // the PTX wrappers (mbarrier, TMA, tcgen05) every family builds on
    const char* common = gpo::family_source("gpo_common");
    if (common) m->source += std::string("\n// ---- gpo_common.cuh ----\n") + common;
  }
  return m->source.c_str();
}

}  // extern "C"

// Host-side launch plumbing and the small C-ABI entry points that launch no kernel.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "host_common.h"

namespace svllm::k {

// The library's own device error word; callers that pass no err pointer read it back with
// svllm_read_device_error.
__device__ int g_library_error_word = 0;

namespace {

std::atomic<int> g_sm_count[kMaxDevices];
std::atomic<int*> g_error_word[kMaxDevices];

// Target bytes per stage, stages per warp, warps per CTA (the occupancy calculator then packs
// as many CTAs per SM as shared memory and registers allow). Chosen by sweeping each op on a
// B200 at 1M tokens of the Qwen3-0.6B shapes: the streaming ops want (stages - 1) * unit bytes *
// resident warps of loads in flight per SM well above the ~45 KB that 6.5 TB/s over 148 SMs
// needs at ~1 us of memory latency; the compute-heavier ops (SiLU, q/k norm + RoPE) also want
// many resident warps to hide their latency chains.
constexpr PipelineShape kDefaultShapes[static_cast<int>(OpId::kCount)] = {
    {8192, 2, 8},   // rms_norm
    {4096, 4, 8},   // add_rms_norm
    {4096, 2, 16},  // qk_norm_rope (a unit is one token; unit_bytes is unused)
    {4096, 3, 10},  // rope
    {8192, 2, 6},   // silu_and_mul (the table path leaves ~99 KB of shared memory for stages)
    {4096, 6, 8},   // embedding (a unit is one row; unit_bytes is unused)
};

const char* const kOpNames[] = {"rms_norm", "add_rms_norm", "qk_norm_rope",
                                "rope",     "silu_and_mul", "embedding"};

// Occupancy per (kernel, block size, dynamic shared memory, device), and the kernels whose
// shared-memory limit is raised on each device: looked up on every launch, so hashed.
struct OccKey {
  const void* func;
  int threads;
  size_t smem;
  int device;
  bool operator==(const OccKey& o) const {
    return func == o.func && threads == o.threads && smem == o.smem && device == o.device;
  }
};

struct OccKeyHash {
  size_t operator()(const OccKey& k) const {
    size_t h = std::hash<const void*>()(k.func);
    h = h * 1000003u ^ std::hash<int>()(k.threads);
    h = h * 1000003u ^ std::hash<size_t>()(k.smem);
    return h * 1000003u ^ std::hash<int>()(k.device);
  }
};

std::mutex g_occ_mutex;
std::unordered_map<OccKey, int, OccKeyHash> g_occ;
std::unordered_map<OccKey, bool, OccKeyHash> g_attr;  // keyed by (func, device) only

// The shapes in force: the defaults, with the overrides of the SVLLM_PIPELINE environment
// variable applied once, on first use, and never changed afterwards (so the C ABI has no mutable
// launch state). The variable is a tuning and test hook: "op=unit_bytes:stages:warps[,op=...]",
// 0 keeping a default; entries that do not parse or are out of range are ignored. Results do not
// depend on the shape.
const PipelineShape* shapes_in_force() {
  static PipelineShape shapes[static_cast<int>(OpId::kCount)];
  static std::once_flag once;
  std::call_once(once, [] {
    std::memcpy(shapes, kDefaultShapes, sizeof(shapes));
    const char* env = std::getenv("SVLLM_PIPELINE");
    if (env == nullptr) return;
    const std::string spec(env);
    size_t pos = 0;
    while (pos <= spec.size()) {
      const size_t end = std::min(spec.find(',', pos), spec.size());
      const std::string item = spec.substr(pos, end - pos);
      pos = end + 1;
      const size_t eq = item.find('=');
      if (eq == std::string::npos) continue;
      long long unit = -1, stages = -1, warps = -1;
      if (std::sscanf(item.c_str() + eq + 1, "%lld:%lld:%lld", &unit, &stages, &warps) != 3 ||
          unit < 0 || stages < 0 || warps < 0 || unit > (1 << 20) || unit % 16 != 0 ||
          stages > 16 || warps > kMaxBulkWarps || (stages != 0 && stages < 2)) {
        continue;
      }
      for (int i = 0; i < static_cast<int>(OpId::kCount); ++i) {
        if (item.compare(0, eq, kOpNames[i]) == 0 && std::strlen(kOpNames[i]) == eq) {
          if (unit) shapes[i].unit_bytes = static_cast<int>(unit);
          if (stages) shapes[i].stages = static_cast<int>(stages);
          if (warps) shapes[i].warps = static_cast<int>(warps);
        }
      }
    }
  });
  return shapes;
}

}  // namespace

PipelineShape pipeline_shape(OpId op) { return shapes_in_force()[static_cast<int>(op)]; }

int current_device(int* device) {
  return cudaGetDevice(device) == cudaSuccess && *device >= 0 && *device < kMaxDevices
             ? SVLLM_OK
             : SVLLM_ERR_CUDA;
}

int sm_count(int device) {
  int n = g_sm_count[device].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        n <= 0) {
      n = 1;
    }
    g_sm_count[device].store(n, std::memory_order_relaxed);
  }
  return n;
}

int blocks_per_sm(const void* func, int threads, size_t smem_bytes, int device) {
  const std::lock_guard<std::mutex> lock(g_occ_mutex);
  const OccKey key{func, threads, smem_bytes, device};
  const auto hit = g_occ.find(key);
  if (hit != g_occ.end()) return hit->second;
  const OccKey attr_key{func, 0, 0, device};
  if (g_attr.find(attr_key) == g_attr.end()) {
    // the dynamic limit is what the CTA's static shared memory leaves of the per-CTA maximum
    cudaFuncAttributes attrs{};
    if (cudaFuncGetAttributes(&attrs, func) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    const size_t dynamic_max = kMaxSmemPerCta > attrs.sharedSizeBytes
                                   ? kMaxSmemPerCta - attrs.sharedSizeBytes
                                   : 0;
    if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(dynamic_max)) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    g_attr.emplace(attr_key, true);
  }
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, func, threads, smem_bytes) !=
      cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  g_occ.emplace(key, blocks);
  return blocks;
}

int* library_error_word(int device) {
  int* p = g_error_word[device].load(std::memory_order_acquire);
  if (p == nullptr) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_library_error_word) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    p = static_cast<int*>(addr);
    g_error_word[device].store(p, std::memory_order_release);
  }
  return p;
}

}  // namespace svllm::k

using namespace svllm::k;

extern "C" {

const char* svllm_status_string(int status) {
  switch (status) {
    case SVLLM_OK:
      return "ok";
    case SVLLM_ERR_INVALID_ARGUMENT:
      return "invalid argument (null pointer, size, stride, alignment or dtype)";
    case SVLLM_ERR_TOO_LARGE:
      return "sizes exceed the kernel's index range";
    case SVLLM_ERR_UNSUPPORTED:
      return "no kernel for this shape";
    case SVLLM_ERR_LAUNCH:
      return "kernel launch failed";
    case SVLLM_ERR_CUDA:
      return "CUDA runtime call failed";
    default:
      return "unknown status";
  }
}

const char* svllm_version(void) { return "0.1.0"; }

int svllm_read_device_error(int device, int reset, int* flags) {
  if (flags == nullptr || device < 0 || device >= kMaxDevices) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(device) != cudaSuccess) {
    return SVLLM_ERR_CUDA;
  }
  int status = SVLLM_OK;
  int* word = library_error_word(device);
  if (word == nullptr || cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpy(flags, word, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
    status = SVLLM_ERR_CUDA;
  } else if (reset && cudaMemset(word, 0, sizeof(int)) != cudaSuccess) {
    status = SVLLM_ERR_CUDA;
  }
  if (status != SVLLM_OK) cudaGetLastError();
  cudaSetDevice(prev);
  return status;
}

}  // extern "C"

// Host-side launch plumbing shared by the C-ABI entry points: argument checks, device
// properties and occupancy caches, the per-op pipeline shape, and the device error word.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <utility>

#include "svllm_kernels.h"

namespace svllm::k {

// Shape of one op's bulk-copy pipeline: target bytes per stage, stages per warp, warps per CTA.
struct PipelineShape {
  int unit_bytes;
  int stages;
  int warps;
};

enum class OpId { kRmsNorm, kAddRmsNorm, kQkNormRope, kRope, kSiluAndMul, kEmbedding, kCount };

// The pipeline shape of one op: the library's tuned default, or the override that the
// SVLLM_PIPELINE environment variable gave when the process first launched a kernel.
PipelineShape pipeline_shape(OpId op);

// Devices the per-device caches hold (current_device rejects higher ordinals).
constexpr int kMaxDevices = 64;

// The current device and its SM count (cached per device).
int current_device(int* device);
int sm_count(int device);

// Maximum resident CTAs of `func` per SM for this block size and dynamic shared memory. Raises
// the function's dynamic shared-memory limit the first time it is seen on a device.
int blocks_per_sm(const void* func, int threads, size_t smem_bytes, int device);

// Largest dynamic shared memory a CTA may use on this architecture.
constexpr size_t kMaxSmemPerCta = 227 * 1024;

// The library's own error word on `device` (a __device__ int, address cached per device).
int* library_error_word(int device);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// Maps the launch's cudaGetLastError() to a status.
inline int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SVLLM_OK : SVLLM_ERR_LAUNCH;
}

// Warps per CTA for a batch of `units` work units: the tuned count, or fewer when the batch is
// too small to give every SM a full CTA (decode-sized batches), so that the grid still spans
// all SMs and each warp's latency chain starts at once.
inline int warps_for(int64_t units, int tuned, int device) {
  const int64_t per_sm = (units + sm_count(device) - 1) / sm_count(device);
  return static_cast<int>(per_sm < tuned ? (per_sm > 0 ? per_sm : 1) : tuned);
}

// One launch through cudaLaunchKernelEx: `early` allows programmatic dependent launch,
// `cluster` > 1 sets the cluster size.
template <class... Params, class... Args>
int launch_with(bool early, void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                cudaStream_t stream, unsigned cluster, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (early) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  const int status = launch_status();  // also clears the error a failed launch leaves
  return err == cudaSuccess ? status : SVLLM_ERR_LAUNCH;
}

// Launches `kernel` with programmatic dependent launch allowed: the grid may be scheduled
// while the kernel before it in the stream is still running, and every kernel of this library
// waits (griddepcontrol.wait, its first statement) until that kernel has completed and its
// memory is visible before touching any. What it hides is the gap between kernels: launch
// processing and CTA start-up. `cluster` > 1 also sets the cluster size.
template <class... Params, class... Args>
int launch(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
           unsigned cluster, Args&&... args) {
  return launch_with(true, kernel, grid, block, smem, stream, cluster,
                     std::forward<Args>(args)...);
}

// Streaming kernels that move at least this many bytes are launched without programmatic
// dependent launch. Early scheduling hides the gap between kernels (a few microseconds): worth it
// for decode- and prefill-sized launches, and measured to cost time for long ones. On a B200,
// eager launches: the 1M-token chain (embedding, add_rms_norm, qk_norm_rope, silu_and_mul, 4-19 GB
// each) ran at 6497 GB/s with early scheduling and 6675 without; the 16384-token Llama chain
// (0.13-0.8 GB per op) at 5939 with and 5837 without. From a CUDA graph both were within 1%.
constexpr int64_t kEarlyLaunchMaxBytes = int64_t{1} << 30;

// `launch` for a streaming kernel that moves `bytes` of HBM traffic: scheduled early below
// kEarlyLaunchMaxBytes, after the kernel before it has completed at or above.
template <class... Params, class... Args>
int launch_streaming(int64_t bytes, void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t stream, unsigned cluster, Args&&... args) {
  return launch_with(bytes < kEarlyLaunchMaxBytes, kernel, grid, block, smem, stream, cluster,
                     std::forward<Args>(args)...);
}

// As `launch`, but the grid starts only once the kernel before it has completed. For grids
// whose CTAs are heavy enough (all of an SM's registers in four CTAs) that scheduling them early
// costs more than the gap it hides: decode attention after the rotary + cache-write kernel in a
// Qwen3-0.6B decode step ran 40% slower per step at batch 256 with early scheduling.
template <class... Params, class... Args>
int launch_serialized(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t stream, unsigned cluster, Args&&... args) {
  return launch_with(false, kernel, grid, block, smem, stream, cluster,
                     std::forward<Args>(args)...);
}

// Grid size for a persistent kernel: enough CTAs to fill every SM at the given occupancy, but
// no more CTAs than there is work for.
inline int64_t persistent_grid(int64_t work_ctas, int device, int per_sm) {
  const int64_t full = static_cast<int64_t>(sm_count(device)) * (per_sm > 0 ? per_sm : 1);
  return work_ctas < full ? (work_ctas > 0 ? work_ctas : 1) : full;
}

}  // namespace svllm::k

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

// Most warps a streaming (bulk-copy) kernel's CTA may have: those kernels are compiled with
// __launch_bounds__(512).
constexpr int kMaxBulkWarps = 16;

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

// The streaming kernels let the next kernel in the stream be scheduled at their start only when
// they move less than this many bytes; a larger launch lets it be scheduled as its CTAs exit.
// Scheduling the next kernel at the start hides its launch and start-up behind this one: it pays
// for decode-sized launches (the Qwen3-0.6B decode step at batch 1, one box: 0.94 ms against
// 1.06 ms with the exit point), and costs time behind long ones (the 1M-token chain launched eagerly ran at
// 6545 GB/s with every kernel triggering at its start, 6721 with the exit point). Measured on a
// B200 against no early scheduling at all for launches of 1 GB or more: the 131k-token chain
// 6437 -> 6505 GB/s, the 73k-token prefill chain 6291 -> 6343, the 1M and 16k (Llama) chains and
// the decode step unchanged.
constexpr int64_t kEarlyDependentsMaxBytes = int64_t{64} << 20;

inline int early_dependents(int64_t bytes) { return bytes < kEarlyDependentsMaxBytes ? 1 : 0; }

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

// Greedy sampling: the index of the largest logit of every row (torch.argmax semantics: the
// first index of the maximum; a NaN counts as larger than any number, the first NaN wins).
//
// This is the step after the final norm and the tied-embedding LM head (the reference's
// src/model/config.h:28 tie_word_embeddings; sampling "on GPU", docs/design-spec.md:28-29):
// logits [rows, vocab] with vocab ~150k are read once. A row is split over the 8 CTAs of a
// thread-block cluster (on 8 SMs), so even a single-sequence decode step streams its 300 KB row
// from eight SMs at once. Each CTA reduces its slice with 16-byte loads, shuffles and one shared
// memory pass; the cluster's eight partial results are then combined by CTA 0 reading the
// others' shared memory through the cluster's distributed shared memory. No global scratch,
// no atomics, no second launch.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "host_common.h"

namespace svllm::k {
namespace {

constexpr int kClusterCtas = 8;  // the portable cluster size
constexpr int kArgmaxThreads = 512;

struct ArgmaxArgs {
  const void* logits;
  int64_t* out;
  int64_t rows;
  int64_t vocab;
  int64_t stride;  // elements between rows
  int vec;         // 16-byte loads are legal (aligned base, stride and vocab)
};

struct Best {
  float v;
  int64_t i;
};

// a beats b: larger value, NaN above every number, the lower index on ties.
__device__ __forceinline__ bool beats(const Best& a, const Best& b) {
  const bool an = a.v != a.v, bn = b.v != b.v;
  if (an != bn) return an;
  if (an || a.v == b.v) return a.i < b.i;
  return a.v > b.v;
}

__device__ __forceinline__ void take(Best& best, float v, int64_t i) {
  const Best c{v, i};
  if (beats(c, best)) best = c;
}

__device__ __forceinline__ Best warp_best(Best b) {
#pragma unroll
  for (int off = 16; off > 0; off /= 2) {
    Best o;
    o.v = __shfl_xor_sync(0xffffffffu, b.v, off);
    o.i = __shfl_xor_sync(0xffffffffu, b.i, off);
    if (beats(o, b)) b = o;
  }
  return b;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t num_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

// Address of `p` (this CTA's shared memory) in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_shared(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_addr(p)), "r"(rank));
  return out;
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ int64_t ld_cluster_s64(uint32_t addr) {
  int64_t v;
  asm volatile("ld.shared::cluster.s64 %0, [%1];" : "=l"(v) : "r"(addr) : "memory");
  return v;
}

template <class E>
__global__ void __cluster_dims__(kClusterCtas, 1, 1) __launch_bounds__(kArgmaxThreads)
    argmax_kernel(const ArgmaxArgs a) {
  using S = typename E::Storage;
  constexpr int kVec = E::kPerVec;
  __shared__ float warp_v[kArgmaxThreads / kWarpSize];
  __shared__ int64_t warp_i[kArgmaxThreads / kWarpSize];
  __shared__ float cta_v;
  __shared__ int64_t cta_i;

  const uint32_t rank = cluster_ctarank();
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x % kWarpSize;
  // this CTA's slice of every row, in whole vectors
  const int64_t units = a.vec ? a.vocab / kVec : a.vocab;
  const int64_t per = (units + kClusterCtas - 1) / kClusterCtas;
  const int64_t u_begin = min(units, per * rank);
  const int64_t u_end = min(units, u_begin + per);

  for (int64_t row = cluster_id_x(); row < a.rows; row += num_clusters_x()) {
    const S* x = static_cast<const S*>(a.logits) + row * a.stride;
    Best best{__int_as_float(0xff800000), INT64_MAX};  // -inf, an index no element has
    if (a.vec) {
      // four 16-byte loads in flight per thread; `beats` is a total order, so the order in
      // which candidates are taken does not change the result
      const int64_t step = blockDim.x;
      int64_t u = u_begin + threadIdx.x;
      for (; u + 3 * step < u_end; u += 4 * step) {
        uint4 raw[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) raw[q] = ld_global_nc_v4(x + (u + q * step) * kVec);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float f[kVec];
          unpack<E>(raw[q], f);
#pragma unroll
          for (int e = 0; e < kVec; ++e) take(best, f[e], (u + q * step) * kVec + e);
        }
      }
      for (; u < u_end; u += step) {
        float f[kVec];
        unpack<E>(ld_global_nc_v4(x + u * kVec), f);
#pragma unroll
        for (int e = 0; e < kVec; ++e) take(best, f[e], u * kVec + e);
      }
    } else {
      for (int64_t u = u_begin + threadIdx.x; u < u_end; u += blockDim.x) {
        take(best, E::to_float(x[u]), u);
      }
    }
    best = warp_best(best);
    if (lane == 0) {
      warp_v[warp] = best.v;
      warp_i[warp] = best.i;
    }
    __syncthreads();
    if (warp == 0) {
      Best b{__int_as_float(0xff800000), INT64_MAX};
      if (lane < static_cast<int>(blockDim.x / kWarpSize)) b = Best{warp_v[lane], warp_i[lane]};
      b = warp_best(b);
      if (lane == 0) {
        cta_v = b.v;
        cta_i = b.i;
      }
    }
    cluster_sync();  // every CTA's partial result is visible cluster-wide
    if (rank == 0 && threadIdx.x == 0) {
      Best b{cta_v, cta_i};
      for (uint32_t r = 1; r < kClusterCtas; ++r) {
        const Best o{ld_cluster_f32(map_shared(&cta_v, r)), ld_cluster_s64(map_shared(&cta_i, r))};
        if (beats(o, b)) b = o;
      }
      a.out[row] = b.i;
    }
    cluster_sync();  // CTA 0 has read everyone's result before the next row overwrites it
  }
}

template <class E>
int launch_argmax(const void* logits, int64_t rows, int64_t vocab, int64_t stride, int64_t* out,
                  cudaStream_t stream) {
  using S = typename E::Storage;
  if (rows < 0 || vocab <= 0 || stride < vocab || vocab >= (int64_t{1} << 40)) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  if (rows == 0) return SVLLM_OK;
  if (logits == nullptr || out == nullptr) return SVLLM_ERR_INVALID_ARGUMENT;
  int device;
  if (current_device(&device) != SVLLM_OK) return SVLLM_ERR_CUDA;

  ArgmaxArgs a{};
  a.logits = logits;
  a.out = out;
  a.rows = rows;
  a.vocab = vocab;
  a.stride = stride;
  a.vec = aligned16(logits) && (stride * sizeof(S)) % 16 == 0 && (vocab * sizeof(S)) % 16 == 0;

  // one cluster per row, as many clusters as fit on the GPU at once
  const int per_sm = blocks_per_sm(reinterpret_cast<const void*>(argmax_kernel<E>),
                                   kArgmaxThreads, 0, device);
  const int64_t max_clusters =
      static_cast<int64_t>(sm_count(device)) * (per_sm > 0 ? per_sm : 1) / kClusterCtas;
  const int64_t clusters = rows < max_clusters ? rows : (max_clusters > 0 ? max_clusters : 1);
  argmax_kernel<E><<<static_cast<unsigned>(clusters * kClusterCtas), kArgmaxThreads, 0, stream>>>(a);
  return launch_status();
}

}  // namespace
}  // namespace svllm::k

extern "C" {

int svllm_argmax_bf16(const void* logits, int64_t num_rows, int64_t vocab, int64_t row_stride,
                      int64_t* out_ids, svllm_stream stream) {
  return svllm::k::launch_argmax<svllm::k::Bf16>(logits, num_rows, vocab, row_stride, out_ids,
                                                 reinterpret_cast<cudaStream_t>(stream));
}

int svllm_argmax_f32(const float* logits, int64_t num_rows, int64_t vocab, int64_t row_stride,
                     int64_t* out_ids, svllm_stream stream) {
  return svllm::k::launch_argmax<svllm::k::F32>(logits, num_rows, vocab, row_stride, out_ids,
                                                reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

// Greedy sampling: the index of the largest logit of every row (torch.argmax semantics: the
// first index of the maximum; a NaN counts as larger than any number, the first NaN wins).
//
// This is the step after the final norm and the tied-embedding LM head (the reference's
// src/model/config.h:28 tie_word_embeddings; sampling "on GPU", docs/design-spec.md:28-29):
// logits [rows, vocab] with vocab ~150k are read once, 16-byte loads, eight in flight per
// thread. A row goes to one CTA, or, when there are too few rows to keep enough loads in flight
// (a decode step's batch), to the 4 or 8 CTAs of a thread-block cluster, whose partial
// results are combined through distributed shared memory: even one sequence streams its 300 KB
// row from eight SMs. No global scratch, no atomics, no second launch.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "host_common.h"

namespace svllm::k {
namespace {

constexpr int kMaxCtasPerRow = 8;  // the portable cluster size
constexpr int kMaxThreads = 1024;
constexpr int kLoadsInFlight = 8;

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

constexpr float kNegInf = -__builtin_huge_valf();

// a beats b: NaN above every number, then the larger value, then the lower index.
__device__ __forceinline__ bool beats(const Best& a, const Best& b) {
  const bool an = a.v != a.v, bn = b.v != b.v;
  if (an != bn) return an;
  if (an || a.v == b.v) return a.i < b.i;
  return a.v > b.v;
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

// The larger of a and b, NaN if either is NaN.
__device__ __forceinline__ float max_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// c replaces the running maximum m of earlier candidates: it is larger, or it is the first NaN.
__device__ __forceinline__ bool exceeds(float c, float m) { return c > m || (c != c && m == m); }

// f is the value v (-0 == +0; every NaN matches a NaN).
__device__ __forceinline__ bool same(float f, float v) { return f == v || (f != f && v != v); }

// The largest element of whole 16-byte vectors, reduced word-wise in the storage type (one
// instruction for two bf16 elements) and finished in fp32; NaN if any element is NaN.
template <class E>
struct VecMax;

template <>
struct VecMax<Bf16> {
  static constexpr uint32_t kNegInfWord = 0xff80ff80u;  // -inf in both halves
  __device__ static __forceinline__ uint32_t combine(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  __device__ static __forceinline__ float finish(uint32_t w) {
    return max_nan(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
};

template <>
struct VecMax<F32> {
  static constexpr uint32_t kNegInfWord = 0xff800000u;
  __device__ static __forceinline__ uint32_t combine(uint32_t a, uint32_t b) {
    return __float_as_uint(max_nan(__uint_as_float(a), __uint_as_float(b)));
  }
  __device__ static __forceinline__ float finish(uint32_t w) { return __uint_as_float(w); }
};

template <class E, int N>
__device__ __forceinline__ float vectors_max(const uint4 (&raw)[N]) {
  uint32_t w[4 * N];
#pragma unroll
  for (int q = 0; q < N; ++q) {
    w[4 * q] = raw[q].x;
    w[4 * q + 1] = raw[q].y;
    w[4 * q + 2] = raw[q].z;
    w[4 * q + 3] = raw[q].w;
  }
  // pairwise tree: 4N words to one
#pragma unroll
  for (int width = 2 * N; width >= 1; width /= 2) {
#pragma unroll
    for (int j = 0; j < width; ++j) w[j] = VecMax<E>::combine(w[j], w[j + width]);
  }
  return VecMax<E>::finish(w[0]);
}

// One thread's pass over its units [u_begin, u_end) of a row (units u_begin + threadIdx.x + k *
// blockDim.x), in chunks of kLoadsInFlight units: the largest value `v` and the chunk holding
// its first occurrence, `n` units starting at unit `u` (u = -1: the thread has no units).
// Candidates arrive in increasing index order, so a strict comparison keeps the first maximum;
// a chunk's maximum costs about one instruction per element pair, and the exact index is looked
// up afterwards, only by the threads that hold the row's maximum.
struct Scan {
  float v;
  int64_t u;
  int n;
};

// The last chunk a thread loaded, kept in registers: when it holds the maximum (always, for a
// thread with one chunk) the index lookup needs no second load.
struct Chunk {
  uint4 raw[kLoadsInFlight];
  int64_t u = -1;
};

template <class E>
__device__ __forceinline__ Scan scan_slice(const typename E::Storage* x, int64_t u_begin,
                                           int64_t u_end, int vec, Chunk& last) {
  constexpr int kVec = E::kPerVec;
  const int64_t step = blockDim.x;
  int64_t u = u_begin + threadIdx.x;
  // -inf in the thread's first unit: if nothing exceeds it, every element is -inf and the
  // first one is the answer
  Scan s{kNegInf, u < u_end ? u : -1, 1};
  if (vec) {
    constexpr uint32_t kFill = VecMax<E>::kNegInfWord;  // units past the slice end read -inf
    for (; u < u_end; u += kLoadsInFlight * step) {
#pragma unroll
      for (int q = 0; q < kLoadsInFlight; ++q) {
        const int64_t uq = u + q * step;
        last.raw[q] = uq < u_end ? ld_global_nc_v4(x + uq * kVec)
                                 : make_uint4(kFill, kFill, kFill, kFill);
      }
      last.u = u;
      const float c = vectors_max<E>(last.raw);
      if (exceeds(c, s.v)) {
        const int64_t n = (u_end - u + step - 1) / step;
        s = Scan{c, u, static_cast<int>(n < kLoadsInFlight ? n : kLoadsInFlight)};
      }
    }
  } else {
    for (; u < u_end; u += step) {
      const float c = E::to_float(x[u]);
      if (exceeds(c, s.v)) s = Scan{c, u, 1};
    }
  }
  return s;
}

// The first index in the thread's chunk `s` whose element is v (the chunk holds one), from the
// registers when `last` is that chunk, else from memory.
template <class E>
__device__ int64_t first_index_of(const typename E::Storage* x, const Scan& s, float v, int vec,
                                  const Chunk& last) {
  constexpr int kVec = E::kPerVec;
  const int64_t step = blockDim.x;
  if (vec && last.u == s.u) {
    int64_t found = INT64_MAX;
    // backwards, so that the last assignment is the first match
#pragma unroll
    for (int q = kLoadsInFlight - 1; q >= 0; --q) {
      float f[kVec];
      unpack<E>(last.raw[q], f);
#pragma unroll
      for (int e = kVec - 1; e >= 0; --e) {
        if (q < s.n && same(f[e], v)) found = (s.u + q * step) * kVec + e;
      }
    }
    return found;
  }
  for (int q = 0; q < s.n; ++q) {
    const int64_t unit = s.u + q * step;
    if (vec) {
      float f[kVec];
      unpack<E>(ld_global_nc_v4(x + unit * kVec), f);
#pragma unroll
      for (int e = 0; e < kVec; ++e) {
        if (same(f[e], v)) return unit * kVec + e;
      }
    } else if (same(E::to_float(x[unit]), v)) {
      return unit;
    }
  }
  return INT64_MAX;
}

// The CTA's (largest value, first index of it) over this row's slice; every thread returns it.
// Two barriers: one after the value reduction, one after the index reduction; each reduction
// has its own scratch, so the next row's writes cannot overtake this row's reads.
template <class E>
__device__ __forceinline__ Best cta_best(const typename E::Storage* x, const Scan& s, int vec,
                                         const Chunk& last, float* red_v, int64_t* red_i) {
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x % kWarpSize;
  const int warps = blockDim.x / kWarpSize;
  float v = s.v;
#pragma unroll
  for (int off = 16; off > 0; off /= 2) v = max_nan(v, __shfl_xor_sync(0xffffffffu, v, off));
  if (lane == 0) red_v[warp] = v;
  __syncthreads();
  v = lane < warps ? red_v[lane] : kNegInf;
#pragma unroll
  for (int off = 16; off > 0; off /= 2) v = max_nan(v, __shfl_xor_sync(0xffffffffu, v, off));

  int64_t i = (s.u >= 0 && same(s.v, v)) ? first_index_of<E>(x, s, v, vec, last) : INT64_MAX;
#pragma unroll
  for (int off = 16; off > 0; off /= 2) i = min(i, __shfl_xor_sync(0xffffffffu, i, off));
  if (lane == 0) red_i[warp] = i;
  __syncthreads();
  i = lane < warps ? red_i[lane] : INT64_MAX;
#pragma unroll
  for (int off = 16; off > 0; off /= 2) i = min(i, __shfl_xor_sync(0xffffffffu, i, off));
  return Best{v, i};
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
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

// Row r goes to CTAs [r * kCtas, (r + 1) * kCtas), one cluster when kCtas > 1; every CTA of a
// cluster runs the same rows, so all meet every cluster barrier.
template <class E, int kCtas>
__global__ void __launch_bounds__(kMaxThreads) argmax_kernel(const ArgmaxArgs a) {
  grid_dependency_sync();
  using S = typename E::Storage;
  __shared__ float red_v[kMaxThreads / kWarpSize];
  __shared__ int64_t red_i[kMaxThreads / kWarpSize];
  __shared__ float cta_v;
  __shared__ int64_t cta_i;

  const uint32_t rank = kCtas > 1 ? cluster_ctarank() : 0;
  // this CTA's slice of every row, in whole units
  const int64_t units = a.vec ? a.vocab / E::kPerVec : a.vocab;
  const int64_t per = (units + kCtas - 1) / kCtas;
  const int64_t u_begin = min(units, per * rank);
  const int64_t u_end = min(units, u_begin + per);
  const int64_t groups = gridDim.x / kCtas;

  for (int64_t row = blockIdx.x / kCtas; row < a.rows; row += groups) {
    const S* x = static_cast<const S*>(a.logits) + row * a.stride;
    Chunk last;
    const Scan sc = scan_slice<E>(x, u_begin, u_end, a.vec, last);
    const Best b = cta_best<E>(x, sc, a.vec, last, red_v, red_i);
    if constexpr (kCtas == 1) {
      if (threadIdx.x == 0) a.out[row] = b.i;
    } else {
      if (threadIdx.x == 0) {
        cta_v = b.v;
        cta_i = b.i;
      }
      cluster_sync();  // every CTA's partial result is visible cluster-wide
      if (rank == 0 && threadIdx.x < kWarpSize) {
        // lane r reads CTA r's result (all loads in flight at once), then one warp merge
        Best o{kNegInf, INT64_MAX};
        if (threadIdx.x < kCtas) {
          o = Best{ld_cluster_f32(map_shared(&cta_v, threadIdx.x)),
                   ld_cluster_s64(map_shared(&cta_i, threadIdx.x))};
        }
        o = warp_best(o);
        if (threadIdx.x == 0) a.out[row] = o.i;
      }
      cluster_sync();  // CTA 0 has read every result before a CTA moves on or exits
    }
  }
}

template <class E, int kCtas>
int launch_split(const ArgmaxArgs& a, int threads, cudaStream_t stream) {
  // kCtas CTAs per row, up to 2^30 CTAs; rows beyond that are taken in a grid-stride loop
  constexpr int64_t kMaxGroups = (int64_t{1} << 30) / kCtas;
  const int64_t groups = a.rows < kMaxGroups ? a.rows : kMaxGroups;
  return launch(argmax_kernel<E, kCtas>, dim3(static_cast<unsigned>(groups * kCtas)),
                dim3(static_cast<unsigned>(threads)), 0, stream, kCtas, a);
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

  // Launch shapes from sweeps of (CTAs per row, threads per CTA) on a B200 (148 SMs) at 1 to
  // 4096 rows of 151,936 bf16 logits. From 2 * SMs rows: one CTA per row, as large as lets every
  // row's CTA be resident at once (a second, part-empty wave costs up to 13%: 600 rows take
  // 32.8 us at 192 threads, 37.7 us at 256), else 128 threads. From SMs/2 rows: 512 threads.
  // Fewer rows: a row is split over a cluster, 4 x 256 threads down to SMs/4 rows and 8 x 512
  // under it (a single row: 5.2 us, about a kernel launch and one L2 round trip). A split whose
  // CTAs do not all fit on the GPU at once loses: each cluster is scheduled whole.
  const int64_t sms = sm_count(device);
  if (rows >= 2 * sms) {
    const void* one = reinterpret_cast<const void*>(argmax_kernel<E, 1>);
    for (const int threads : {256, 192, 128}) {
      if (rows <= sms * blocks_per_sm(one, threads, 0, device)) {
        return launch_split<E, 1>(a, threads, stream);
      }
    }
    return launch_split<E, 1>(a, 128, stream);
  }
  if (2 * rows >= sms) return launch_split<E, 1>(a, 512, stream);
  if (4 * rows >= sms) return launch_split<E, 4>(a, 256, stream);
  return launch_split<E, kMaxCtasPerRow>(a, 512, stream);
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

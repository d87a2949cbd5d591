// Decode attention over a paged KV cache: one query token per request, every query head of a
// KV head (grouped-query attention) served by the same pass over that head's cached rows.
//
//   o[b, h] = sum_j softmax_j(scale * q[b, h] . k[slot(b, j), h / G]) * v[slot(b, j), h / G],
//   j < seq_lens[b], slot(b, j) = block_tables[b][j / block_size] * block_size + j % block_size
//
// with the cache laid out [num_blocks, block_size, num_kv_heads, head_dim] (the reference's
// paged KV names, AGENTS.md "Names": block_table, slot_mapping, seq_lens). It replaces, for decode
// steps, the gather-then-SDPA composite of the model forward; the reference plans the kernel
// ("Decode attention: Split-KV paged kernel, GQA-aware", docs/ROADMAP.md).
//
// A CTA of 128 threads owns (request, KV head, context split). It walks its share of the
// context in sub-chunks of kSub tokens: scores into shared memory (D/8 lanes per row, one
// 16-byte load each), an online-softmax rescale, then p * v accumulated per lane over 8
// consecutive dims. Splits of one (request, KV head) form a thread-block cluster whose CTAs
// merge their (max, sum, partial output) through distributed shared memory, each writing a
// slice of the bf16 output. Scores, softmax and accumulation are fp32. No scratch memory, one
// launch.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "host_common.h"

namespace svllm::k {
namespace {

constexpr int kThreads = 128;
constexpr int kSub = 256;       // context tokens per sub-chunk
constexpr int kMaxSplits = 8;   // the portable cluster size
constexpr int kUnroll = 8;      // cache rows a lane has in flight

struct AttnArgs {
  void* out;                 // [num_seqs, num_heads, head_dim] bf16, contiguous
  const void* q;             // [num_seqs, num_heads, head_dim] bf16, token stride q_stride
  const void* k_cache;       // [num_blocks, block_size, num_kv_heads, head_dim] bf16
  const void* v_cache;
  const int32_t* block_tables;  // [num_seqs, max_blocks]
  const int32_t* seq_lens;      // [num_seqs]
  int64_t q_stride;
  int64_t num_blocks;
  int max_blocks;
  int block_size;
  int num_kv_heads;
  int splits;
  float scale;
  int* err;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

// A float of cluster CTA `rank`'s shared memory at the address of `p` in this CTA's. Not
// volatile: the loads of a merge are independent and may be in flight together (the cluster
// barrier before them orders them after the writes).
__device__ __forceinline__ float ld_remote_f32(const float* p, uint32_t rank) {
  uint32_t addr;
  asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(addr) : "r"(smem_addr(p)), "r"(rank));
  float v;
  asm("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

// Block-wide reduction of G floats per thread (max or sum) into `red` [warps][G]; every thread
// gets the G results. One barrier; `red` must not be rewritten before the next barrier.
template <bool kMax, int G>
__device__ __forceinline__ void block_reduce(float (&v)[G], float (*red)[G]) {
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int off = 16; off > 0; off /= 2) {
      const float o = __shfl_xor_sync(0xffffffffu, v[g], off);
      v[g] = kMax ? fmaxf(v[g], o) : v[g] + o;
    }
  }
  const int warp = threadIdx.x / kWarpSize;
  if (threadIdx.x % kWarpSize == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) red[warp][g] = v[g];
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float r = red[0][g];
#pragma unroll
    for (int w = 1; w < kThreads / kWarpSize; ++w) r = kMax ? fmaxf(r, red[w][g]) : r + red[w][g];
    v[g] = r;
  }
}

template <int D, int G>
__global__ void __launch_bounds__(kThreads) decode_attention_kernel(const AttnArgs a) {
  grid_dependency_sync();
  constexpr int kLpr = D / 8;              // lanes per cache row, 8 dims (16 bytes) each
  constexpr int kRows = kThreads / kLpr;   // rows in flight per pass
  static_assert(kWarpSize % kLpr == 0, "a row's lanes stay in one warp");

  __shared__ float scores[G][kSub];
  __shared__ float red_max[kThreads / kWarpSize][G];
  __shared__ float red_sum[kThreads / kWarpSize][G];
  __shared__ float part[kRows][G][D];  // per row group: partial outputs, summed at the end
  __shared__ float m_sm[G], l_sm[G];
  __shared__ int64_t slot_base[kSub + 1];  // the sub-chunk's blocks, first slot of each

  const int split = static_cast<int>(blockIdx.x % a.splits);
  const int64_t pair = blockIdx.x / a.splits;
  const int64_t b = pair / a.num_kv_heads;
  const int kh = static_cast<int>(pair % a.num_kv_heads);
  const int rg = threadIdx.x / kLpr;   // row group
  const int sub = threadIdx.x % kLpr;  // this lane's 8 dims: [8 sub, 8 sub + 8)

  int seq_len = a.seq_lens[b];
  if (seq_len < 0 || seq_len > a.max_blocks * a.block_size) {  // past the block table
    if (threadIdx.x == 0) raise_error(a.err, kErrBadIndex);
    seq_len = seq_len < 0 ? 0 : a.max_blocks * a.block_size;
  }
  const int chunk = (seq_len + a.splits - 1) / a.splits;
  const int j_begin = min(seq_len, split * chunk);
  const int j_end = min(seq_len, j_begin + chunk);
  const int32_t* table = a.block_tables + b * a.max_blocks;

  // this lane's slice of each query head, fp32
  float q[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint8_t* qp = static_cast<const uint8_t*>(a.q) +
                        (b * a.q_stride + static_cast<int64_t>(kh * G + g) * D + sub * 8) * 2;
    float f[8];
    unpack<Bf16>(ld_global_nc_v4(qp), f);
#pragma unroll
    for (int e = 0; e < 8; ++e) q[g][e] = f[e];
  }

  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -__builtin_huge_valf();
    l[g] = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] = 0.0f;
  }

  const int64_t row_elems = static_cast<int64_t>(a.num_kv_heads) * D;
  const int64_t head_offset = static_cast<int64_t>(kh) * D + sub * 8;
  const Bf16::Storage* kc = static_cast<const Bf16::Storage*>(a.k_cache);
  const Bf16::Storage* vc = static_cast<const Bf16::Storage*>(a.v_cache);

  for (int s0 = j_begin; s0 < j_end; s0 += kSub) {
    const int n = min(kSub, j_end - s0);
    // the sub-chunk's block-table entries, once, as first slots
    const int blk0 = s0 / a.block_size;
    const int nblk = (s0 + n - 1) / a.block_size - blk0 + 1;
    for (int t = threadIdx.x; t < nblk; t += kThreads) {
      int blk = table[blk0 + t];
      if (blk < 0 || blk >= a.num_blocks) {  // an entry outside the cache: read block 0
        raise_error(a.err, kErrBadIndex);
        blk = 0;
      }
      slot_base[t] = static_cast<int64_t>(blk) * a.block_size;
    }
    __syncthreads();
    auto row_offset = [&](int i) -> int64_t {  // element offset of sub-chunk row i, this head
      const int j = s0 + i;
      return (slot_base[j / a.block_size - blk0] + j % a.block_size) * row_elems + head_offset;
    };
    // scores of this sub-chunk, kUnroll rows per lane in flight; the loop is warp-uniform
    // (a row's lanes reduce by shuffles)
    for (int i0 = 0; i0 < n; i0 += kRows * kUnroll) {
      uint4 raw[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i = i0 + u * kRows + rg;
        raw[u] = i < n ? ld_global_nc_v4(kc + row_offset(i)) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i = i0 + u * kRows + rg;
        float kf[8];
        unpack<Bf16>(raw[u], kf);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float d = 0.0f;
#pragma unroll
          for (int e = 0; e < 8; ++e) d = __fmaf_rn(q[g][e], kf[e], d);
#pragma unroll
          for (int off = kLpr / 2; off > 0; off /= 2) d += __shfl_xor_sync(0xffffffffu, d, off);
          if (sub == 0 && i < n) scores[g][i] = d * a.scale;
        }
      }
    }
    __syncthreads();
    // online softmax: new running max, rescale what is accumulated, p = exp(s - max)
    float cm[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      cm[g] = -__builtin_huge_valf();
      for (int i = threadIdx.x; i < n; i += kThreads) cm[g] = fmaxf(cm[g], scores[g][i]);
    }
    block_reduce<true>(cm, red_max);
    float ps[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float m_new = fmaxf(m[g], cm[g]);
      const float alpha = __expf(m[g] - m_new);
      ps[g] = 0.0f;
      for (int i = threadIdx.x; i < n; i += kThreads) {
        const float p = __expf(scores[g][i] - m_new);
        scores[g][i] = p;
        ps[g] += p;
      }
      l[g] *= alpha;
      m[g] = m_new;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] *= alpha;
    }
    block_reduce<false>(ps, red_sum);  // its barrier also publishes the p values
#pragma unroll
    for (int g = 0; g < G; ++g) l[g] += ps[g];
    // p * v over this lane's 8 dims, kUnroll rows in flight
    for (int i0 = 0; i0 < n; i0 += kRows * kUnroll) {
      uint4 raw[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i = i0 + u * kRows + rg;
        raw[u] = i < n ? ld_global_nc_v4(vc + row_offset(i)) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i = i0 + u * kRows + rg;
        if (i < n) {
          float vf[8];
          unpack<Bf16>(raw[u], vf);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float p = scores[g][i];
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[g][e] = __fmaf_rn(p, vf[e], acc[g][e]);
          }
        }
      }
    }
    __syncthreads();  // scores and slot_base are rewritten by the next sub-chunk
  }

  // the row groups' partial outputs summed: part[0] holds this CTA's result
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int e = 0; e < 8; ++e) part[rg][g][sub * 8 + e] = acc[g][e];
  }
  if (threadIdx.x < G) {
    m_sm[threadIdx.x] = m[threadIdx.x];
    l_sm[threadIdx.x] = l[threadIdx.x];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += kThreads) {
    const int g = idx / D, d = idx % D;
    float s = part[0][g][d];
    for (int r = 1; r < kRows; ++r) s += part[r][g][d];
    part[0][g][d] = s;
  }

  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + (b * a.num_kv_heads + kh) * G * D;
  if (a.splits == 1) {
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * D; idx += kThreads) {
      const int g = idx / D;
      out[idx] = __float2bfloat16_rn(l_sm[g] > 0.0f ? part[0][g][idx % D] / l_sm[g] : 0.0f);
    }
    return;
  }
  // Splits of one (request, KV head) are one cluster; its CTAs share the merge: CTA r combines
  // and writes output elements [r * per, (r + 1) * per) from every split's (max, sum, part).
  cluster_sync_all();
  const int per = G * D / a.splits;
  const int first = static_cast<int>(cluster_rank()) * per;
  for (int idx = first + threadIdx.x; idx < first + per; idx += kThreads) {
    const int g = idx / D, d = idx % D;
    float mr[kMaxSplits], lr[kMaxSplits], pr[kMaxSplits];
#pragma unroll
    for (int r = 0; r < kMaxSplits; ++r) {
      if (r < a.splits) {
        mr[r] = ld_remote_f32(&m_sm[g], r);
        lr[r] = ld_remote_f32(&l_sm[g], r);
        pr[r] = ld_remote_f32(&part[0][g][d], r);
      }
    }
    float mx = -__builtin_huge_valf();
#pragma unroll
    for (int r = 0; r < kMaxSplits; ++r) {
      if (r < a.splits) mx = fmaxf(mx, mr[r]);
    }
    float o = 0.0f, lsum = 0.0f;
#pragma unroll
    for (int r = 0; r < kMaxSplits; ++r) {
      if (r < a.splits) {
        const float w = mr[r] == -__builtin_huge_valf() ? 0.0f : __expf(mr[r] - mx);
        o += w * pr[r];
        lsum += w * lr[r];
      }
    }
    out[idx] = __float2bfloat16_rn(lsum > 0.0f ? o / lsum : 0.0f);
  }
  cluster_sync_all();  // every CTA's shared memory stays valid until the others have read it
}

template <int D, int G>
int launch_attention(const AttnArgs& a, int64_t num_seqs, cudaStream_t stream) {
  const int64_t blocks = num_seqs * a.num_kv_heads * a.splits;
  return launch(decode_attention_kernel<D, G>, dim3(static_cast<unsigned>(blocks)),
                dim3(kThreads), 0, stream, a.splits > 1 ? static_cast<unsigned>(a.splits) : 1u,
                a);
}

template <int D>
int dispatch_group(const AttnArgs& a, int64_t num_seqs, int group, cudaStream_t stream) {
  switch (group) {
    case 1: return launch_attention<D, 1>(a, num_seqs, stream);
    case 2: return launch_attention<D, 2>(a, num_seqs, stream);
    case 4: return launch_attention<D, 4>(a, num_seqs, stream);
    case 8: return launch_attention<D, 8>(a, num_seqs, stream);
    default: return SVLLM_ERR_UNSUPPORTED;
  }
}

}  // namespace
}  // namespace svllm::k

extern "C" int svllm_paged_decode_attention_bf16(
    void* out, const void* q, int64_t q_token_stride, const void* k_cache, const void* v_cache,
    int64_t num_blocks, int64_t block_size, const int32_t* block_tables, int64_t max_blocks,
    const int32_t* seq_lens, int64_t num_seqs, int64_t num_heads, int64_t num_kv_heads,
    int64_t head_dim, int64_t max_seq_len, float scale, svllm_stream stream) {
  using namespace svllm::k;
  if (num_seqs < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0 ||
      block_size <= 0 || max_blocks <= 0 || num_blocks <= 0 || max_seq_len <= 0 ||
      max_seq_len > max_blocks * block_size || q_token_stride < num_heads * head_dim) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  if (num_seqs == 0) return SVLLM_OK;
  if (out == nullptr || q == nullptr || k_cache == nullptr || v_cache == nullptr ||
      block_tables == nullptr || seq_lens == nullptr) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  const int64_t group = num_heads / num_kv_heads;
  if ((head_dim != 64 && head_dim != 128) || group > 8 || (group & (group - 1)) != 0 ||
      !aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || (q_token_stride * 2) % 16 != 0 ||
      num_seqs * num_kv_heads * kMaxSplits >= (int64_t{1} << 31) ||
      max_blocks >= (int64_t{1} << 31) || block_size >= (int64_t{1} << 20)) {
    return SVLLM_ERR_UNSUPPORTED;
  }
  int device;
  if (current_device(&device) != SVLLM_OK) return SVLLM_ERR_CUDA;
  int* err = library_error_word(device);
  if (err == nullptr) return SVLLM_ERR_CUDA;

  AttnArgs a{};
  a.out = out;
  a.q = q;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.block_tables = block_tables;
  a.seq_lens = seq_lens;
  a.q_stride = q_token_stride;
  a.num_blocks = num_blocks;
  a.max_blocks = static_cast<int>(max_blocks);
  a.block_size = static_cast<int>(block_size);
  a.num_kv_heads = static_cast<int>(num_kv_heads);
  a.scale = scale;
  a.err = err;
  // Split the context until there are about two CTAs per SM, never below 64 tokens per split.
  const int64_t pairs = num_seqs * num_kv_heads;
  int64_t splits = (2 * sm_count(device) + pairs - 1) / pairs;
  const int64_t by_length = (max_seq_len + 63) / 64;
  splits = splits < by_length ? splits : by_length;
  int pow2 = 1;  // a power of two: the cluster sizes are 1, 2, 4 or 8
  while (pow2 * 2 <= splits && pow2 * 2 <= kMaxSplits) pow2 *= 2;
  a.splits = pow2;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return head_dim == 128 ? dispatch_group<128>(a, num_seqs, static_cast<int>(group), s)
                         : dispatch_group<64>(a, num_seqs, static_cast<int>(group), s);
}

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
// A CTA of 128 threads owns (request, KV head, context split), and each of its 4 warps a
// contiguous share of that split. A warp streams its rows kUnroll per lane at a time, the K and
// V loads (16 bytes each, D/8 lanes per row) in flight together, and keeps its own online
// softmax (running max and sum by shuffles) and p * v accumulators: no block barrier until the
// warps merge at the end. Splits of one (request, KV head) form a thread-block cluster whose
// CTAs merge their (max, sum, partial output) through distributed shared memory, each writing a
// slice of the bf16 output. Scores, softmax and accumulation are fp32. No scratch memory, one
// launch.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "host_common.h"

namespace svllm::k {
namespace {

constexpr int kThreads = 128;
constexpr int kMaxSplits = 8;   // the portable cluster size
constexpr int kMaxUnroll = 8;   // cache rows a lane has in flight (fewer when more CTAs must fit)

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

template <int D, int G, int kUnroll>
__global__ void __launch_bounds__(kThreads) decode_attention_kernel(const AttnArgs a) {
  grid_dependency_sync();
  constexpr int kLpr = D / 8;                  // lanes per cache row, 8 dims (16 bytes) each
  constexpr int kGroups = kWarpSize / kLpr;    // rows one warp-wide load covers
  constexpr int kStep = kGroups * kUnroll;     // rows per warp per iteration
  constexpr int kWarps = kThreads / kWarpSize;
  static_assert(kWarpSize % kLpr == 0, "a row's lanes stay in one warp");

  __shared__ float warp_m[kWarps][G], warp_l[kWarps][G];
  __shared__ float warp_acc[kWarps][G][D];
  __shared__ float m_sm[G], l_sm[G];
  __shared__ float part[G][D];

  const int split = static_cast<int>(blockIdx.x % a.splits);
  const int64_t pair = blockIdx.x / a.splits;
  const int64_t b = pair / a.num_kv_heads;
  const int kh = static_cast<int>(pair % a.num_kv_heads);
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x % kWarpSize;
  const int grp = lane / kLpr;  // which of the warp's kGroups rows this lane reads
  const int sub = lane % kLpr;  // this lane's 8 dims: [8 sub, 8 sub + 8)

  int seq_len = a.seq_lens[b];
  if (seq_len < 0 || seq_len > a.max_blocks * a.block_size) {  // past the block table
    if (threadIdx.x == 0) raise_error(a.err, kErrBadIndex);
    seq_len = seq_len < 0 ? 0 : a.max_blocks * a.block_size;
  }
  // this CTA's split of the context, then this warp's contiguous share of it
  const int chunk = (seq_len + a.splits - 1) / a.splits;
  const int c_begin = min(seq_len, split * chunk);
  const int c_end = min(seq_len, c_begin + chunk);
  const int per_warp = (c_end - c_begin + kWarps - 1) / kWarps;
  const int w_begin = min(c_end, c_begin + warp * per_warp);
  const int w_end = min(c_end, w_begin + per_warp);
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

  // Each iteration: kUnroll rows per lane, K and V loads all in flight together; the scores of
  // the warp's kStep rows, their running max and sum by shuffles, then p * v into this lane's 8
  // dims. No block-wide barrier until the warps meet at the end.
  for (int r0 = w_begin; r0 < w_end; r0 += kStep) {
    uint4 kraw[kUnroll], vraw[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int j = r0 + u * kGroups + grp;
      if (j < w_end) {
        int blk = __ldg(table + j / a.block_size);
        if (blk < 0 || blk >= a.num_blocks) {  // an entry outside the cache: read block 0
          raise_error(a.err, kErrBadIndex);
          blk = 0;
        }
        const int64_t off = (static_cast<int64_t>(blk) * a.block_size + j % a.block_size) *
                                row_elems + head_offset;
        kraw[u] = ld_global_nc_v4(kc + off);
        vraw[u] = ld_global_nc_v4(vc + off);
      } else {
        kraw[u] = make_uint4(0, 0, 0, 0);
        vraw[u] = make_uint4(0, 0, 0, 0);
      }
    }
    float s[kUnroll][G];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const bool valid = r0 + u * kGroups + grp < w_end;
      float kf[8];
      unpack<Bf16>(kraw[u], kf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float d = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) d = __fmaf_rn(q[g][e], kf[e], d);
#pragma unroll
        for (int off = kLpr / 2; off > 0; off /= 2) d += __shfl_xor_sync(0xffffffffu, d, off);
        s[u][g] = valid ? d * a.scale : -__builtin_huge_valf();
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = s[0][g];
#pragma unroll
      for (int u = 1; u < kUnroll; ++u) mx = fmaxf(mx, s[u][g]);
#pragma unroll
      for (int off = kLpr; off < kWarpSize; off *= 2) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      }
      const float m_new = fmaxf(m[g], mx);  // finite: the iteration has a valid row
      const float alpha = __expf(m[g] - m_new);
      float ps = 0.0f;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        s[u][g] = __expf(s[u][g] - m_new);  // 0 for rows past the share
        ps += s[u][g];
      }
#pragma unroll
      for (int off = kLpr; off < kWarpSize; off *= 2) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l[g] = l[g] * alpha + ps;
      m[g] = m_new;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] *= alpha;
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float vf[8];
      unpack<Bf16>(vraw[u], vf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = __fmaf_rn(s[u][g], vf[e], acc[g][e]);
      }
    }
  }
  // the warp's row groups hold partial sums of the same dims: add them up
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
#pragma unroll
      for (int off = kLpr; off < kWarpSize; off *= 2) {
        acc[g][e] += __shfl_xor_sync(0xffffffffu, acc[g][e], off);
      }
    }
  }
  if (grp == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int e = 0; e < 8; ++e) warp_acc[warp][g][sub * 8 + e] = acc[g][e];
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      warp_m[warp][g] = m[g];
      warp_l[warp][g] = l[g];
    }
  }
  __syncthreads();
  // the warps' (max, sum, partial) merged into the CTA's
  if (threadIdx.x < G) {
    const int g = threadIdx.x;
    float mx = warp_m[0][g];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) mx = fmaxf(mx, warp_m[w][g]);
    float ls = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      ls += warp_m[w][g] == -__builtin_huge_valf() ? 0.0f : warp_l[w][g] * __expf(warp_m[w][g] - mx);
    }
    m_sm[g] = mx;
    l_sm[g] = ls;
  }
  for (int idx = threadIdx.x; idx < G * D; idx += kThreads) {
    const int g = idx / D, d = idx % D;
    float mx = warp_m[0][g];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) mx = fmaxf(mx, warp_m[w][g]);
    float o = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      o += warp_m[w][g] == -__builtin_huge_valf() ? 0.0f
                                                    : warp_acc[w][g][d] * __expf(warp_m[w][g] - mx);
    }
    part[g][d] = o;
  }
  __syncthreads();

  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + (b * a.num_kv_heads + kh) * G * D;
  if (a.splits == 1) {
    for (int idx = threadIdx.x; idx < G * D; idx += kThreads) {
      const int g = idx / D;
      out[idx] = __float2bfloat16_rn(l_sm[g] > 0.0f ? part[g][idx % D] / l_sm[g] : 0.0f);
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
        pr[r] = ld_remote_f32(&part[g][d], r);
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

// Rows in flight per lane: 8 while every CTA of the launch is resident at once (each warp's
// latency chain is then what bounds it), 4 when the CTAs run in waves (then occupancy does);
// half of that with 8 query heads per KV head, whose accumulators take the registers. Measured
// on a B200: 64 requests x 512 tokens 36 us at 8 rows, 44 us at 4; 256 requests 141 vs 128 us.
template <int D, int G>
int launch_attention(const AttnArgs& a, int64_t num_seqs, int device, cudaStream_t stream) {
  constexpr int kDeep = G >= 8 ? kMaxUnroll / 2 : kMaxUnroll;
  const int64_t blocks = num_seqs * a.num_kv_heads * a.splits;
  const unsigned cluster = a.splits > 1 ? static_cast<unsigned>(a.splits) : 1u;
  const int per_sm = blocks_per_sm(reinterpret_cast<const void*>(decode_attention_kernel<D, G, kDeep>),
                                   kThreads, 0, device);
  if (blocks <= static_cast<int64_t>(sm_count(device)) * (per_sm > 0 ? per_sm : 1)) {
    return launch(decode_attention_kernel<D, G, kDeep>, dim3(static_cast<unsigned>(blocks)),
                  dim3(kThreads), 0, stream, cluster, a);
  }
  return launch(decode_attention_kernel<D, G, kDeep / 2>, dim3(static_cast<unsigned>(blocks)),
                dim3(kThreads), 0, stream, cluster, a);
}

template <int D>
int dispatch_group(const AttnArgs& a, int64_t num_seqs, int group, int device,
                   cudaStream_t stream) {
  switch (group) {
    case 1: return launch_attention<D, 1>(a, num_seqs, device, stream);
    case 2: return launch_attention<D, 2>(a, num_seqs, device, stream);
    case 4: return launch_attention<D, 4>(a, num_seqs, device, stream);
    case 8: return launch_attention<D, 8>(a, num_seqs, device, stream);
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
  return head_dim == 128 ? dispatch_group<128>(a, num_seqs, static_cast<int>(group), device, s)
                         : dispatch_group<64>(a, num_seqs, static_cast<int>(group), device, s);
}

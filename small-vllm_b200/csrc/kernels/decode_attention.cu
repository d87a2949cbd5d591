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
// A CTA of 4 warps (8 or 16 when the grid is small) owns (request, KV head, context split), and
// each warp a contiguous share of that split, in tiles of 16 cache rows. Both products of a tile run on the
// tensor cores (mma.sync m16n8k16, bf16 in, fp32 accumulate), with the query heads of the KV
// head as the N = 8 columns: S^T = K Q^T straight from the rows a lane loads, then P^T (the
// tile's softmax numerators, rounded to bf16 as flash attention does) and V^T transposed in
// registers by movmatrix for O^T += V^T P^T. The running max and sum are per warp (base-2
// exponent domain); the accumulators are rescaled only when the max moves. Splits of one
// (request, KV head) form a thread-block cluster whose CTAs merge their (max, sum, partial
// output) through distributed shared memory, each writing a slice of the bf16 output. No scratch
// memory, one launch.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "common.cuh"
#include "host_common.h"

namespace svllm::k {
namespace {

constexpr int kMaxSplits = 8;  // the portable cluster size
constexpr int kTileRows = 16;  // cache rows per tensor-core tile (the M of m16n8k16)

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
  uint32_t page_magic;       // j / block_size = (umulhi(j, page_magic) + j) >> page_shift
  int page_shift;
  int num_kv_heads;
  int splits;
  float scale_log2;          // scale * log2(e): scores are kept in the base-2 exponent domain
  int* err;
};

// 2^x (the ex2 instruction; 2^-inf = 0).
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The warp's 8x8 bf16 matrix (lane l holds row l / 4, columns 2 (l % 4) and 2 (l % 4) + 1)
// transposed, in the same layout.
__device__ __forceinline__ uint32_t transpose8x8(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// Byte offset of cache row j of a request (its page looked up in the block table) from the
// start of the cache. Division by the block size: multiply by a precomputed reciprocal and
// shift (Granlund and Montgomery, "Division by invariant integers using multiplication", 1994,
// exact for j < 2^31).
__device__ __forceinline__ int64_t cache_row_offset(const AttnArgs& a, const int32_t* table,
                                                    int j, int64_t row_bytes) {
  const int page = static_cast<int>((__umulhi(static_cast<uint32_t>(j), a.page_magic) +
                                     static_cast<uint32_t>(j)) >> a.page_shift);
  int blk = __ldg(table + page);
  if (static_cast<uint64_t>(blk) >= static_cast<uint64_t>(a.num_blocks)) {
    raise_error(a.err, kErrBadIndex);  // an entry outside the cache: read block 0
    blk = 0;
  }
  return (static_cast<int64_t>(blk) * a.block_size + (j - page * a.block_size)) * row_bytes;
}

// One CTA: one (request, KV head, context split); each warp a contiguous share of the split, in
// tiles of 16 cache rows. Per tile, with lane l = 4 g + t:
//   S^T[16 rows x 8 heads] = K[16 x D] . Q^T[D x 8]   (mma; lane loads rows g and g + 8)
//   P^T = 2^(S^T * scale log2 e - running max), rounded to bf16, transposed by movmatrix into
//         the B operand of
//   O^T[D x 8 heads] += V^T[D x 16 rows] . P^T[16 x 8] (mma; V^T by movmatrix of the V rows)
// The head dimension is permuted consistently inside each product: lane t's 16-byte piece c
// of a row holds dims [32 c + 8 t, 32 c + 8 t + 8), which serve as the k-steps 2c and 2c + 1
// of Q K^T and as four 8x8 blocks of V. Query heads beyond G are zero columns.
template <int D, int G, int kWarps>
__global__ void __launch_bounds__(kWarps * kWarpSize) decode_attention_kernel(const AttnArgs a) {
  constexpr int kThreads = kWarps * kWarpSize;
  grid_dependency_sync();
  constexpr int kPieces = D / 32;  // 16-byte pieces per lane per cache row
  static_assert(G <= 8, "the query heads of a KV head fill at most the N = 8 of one mma");

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
  const int g = lane >> 2;  // the tile rows g and g + 8; query head g of the Q^T operand
  const int t = lane & 3;   // dims 8t.. of each piece; query heads 2t, 2t + 1 of the results

  int seq_len = a.seq_lens[b];
  if (seq_len < 0 || seq_len > a.max_blocks * a.block_size) {  // past the block table
    if (threadIdx.x == 0) raise_error(a.err, kErrBadIndex);
    seq_len = seq_len < 0 ? 0 : a.max_blocks * a.block_size;
  }
  // this CTA's split of the context, then this warp's share of it, both in whole tiles
  const int tiles = (seq_len + kTileRows - 1) / kTileRows;
  const int split_tiles = (tiles + a.splits - 1) / a.splits;
  const int warp_tiles = (split_tiles + kWarps - 1) / kWarps;
  const int w_begin = min(seq_len, (split * split_tiles + warp * warp_tiles) * kTileRows);
  const int w_end = min(seq_len, min((split + 1) * split_tiles,
                                     split * split_tiles + (warp + 1) * warp_tiles) * kTileRows);
  const int32_t* table = a.block_tables + b * a.max_blocks;

  // Q^T's B fragments: query head g of this KV head, this lane's dims of each piece
  uint4 qf[kPieces];
#pragma unroll
  for (int c = 0; c < kPieces; ++c) qf[c] = make_uint4(0, 0, 0, 0);
  if (g < G) {
    const uint8_t* qp = static_cast<const uint8_t*>(a.q) +
                        (b * a.q_stride + static_cast<int64_t>(kh * G + g) * D + 8 * t) * 2;
#pragma unroll
    for (int c = 0; c < kPieces; ++c) qf[c] = ld_global_nc_v4(qp + 64 * c);
  }

  // O^T accumulators: m-tile (c, i) covers the blocks (c, 2i), (c, 2i + 1) of V's dims
  float acc[kPieces][2][4];
#pragma unroll
  for (int c = 0; c < kPieces; ++c) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[c][i][e] = 0.0f;
    }
  }
  float m0 = -__builtin_huge_valf(), m1 = -__builtin_huge_valf();  // heads 2t, 2t + 1
  float l0 = 0.0f, l1 = 0.0f;  // this lane's rows only; summed over the warp at the end

  const int64_t row_bytes = static_cast<int64_t>(a.num_kv_heads) * D * 2;
  const uint8_t* kc = static_cast<const uint8_t*>(a.k_cache) + (static_cast<int64_t>(kh) * D + 8 * t) * 2;
  const uint8_t* vc = static_cast<const uint8_t*>(a.v_cache) + (static_cast<int64_t>(kh) * D + 8 * t) * 2;

  // One tile: rows r0 + g and r0 + g + 8 of this lane, K and V, all pieces.
  struct Tile {
    uint4 k0[kPieces], k1[kPieces], v0[kPieces], v1[kPieces];
    bool ok0, ok1;
  };
  const auto load = [&](Tile& tl, int r0) {
    const int j0 = r0 + g, j1 = r0 + g + 8;
    tl.ok0 = j0 < w_end;
    tl.ok1 = j1 < w_end;
    const int64_t o0 = tl.ok0 ? cache_row_offset(a, table, j0, row_bytes) : 0;
    const int64_t o1 = tl.ok1 ? cache_row_offset(a, table, j1, row_bytes) : 0;
#pragma unroll
    for (int c = 0; c < kPieces; ++c) {
      tl.k0[c] = tl.ok0 ? ld_global_nc_v4(kc + o0 + 64 * c) : make_uint4(0, 0, 0, 0);
      tl.k1[c] = tl.ok1 ? ld_global_nc_v4(kc + o1 + 64 * c) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int c = 0; c < kPieces; ++c) {  // rows past the share read as zeros: 0 * p, never NaN
      tl.v0[c] = tl.ok0 ? ld_global_nc_v4(vc + o0 + 64 * c) : make_uint4(0, 0, 0, 0);
      tl.v1[c] = tl.ok1 ? ld_global_nc_v4(vc + o1 + 64 * c) : make_uint4(0, 0, 0, 0);
    }
  };
  const auto process = [&](const Tile& tl) {
    // S^T: lane holds rows g, g + 8 x heads 2t, 2t + 1
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int c = 0; c < kPieces; ++c) {
      mma_16816(s, tl.k0[c].x, tl.k1[c].x, tl.k0[c].y, tl.k1[c].y, qf[c].x, qf[c].y);
      mma_16816(s, tl.k0[c].z, tl.k1[c].z, tl.k0[c].w, tl.k1[c].w, qf[c].z, qf[c].w);
    }
    const float x00 = tl.ok0 ? s[0] * a.scale_log2 : -__builtin_huge_valf();
    const float x01 = tl.ok0 ? s[1] * a.scale_log2 : -__builtin_huge_valf();
    const float x10 = tl.ok1 ? s[2] * a.scale_log2 : -__builtin_huge_valf();
    const float x11 = tl.ok1 ? s[3] * a.scale_log2 : -__builtin_huge_valf();
    float mx0 = fmaxf(x00, x10), mx1 = fmaxf(x01, x11);
#pragma unroll
    for (int off = 4; off < kWarpSize; off *= 2) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);  // finite: the tile's first row is valid
    if (__any_sync(0xffffffffu, n0 > m0 || n1 > m1)) {    // the running max moved: rescale
      const float al0 = exp2_approx(m0 - n0), al1 = exp2_approx(m1 - n1);
      l0 *= al0;
      l1 *= al1;
#pragma unroll
      for (int c = 0; c < kPieces; ++c) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          acc[c][i][0] *= al0;
          acc[c][i][1] *= al1;
          acc[c][i][2] *= al0;
          acc[c][i][3] *= al1;
        }
      }
      m0 = n0;
      m1 = n1;
    }
    const float p00 = exp2_approx(x00 - m0), p01 = exp2_approx(x01 - m1);
    const float p10 = exp2_approx(x10 - m0), p11 = exp2_approx(x11 - m1);
    l0 += p00 + p10;
    l1 += p01 + p11;
    // P^T's B fragments: rows 2t, 2t + 1 (and + 8) of head g
    const uint32_t pb0 = transpose8x8(pack_bf16x2(p00, p01));
    const uint32_t pb1 = transpose8x8(pack_bf16x2(p10, p11));
#pragma unroll
    for (int c = 0; c < kPieces; ++c) {
      mma_16816(acc[c][0], transpose8x8(tl.v0[c].x), transpose8x8(tl.v0[c].y),
                transpose8x8(tl.v1[c].x), transpose8x8(tl.v1[c].y), pb0, pb1);
      mma_16816(acc[c][1], transpose8x8(tl.v0[c].z), transpose8x8(tl.v0[c].w),
                transpose8x8(tl.v1[c].z), transpose8x8(tl.v1[c].w), pb0, pb1);
    }
  };

  for (int r0 = w_begin; r0 < w_end; r0 += kTileRows) {
    Tile tl;
    load(tl, r0);
    process(tl);
  }
#pragma unroll
  for (int off = 4; off < kWarpSize; off *= 2) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const int h0 = 2 * t, h1 = 2 * t + 1;
  if (g == 0) {
    if (h0 < G) {
      warp_m[warp][h0] = m0;
      warp_l[warp][h0] = l0;
    }
    if (h1 < G) {
      warp_m[warp][h1] = m1;
      warp_l[warp][h1] = l1;
    }
  }
  // O^T element (dim, head): m-tile (c, i) row g is dim 32c + 8(g/2) + 4i + g%2, row g + 8
  // that dim + 2 (block (c, j) column 2t' + e is dim 32c + 8t' + 2j + e)
#pragma unroll
  for (int c = 0; c < kPieces; ++c) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int d = 32 * c + 8 * (g >> 1) + 4 * i + (g & 1);
      if (h0 < G) {
        warp_acc[warp][h0][d] = acc[c][i][0];
        warp_acc[warp][h0][d + 2] = acc[c][i][2];
      }
      if (h1 < G) {
        warp_acc[warp][h1][d] = acc[c][i][1];
        warp_acc[warp][h1][d + 2] = acc[c][i][3];
      }
    }
  }
  __syncthreads();
  // the warps' (max, sum, partial) merged into the CTA's
  if (threadIdx.x < G) {
    const int h = threadIdx.x;
    float mx = warp_m[0][h];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) mx = fmaxf(mx, warp_m[w][h]);
    float ls = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      ls += warp_m[w][h] == -__builtin_huge_valf() ? 0.0f
                                                   : warp_l[w][h] * exp2_approx(warp_m[w][h] - mx);
    }
    m_sm[h] = mx;
    l_sm[h] = ls;
  }
  for (int idx = threadIdx.x; idx < G * D; idx += kThreads) {
    const int h = idx / D, d = idx % D;
    float mx = warp_m[0][h];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) mx = fmaxf(mx, warp_m[w][h]);
    float o = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      o += warp_m[w][h] == -__builtin_huge_valf()
               ? 0.0f
               : warp_acc[w][h][d] * exp2_approx(warp_m[w][h] - mx);
    }
    part[h][d] = o;
  }
  __syncthreads();

  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + (b * a.num_kv_heads + kh) * G * D;
  if (a.splits == 1) {
    for (int idx = threadIdx.x; idx < G * D; idx += kThreads) {
      const int h = idx / D;
      out[idx] = __float2bfloat16_rn(l_sm[h] > 0.0f ? part[h][idx % D] / l_sm[h] : 0.0f);
    }
    return;
  }
  // Splits of one (request, KV head) are one cluster; its CTAs share the merge: CTA r combines
  // and writes output elements [r * per, (r + 1) * per) from every split's (max, sum, part).
  cluster_sync_all();
  const int per = G * D / a.splits;
  const int first = static_cast<int>(cluster_rank()) * per;
  for (int idx = first + threadIdx.x; idx < first + per; idx += kThreads) {
    const int h = idx / D, d = idx % D;
    float mr[kMaxSplits], lr[kMaxSplits], pr[kMaxSplits];
#pragma unroll
    for (int r = 0; r < kMaxSplits; ++r) {
      if (r < a.splits) {
        mr[r] = ld_remote_f32(&m_sm[h], r);
        lr[r] = ld_remote_f32(&l_sm[h], r);
        pr[r] = ld_remote_f32(&part[h][d], r);
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
        const float w = mr[r] == -__builtin_huge_valf() ? 0.0f : exp2_approx(mr[r] - mx);
        o += w * pr[r];
        lsum += w * lr[r];
      }
    }
    out[idx] = __float2bfloat16_rn(lsum > 0.0f ? o / lsum : 0.0f);
  }
  cluster_sync_all();  // every CTA's shared memory stays valid until the others have read it
}

// Warps per CTA: 4 when the grid fills the SMs several times over; more when it is small
// (decode of a few requests), so that each SM still has enough cache rows in flight, but no
// more than the split has tiles of 16 rows, and at most what keeps the warps' partial outputs
// within 40 KB of shared memory. Measured on a B200 (one Qwen3-0.6B layer): one request of
// 2048 tokens 8.0 -> 7.0 us with 16 warps, 8 requests 14.6 -> 12.2 us with 8.
template <int D, int G>
int launch_attention(const AttnArgs& a, int64_t num_seqs, int64_t split_tiles, int device,
                     cudaStream_t stream) {
  constexpr int kMaxWarps = 40960 / (G * D * 4) >= 16 ? 16 : 40960 / (G * D * 4) >= 8 ? 8 : 4;
  const int64_t blocks = num_seqs * a.num_kv_heads * a.splits;
  const int64_t sms = sm_count(device);
  const unsigned cluster = a.splits > 1 ? static_cast<unsigned>(a.splits) : 1u;
  const dim3 grid(static_cast<unsigned>(blocks));
  // not scheduled early behind the previous kernel: its CTAs take all of an SM's registers
  if (kMaxWarps >= 16 && blocks <= sms && split_tiles >= 16) {
    return launch_serialized(decode_attention_kernel<D, G, (kMaxWarps >= 16 ? 16 : 4)>, grid,
                             dim3((kMaxWarps >= 16 ? 16 : 4) * kWarpSize), 0, stream, cluster, a);
  }
  if (kMaxWarps >= 8 && blocks <= 2 * sms && split_tiles >= 8) {
    return launch_serialized(decode_attention_kernel<D, G, (kMaxWarps >= 8 ? 8 : 4)>, grid,
                             dim3((kMaxWarps >= 8 ? 8 : 4) * kWarpSize), 0, stream, cluster, a);
  }
  return launch_serialized(decode_attention_kernel<D, G, 4>, grid, dim3(4 * kWarpSize), 0, stream,
                           cluster, a);
}

template <int D>
int dispatch_group(const AttnArgs& a, int64_t num_seqs, int64_t split_tiles, int group,
                   int device, cudaStream_t stream) {
  switch (group) {
    case 1: return launch_attention<D, 1>(a, num_seqs, split_tiles, device, stream);
    case 2: return launch_attention<D, 2>(a, num_seqs, split_tiles, device, stream);
    case 4: return launch_attention<D, 4>(a, num_seqs, split_tiles, device, stream);
    case 8: return launch_attention<D, 8>(a, num_seqs, split_tiles, device, stream);
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
  // the reciprocal of the block size for the page lookup: shift = ceil(log2 block_size),
  // magic = floor(2^32 (2^shift - block_size) / block_size) + 1
  int shift = 0;
  while ((int64_t{1} << shift) < block_size) ++shift;
  a.page_shift = shift;
  a.page_magic = static_cast<uint32_t>(
      ((uint64_t{1} << 32) * ((uint64_t{1} << shift) - static_cast<uint64_t>(block_size))) /
          static_cast<uint64_t>(block_size) + 1);
  a.num_kv_heads = static_cast<int>(num_kv_heads);
  a.scale_log2 = static_cast<float>(static_cast<double>(scale) / std::log(2.0));
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
  // tiles of 16 cache rows per split of the longest request
  const int64_t split_tiles = ((max_seq_len + 15) / 16 + pow2 - 1) / pow2;
  return head_dim == 128
             ? dispatch_group<128>(a, num_seqs, split_tiles, static_cast<int>(group), device, s)
             : dispatch_group<64>(a, num_seqs, split_tiles, static_cast<int>(group), device, s);
}

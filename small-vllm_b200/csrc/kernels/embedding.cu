// Token-embedding gather: out[t] = table[ids[t]], a bit-exact row copy of any element size.
//
// The reference loads the table (model.embed_tokens.weight, [vocab, hidden]; small-vLLM
// tests/cpp/safetensors_test.cpp:161-162) but has no gather yet; ids are int32 as its tokenizer
// returns them (src/tokenizer/tokenizer.h:22) or int64 as torch callers pass them.
//
//   * Bulk-copy path: the data never passes through registers. Each warp owns a ring of
//     shared-memory stages and a contiguous range of tokens; lane 0 loads table rows with
//     cp.async.bulk (completing on the stage's mbarrier) and writes each landed row to its
//     output row with a bulk shared->global store, refilling a stage once the store that read it
//     has drained. The warp's 32 lanes fetch ids 32 at a time (coalesced, three batches ahead) and
//     hand them to lane 0 by shuffle.
//   * Vocabulary buckets: when the batch has at least half a token per table row, the warp
//     walks its tokens in `passes` rounds and round p copies only the tokens whose id lies in
//     the p-th slice of the vocabulary. The whole grid then reads from one L2-sized slice of the
//     table at a time, so repeated rows come from L2 instead of HBM (at 1M tokens over a
//     151,936-row table each row is read ~6.9 times). Output rows are written where they belong,
//     so the result does not depend on the order. Table loads carry an L2 evict-last policy and
//     the output stores an evict-first one, so the stream of output rows does not push the slice
//     out of L2.
//   * An id outside [0, vocab) zeroes its row and raises SVLLM_DEVERR_BAD_INDEX; nothing faults.
//   * Plain path for unaligned or odd-sized rows: one warp per row, element copies.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "host_common.h"

namespace svllm::k {
namespace {

struct EmbArgs {
  void* out;
  const void* ids;
  const void* table;
  int64_t num_tokens;
  int64_t vocab;
  int64_t out_stride_bytes;
  int64_t table_stride_bytes;
  uint32_t row_bytes;
  int ids_i64;
  int elem_bytes;        // plain path: 2 or 4
  int* err;
  // bulk-copy path
  int stages;
  int stage_bytes;
  int ring_offset;       // after the mbarriers and the per-stage token slots
  int passes;            // vocabulary buckets, one per pass over the warp's tokens
  int early_dependents;  // let the next kernel be scheduled at this one's start
  int64_t bucket_rows;   // rows per bucket: ceil(vocab / passes)
};

__device__ __forceinline__ int64_t load_id(const void* ids, int is_i64, int64_t t) {
  return is_i64 ? static_cast<int64_t>(__ldg(static_cast<const long long*>(ids) + t))
                : static_cast<int64_t>(__ldg(static_cast<const int*>(ids) + t));
}

__global__ void __launch_bounds__(512) embedding_bulk_kernel(const EmbArgs a) {
  grid_dependency_wait();
  if (a.early_dependents) allow_dependents();
  extern __shared__ __align__(128) uint8_t smem[];
  const int warps = blockDim.x / kWarpSize;
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x % kWarpSize;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * a.stages;
  // the output row each stage holds (-1: nothing to store), written and read by lane 0 only
  int64_t* stage_token = reinterpret_cast<int64_t*>(smem) + (warps + warp) * a.stages;
  uint8_t* ring = smem + a.ring_offset + static_cast<size_t>(warp) * a.stages * a.stage_bytes;
  const uint64_t load_policy = l2_policy_evict_last();
  const uint64_t store_policy = l2_policy_evict_first();

  if (lane == 0) {
    for (int s = 0; s < a.stages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  int64_t t0, t1;
  partition(a.num_tokens, static_cast<int64_t>(gridDim.x) * warps,
            static_cast<int64_t>(blockIdx.x) * warps + warp, t0, t1);
  const int64_t n = t1 - t0;
  if (n <= 0) return;

  // The warp's tokens in pass order: pass p visits the tokens t0.. t1-1 whose id is in bucket p
  // (an id outside the table belongs to pass 0). `chunk` holds this lane's id in the current
  // 32-token chunk and next_chunk .. next3_chunk the three chunks after it in walk order (loads
  // three ahead, so the scan rarely waits on one: the gather at 1M tokens 9090 -> 9610 GB/s
  // against one ahead); `pending` the lanes of the current chunk still to be visited in this
  // pass. The bucket test compares the id with the pass's row range (no division).
  auto load_chunk = [&](int64_t base) -> int64_t {
    return base + lane < n ? load_id(a.ids, a.ids_i64, t0 + base + lane) : -1;
  };
  auto in_pass = [&](int64_t id, int pass) -> bool {
    if (id < 0 || id >= a.vocab) return pass == 0;
    const int64_t lo = pass * a.bucket_rows;
    return id >= lo && id < lo + a.bucket_rows;
  };
  auto after = [&](int64_t b) -> int64_t { return b + kWarpSize < n ? b + kWarpSize : 0; };
  int pass = 0;
  int64_t base = 0;
  int64_t chunk = load_chunk(0);
  int64_t ahead = after(0);
  int64_t next_chunk = load_chunk(ahead);
  ahead = after(ahead);
  int64_t next2_chunk = load_chunk(ahead);
  ahead = after(ahead);
  int64_t next3_chunk = load_chunk(ahead);
  uint32_t pending = __ballot_sync(0xffffffffu, base + lane < n && in_pass(chunk, 0));

  // Warp-collective: the next (token, id) in pass order; token -1 once every pass is done
  // (never reached when called at most n times, since every token is in exactly one pass).
  auto next = [&](int64_t& token, int64_t& id) {
    while (pending == 0) {
      if (pass >= a.passes) {
        token = -1;
        id = 0;
        return;
      }
      base += kWarpSize;
      if (base >= n) {
        base = 0;
        ++pass;
      }
      chunk = next_chunk;
      next_chunk = next2_chunk;
      next2_chunk = next3_chunk;
      ahead = after(ahead);
      next3_chunk = load_chunk(ahead);
      pending = __ballot_sync(0xffffffffu, base + lane < n && in_pass(chunk, pass));
    }
    const int l = __ffs(pending) - 1;
    pending &= pending - 1;
    id = __shfl_sync(0xffffffffu, chunk, l);
    token = t0 + base + l;
  };

  // Warp-collective: fills stage s with the next token's table row.
  auto refill = [&](int s) {
    int64_t token, id;
    next(token, id);
    uint8_t* st = ring + static_cast<size_t>(s) * a.stage_bytes;
    // The stage's previous row must have been read out by its bulk store before it is reused.
    if (lane == 0) {
      bulk_wait_read<1>();
      stage_token[s] = token;
    }
    if (token < 0) {
      if (lane == 0) mbar_arrive(&bars[s]);
    } else if (id >= 0 && id < a.vocab) {
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars[s], a.row_bytes);
        bulk_load_policy(st, static_cast<const uint8_t*>(a.table) + id * a.table_stride_bytes,
                         a.row_bytes, &bars[s], load_policy);
      }
    } else {
      __syncwarp();
      for (uint32_t b = lane * 16; b < a.row_bytes; b += kWarpSize * 16) {
        *reinterpret_cast<uint4*>(st + b) = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        raise_error(a.err, kErrBadIndex);
        mbar_arrive(&bars[s]);
      }
    }
  };

  for (int64_t j = 0; j < min(static_cast<int64_t>(a.stages), n); ++j) {
    refill(static_cast<int>(j));
  }

  int64_t j = 0;
  for (; j < n; ++j) {
    const int s = static_cast<int>(j % a.stages);
    const uint32_t parity = static_cast<uint32_t>((j / a.stages) & 1);
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bars[s], parity))) break;
    if (lane == 0 && stage_token[s] >= 0) {
      bulk_store_policy(static_cast<uint8_t*>(a.out) + stage_token[s] * a.out_stride_bytes,
                        ring + static_cast<size_t>(s) * a.stage_bytes, a.row_bytes,
                        store_policy);
      bulk_commit();
    }
    // Refill the stage of the previous row, whose store has had a row's time to drain.
    if (j >= 1 && j - 1 + a.stages < n) {
      refill(static_cast<int>((j - 1) % a.stages));
    }
  }

  if (j < n && lane == 0) {
    raise_error(a.err, kErrWaitTimeout);
    for (int64_t m = j; m < min(j + a.stages, n); ++m) {
      mbar_wait_bounded(&bars[m % a.stages], static_cast<uint32_t>((m / a.stages) & 1));
    }
  }
  if (lane == 0) bulk_wait_all();
  __syncwarp();
}

__global__ void __launch_bounds__(256) embedding_plain_kernel(const EmbArgs a) {
  grid_dependency_sync();
  const int lane = threadIdx.x % kWarpSize;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x / kWarpSize);
  const int64_t elems = a.row_bytes / a.elem_bytes;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x / kWarpSize) +
                   threadIdx.x / kWarpSize;
       t < a.num_tokens; t += warps_total) {
    const int64_t id = load_id(a.ids, a.ids_i64, t);
    const bool ok = id >= 0 && id < a.vocab;
    uint8_t* dst = static_cast<uint8_t*>(a.out) + t * a.out_stride_bytes;
    const uint8_t* src = static_cast<const uint8_t*>(a.table) + (ok ? id : 0) * a.table_stride_bytes;
    if (!ok && lane == 0) raise_error(a.err, kErrBadIndex);
    if (a.elem_bytes == 4) {
      for (int64_t i = lane; i < elems; i += kWarpSize) {
        reinterpret_cast<uint32_t*>(dst)[i] = ok ? reinterpret_cast<const uint32_t*>(src)[i] : 0u;
      }
    } else {
      for (int64_t i = lane; i < elems; i += kWarpSize) {
        reinterpret_cast<uint16_t*>(dst)[i] = ok ? reinterpret_cast<const uint16_t*>(src)[i] : 0;
      }
    }
  }
}

int launch_embedding(void* out, const void* ids, int id_type, const void* table,
                     int64_t num_tokens, int64_t vocab, int64_t hidden, int64_t out_stride,
                     int64_t table_stride, int* err, int elem_bytes, cudaStream_t stream) {
  if (num_tokens < 0 || vocab <= 0 || hidden <= 0 || out_stride < hidden ||
      table_stride < hidden || (id_type != SVLLM_INDEX_I32 && id_type != SVLLM_INDEX_I64)) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  if (num_tokens == 0) return SVLLM_OK;
  if (out == nullptr || ids == nullptr || table == nullptr) return SVLLM_ERR_INVALID_ARGUMENT;
  if (hidden * elem_bytes >= (1 << 30)) return SVLLM_ERR_TOO_LARGE;

  int device;
  if (current_device(&device) != SVLLM_OK) return SVLLM_ERR_CUDA;
  if (err == nullptr) err = library_error_word(device);
  if (err == nullptr) return SVLLM_ERR_CUDA;

  EmbArgs a{};
  a.out = out;
  a.ids = ids;
  a.table = table;
  a.num_tokens = num_tokens;
  a.vocab = vocab;
  a.out_stride_bytes = out_stride * elem_bytes;
  a.table_stride_bytes = table_stride * elem_bytes;
  a.row_bytes = static_cast<uint32_t>(hidden * elem_bytes);
  a.ids_i64 = id_type == SVLLM_INDEX_I64;
  a.elem_bytes = elem_bytes;
  a.err = err;

  const bool bulk_ok = aligned16(out) && aligned16(table) && a.row_bytes % 16 == 0 &&
                       a.out_stride_bytes % 16 == 0 && a.table_stride_bytes % 16 == 0;
  if (bulk_ok) {
    const PipelineShape shape = pipeline_shape(OpId::kEmbedding);
    a.stage_bytes = static_cast<int>(round_up(a.row_bytes, 128));
    // Vocabulary buckets of about kBucketBytes of table each (measured on a B200 at 1M tokens
    // of 2 KB rows over a 151,936-row table: 8 buckets 7.8, 16 8.5, 24 9.9, 32 9.4 TB/s of
    // algorithmic bytes). From half a token per table row on: at 131,072 tokens over that table
    // (a third of the reads repeat a row) 6.0 -> 6.5 TB/s. Below, the gather walks its tokens
    // once.
    constexpr int64_t kBucketBytes = 13ll << 20;
    constexpr int kMaxPasses = 64;
    const int64_t table_bytes = vocab * static_cast<int64_t>(a.row_bytes);
    a.passes = num_tokens * 2 >= vocab
                   ? static_cast<int>(std::min<int64_t>(
                         kMaxPasses, std::max<int64_t>(1, (table_bytes + kBucketBytes - 1) /
                                                              kBucketBytes)))
                   : 1;
    a.bucket_rows = (vocab + a.passes - 1) / a.passes;
    int warps = warps_for(num_tokens, shape.warps, device);
    int stages = shape.stages;
    // per stage: an mbarrier and the token slot (8 bytes each), then the row
    auto smem_for = [&](int w, int s) {
      return round_up(static_cast<int64_t>(w) * s * 16, 128) +
             static_cast<int64_t>(w) * s * a.stage_bytes;
    };
    while (smem_for(warps, stages) > static_cast<int64_t>(kMaxSmemPerCta) && stages > 2) --stages;
    while (smem_for(warps, stages) > static_cast<int64_t>(kMaxSmemPerCta) && warps > 1) --warps;
    if (smem_for(warps, stages) <= static_cast<int64_t>(kMaxSmemPerCta)) {
      a.stages = stages;
      a.ring_offset = static_cast<int>(round_up(static_cast<int64_t>(warps) * stages * 16, 128));
      const size_t smem = static_cast<size_t>(smem_for(warps, stages));
      const int threads = warps * kWarpSize;
      const int per_sm = blocks_per_sm(reinterpret_cast<const void*>(embedding_bulk_kernel),
                                       threads, smem, device);
      if (per_sm > 0) {
        const int64_t grid = persistent_grid((num_tokens + warps - 1) / warps, device, per_sm);
        a.early_dependents = early_dependents(num_tokens * static_cast<int64_t>(a.row_bytes) * 2);
        return launch(embedding_bulk_kernel, dim3(static_cast<unsigned>(grid)), dim3(threads),
                      smem, stream, 1, a);
      }
    }
  }

  const int64_t grid = persistent_grid((num_tokens + 7) / 8, device, 8);
  return launch(embedding_plain_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), 0, stream, 1,
                a);
}

}  // namespace
}  // namespace svllm::k

using svllm::k::launch_embedding;

extern "C" {

int svllm_embedding_bf16(void* out, const void* ids, int id_type, const void* table,
                         int64_t num_tokens, int64_t vocab_size, int64_t hidden,
                         int64_t out_row_stride, int64_t table_row_stride, int* err,
                         svllm_stream stream) {
  return launch_embedding(out, ids, id_type, table, num_tokens, vocab_size, hidden,
                          out_row_stride, table_row_stride, err, 2,
                          reinterpret_cast<cudaStream_t>(stream));
}

int svllm_embedding_f32(float* out, const void* ids, int id_type, const float* table,
                        int64_t num_tokens, int64_t vocab_size, int64_t hidden,
                        int64_t out_row_stride, int64_t table_row_stride, int* err,
                        svllm_stream stream) {
  return launch_embedding(out, ids, id_type, table, num_tokens, vocab_size, hidden,
                          out_row_stride, table_row_stride, err, 4,
                          reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

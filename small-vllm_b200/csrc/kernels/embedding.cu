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
//     has drained. The warp's 32 lanes fetch ids 32 at a time (coalesced, one batch ahead) and
//     hand them to lane 0 by shuffle.
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
  int ring_offset;
};

__device__ __forceinline__ int64_t load_id(const void* ids, int is_i64, int64_t t) {
  return is_i64 ? static_cast<int64_t>(__ldg(static_cast<const long long*>(ids) + t))
                : static_cast<int64_t>(__ldg(static_cast<const int*>(ids) + t));
}

__global__ void __launch_bounds__(512) embedding_bulk_kernel(const EmbArgs a) {
  grid_dependency_sync();
  extern __shared__ __align__(128) uint8_t smem[];
  const int warps = blockDim.x / kWarpSize;
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x % kWarpSize;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * a.stages;
  uint8_t* ring = smem + a.ring_offset + static_cast<size_t>(warp) * a.stages * a.stage_bytes;

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

  // ids of rows [base, base + 32) in `cur`, the next 32 in `nxt` (one lane each).
  auto load_batch = [&](int64_t base) -> int64_t {
    return base + lane < n ? load_id(a.ids, a.ids_i64, t0 + base + lane) : 0;
  };
  int64_t cur_base = 0;
  int64_t cur = load_batch(0);
  int64_t nxt = load_batch(kWarpSize);

  // Warp-collective: fills stage s with the table row of token index i (i increasing).
  auto refill = [&](int64_t i, int s) {
    while (i >= cur_base + kWarpSize) {
      cur = nxt;
      cur_base += kWarpSize;
      nxt = load_batch(cur_base + kWarpSize);
    }
    const int64_t id = __shfl_sync(0xffffffffu, cur, static_cast<int>(i - cur_base));
    uint8_t* st = ring + static_cast<size_t>(s) * a.stage_bytes;
    // The stage's previous row must have been read out by its bulk store before it is reused.
    if (lane == 0) bulk_wait_read<1>();
    if (id >= 0 && id < a.vocab) {
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars[s], a.row_bytes);
        bulk_load(st, static_cast<const uint8_t*>(a.table) + id * a.table_stride_bytes,
                  a.row_bytes, &bars[s]);
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
    refill(j, static_cast<int>(j));
  }

  int64_t j = 0;
  for (; j < n; ++j) {
    const int s = static_cast<int>(j % a.stages);
    const uint32_t parity = static_cast<uint32_t>((j / a.stages) & 1);
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bars[s], parity))) break;
    if (lane == 0) {
      bulk_store(static_cast<uint8_t*>(a.out) + (t0 + j) * a.out_stride_bytes,
                 ring + static_cast<size_t>(s) * a.stage_bytes, a.row_bytes);
      bulk_commit();
    }
    // Refill the stage of the previous row, whose store has had a row's time to drain.
    if (j >= 1 && j - 1 + a.stages < n) {
      refill(j - 1 + a.stages, static_cast<int>((j - 1) % a.stages));
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
    int warps = warps_for(num_tokens, shape.warps, device);
    int stages = shape.stages;
    auto smem_for = [&](int w, int s) {
      return round_up(static_cast<int64_t>(w) * s * 8, 128) +
             static_cast<int64_t>(w) * s * a.stage_bytes;
    };
    while (smem_for(warps, stages) > static_cast<int64_t>(kMaxSmemPerCta) && stages > 2) --stages;
    while (smem_for(warps, stages) > static_cast<int64_t>(kMaxSmemPerCta) && warps > 1) --warps;
    if (smem_for(warps, stages) <= static_cast<int64_t>(kMaxSmemPerCta)) {
      a.stages = stages;
      a.ring_offset = static_cast<int>(round_up(static_cast<int64_t>(warps) * stages * 8, 128));
      const size_t smem = static_cast<size_t>(smem_for(warps, stages));
      const int threads = warps * kWarpSize;
      const int per_sm = blocks_per_sm(reinterpret_cast<const void*>(embedding_bulk_kernel),
                                       threads, smem, device);
      if (per_sm > 0) {
        const int64_t grid = persistent_grid((num_tokens + warps - 1) / warps, device, per_sm);
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

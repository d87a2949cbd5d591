// Greedy sampling fused with the LM-head GEMM: ids[m] = argmax_n bf16(sum_k hidden[m, k] * W[n, k])
// (the tied-embedding LM head of the reference's src/model/config.h:28 followed by greedy
// sampling on GPU, docs/design-spec.md:28-29), without writing the logits to memory.
//
// A warp-specialised tcgen05 GEMM over a persistent grid, one CTA per SM:
//   * warp 0 (one lane): TMA producer. K-blocks of the MMA's A operand [128 rows x 64 k] and B
//     operand [N rows x 64 k] land in a shared-memory ring through tensor maps with the 128-byte
//     swizzle (rows past a matrix read as zeros).
//   * warp 1 (one lane): issues tcgen05.mma (M = 128, K = 16; bf16 in, fp32 out) into one of two
//     TMEM accumulators, and frees each smem stage with tcgen05.commit once the MMAs reading it
//     are done. Warp 1 also allocates the TMEM.
//   * warps 2-5: epilogue. tcgen05.ld brings the accumulator into registers 16 columns at a time;
//     each logit is rounded to bf16 (what a bf16 matmul would have stored) and the first maximum
//     is kept; each row's winner of a tile is merged into a 64-bit key per row with atomicMax.
//     The second accumulator lets the epilogue of one tile run under the MMAs of the next.
// Two orientations. Decode-sized batches (up to 64 tokens) put the vocabulary on the MMA's M
// and the tokens (rounded up to 16) on its N, so every A tile is 128 real rows of the weight;
// larger batches put the tokens on M and a vocabulary tile of BN rows on N.
// A second kernel turns each row's key into its id and clears the key, so the workspace is zero
// again for the next call. All kernels wait for their predecessor with griddepcontrol.
//
// Every mbarrier wait is bounded: a wait that runs out raises the timeout bit in the error word
// and an abort flag that ends every role's loop; the producer then waits (bounded) for the
// copies it issued, the MMA warp for its MMAs, and the TMEM is freed before the CTA exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "host_common.h"
#include "umma.cuh"

namespace svllm::k {
namespace {

constexpr int kBlockM = 128;           // UMMA M (one CTA, cta_group::1)
constexpr int kBlockK = 64;            // 64 bf16 = 128 bytes: one swizzle atom wide
constexpr int kUmmaK = 16;             // K per tcgen05.mma of kind::f16
constexpr int kMaxStages = 8;
constexpr int kMaxTokens = 256;        // the vocabulary-on-M orientation, tokens on N
// Batches up to this many rows take the vocabulary-on-M orientation (measured on a B200: at 64
// tokens it streams the weight at 5.5 TB/s; at 128 its per-token epilogue already costs more
// than the tokens-on-M kernel wastes on a part-empty row tile).
constexpr int64_t kSwapMaxRows = 64;
constexpr int kThreads = 192;          // 6 warps: producer, MMA, 4 epilogue
constexpr int kTmemColumns = 512;      // two accumulators at columns 0 and 256
constexpr int kAccStride = 256;
constexpr uint32_t kATileBytes = kBlockM * kBlockK * 2;
constexpr size_t kRingBudget = 200 * 1024;  // shared memory for the stage ring

struct LmHeadArgs {
  int64_t m;             // rows of hidden
  int64_t n;             // vocabulary
  int64_t k;             // hidden size
  uint64_t* keys;        // [m] workspace, zero on entry
  void* logits;          // optional [m, n] bf16 output (row stride logits_stride), or null
  int64_t logits_stride;
  int* err;
  int stages;            // depth of the stage ring
  int n_tok;             // tokens on the MMA's N (vocabulary-on-M orientation)
};

// The order of a bf16-rounded logit: larger values higher, -0 == +0, every NaN highest; 0 is
// below every value (-inf maps to 0x007FFFFF).
__device__ __forceinline__ uint32_t value_order(float v) {
  if (v != v) return 0xFFFFFFFFu;
  uint32_t bits = __float_as_uint(v);
  if (v == 0.0f) bits = 0;
  return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}

// (value, index) as one integer: a larger value wins, then the lower index (torch.argmax on bf16
// logits). 0 is below every key.
__device__ __forceinline__ uint64_t argmax_key(float v, int64_t n) {
  return (static_cast<uint64_t>(value_order(v)) << 32) |
         (0xFFFFFFFFu - static_cast<uint32_t>(n));
}

__device__ __forceinline__ float round_bf16(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

__device__ __forceinline__ float max_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// The shared-memory state of one CTA's pipeline.
struct Sync {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint64_t epilogue;  // the four epilogue warps meet here once per tile
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void sync_init(Sync& sy, int stages) {
  for (int s = 0; s < stages; ++s) {
    mbar_init(&sy.full[s], 1);
    mbar_init(&sy.empty[s], 1);
  }
  for (int b = 0; b < 2; ++b) {
    mbar_init(&sy.tfull[b], 1);
    mbar_init(&sy.tempty[b], 4 * kWarpSize);
  }
  mbar_init(&sy.drain, 1);
  mbar_init(&sy.epilogue, 4 * kWarpSize);
  sy.abort = 0;
  fence_mbar_init();
}

// Producer (one lane): for every tile of this CTA, num_kb k-blocks of the MMA's A operand
// (kBlockM rows from row a_row of map_a) and B operand (b_rows rows from row b_row of map_b).
template <class TileRows>
__device__ void produce(Sync& sy, uint8_t* ring, int stages, uint32_t stage_bytes,
                        const CUtensorMap* map_a, const CUtensorMap* map_b, int64_t tiles,
                        int num_kb, TileRows tile_rows, int* err) {
  volatile int* abort = &sy.abort;
  int stage = 0;
  uint32_t phase = 0;
  int64_t issued = 0;
  bool ok = true;
  for (int64_t t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
    int32_t a_row, b_row;
    tile_rows(t, a_row, b_row);
    for (int kb = 0; kb < num_kb; ++kb) {
      if (!wait_phase(&sy.empty[stage], phase ^ 1, abort, err)) {
        ok = false;
        break;
      }
      uint8_t* st = ring + static_cast<size_t>(stage) * stage_bytes;
      mbar_arrive_expect_tx(&sy.full[stage], stage_bytes);
      tma_load_2d(st, map_a, kb * kBlockK, a_row, &sy.full[stage]);
      tma_load_2d(st + kATileBytes, map_b, kb * kBlockK, b_row, &sy.full[stage]);
      ++issued;
      if (++stage == stages) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
  // every copy this CTA issued has landed before it may exit: the last use of each slot
  for (int64_t j = issued - 1; j >= 0 && j >= issued - stages; --j) {
    mbar_wait_bounded(&sy.full[j % stages], static_cast<uint32_t>((j / stages) & 1));
  }
}

// MMA issuer (one lane): per tile, num_kb k-blocks of 4 tcgen05.mma into accumulator acc.
__device__ void mma_loop(Sync& sy, uint8_t* ring, int stages, uint32_t stage_bytes,
                         uint32_t idesc, int64_t tiles, int num_kb, int* err) {
  volatile int* abort = &sy.abort;
  int stage = 0;
  uint32_t phase = 0;
  int acc = 0;
  uint32_t acc_phase = 0;
  bool ok = true;
  for (int64_t t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
    if (!wait_phase(&sy.tempty[acc], acc_phase ^ 1, abort, err)) break;
    tc_fence_after();
    const uint32_t d_tmem = sy.tmem_base + acc * kAccStride;
    for (int kb = 0; kb < num_kb; ++kb) {
      if (!wait_phase(&sy.full[stage], phase, abort, err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint8_t* st = ring + static_cast<size_t>(stage) * stage_bytes;
      const uint64_t a_desc = smem_desc_k_sw128(st);
      const uint64_t b_desc = smem_desc_k_sw128(st + kATileBytes);
#pragma unroll
      for (int kk = 0; kk < kBlockK / kUmmaK; ++kk) {
        // K advances by 16 bf16 (32 bytes) inside the swizzle atom: the start address moves
        const uint64_t step = static_cast<uint64_t>((kk * kUmmaK * 2) >> 4);
        umma_bf16(d_tmem, a_desc + step, b_desc + step, idesc, (kb | kk) != 0);
      }
      umma_commit(&sy.empty[stage]);  // the slot is free once these MMAs have read it
      if (++stage == stages) {
        stage = 0;
        phase ^= 1;
      }
    }
    if (!ok) break;
    umma_commit(&sy.tfull[acc]);  // the accumulator is complete
    acc ^= 1;
    if (acc == 0) acc_phase ^= 1;
  }
  // every MMA this thread issued has completed before the TMEM is freed
  umma_commit(&sy.drain);
  mbar_wait_bounded(&sy.drain, 0);
}

// Token rows as the MMA's M (128 per tile), BN vocabulary rows as its N: for larger batches.
// TMEM lane = token row, column = vocabulary entry; each epilogue thread owns one token row.
template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    lm_head_argmax_kernel(const __grid_constant__ CUtensorMap map_a,
                          const __grid_constant__ CUtensorMap map_b, const LmHeadArgs a) {
  grid_dependency_sync();
  constexpr uint32_t kStageBytes = kATileBytes + BN * kBlockK * 2;
  static_assert(kStageBytes % 1024 == 0, "1 KB-aligned stages");
  extern __shared__ uint8_t smem_raw[];
  __shared__ Sync sy;
  uint8_t* ring = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);

  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x % kWarpSize;
  const int64_t m_tiles = (a.m + kBlockM - 1) / kBlockM;
  const int64_t tiles = m_tiles * ((a.n + BN - 1) / BN);
  const int num_kb = static_cast<int>((a.k + kBlockK - 1) / kBlockK);
  const int stages = a.stages;

  if (threadIdx.x == 0) sync_init(sy, stages);
  if (warp == 1) tmem_alloc(&sy.tmem_base, kTmemColumns);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == 0) {
    if (lane == 0) {
      produce(sy, ring, stages, kStageBytes, &map_a, &map_b, tiles, num_kb,
              [&](int64_t t, int32_t& a_row, int32_t& b_row) {
                a_row = static_cast<int32_t>((t % m_tiles) * kBlockM);
                b_row = static_cast<int32_t>((t / m_tiles) * BN);
              },
              a.err);
    }
  } else if (warp == 1) {
    if (lane == 0) mma_loop(sy, ring, stages, kStageBytes, idesc_bf16(kBlockM, BN), tiles, num_kb, a.err);
  } else {
    // epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31, one token row per thread
    volatile int* abort = &sy.abort;
    const int quarter = warp % 4;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * kWarpSize) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
      const int64_t row0 = (t % m_tiles) * kBlockM + quarter * kWarpSize;
      const int64_t m = row0 + lane;
      const int64_t n0 = (t / m_tiles) * BN;
      const int valid_cols = static_cast<int>(a.n - n0 < BN ? a.n - n0 : BN);
      // the warp leaves together: tcgen05.ld below is warp-collective
      if (!__all_sync(0xffffffffu, wait_phase(&sy.tfull[acc], acc_phase, abort, a.err))) break;
      tc_fence_after();
      if (row0 < a.m) {  // warp-uniform: a quarter past the last token reads nothing
        // running first maximum of the bf16-rounded logits, 16 columns at a time: the chunk's
        // maximum (rounding is monotonic) decides whether to look for its first index
        float best = -__builtin_huge_valf();
        int best_c = 0;
        __nv_bfloat16* lrow = a.logits != nullptr && m < a.m
                                  ? static_cast<__nv_bfloat16*>(a.logits) + m * a.logits_stride + n0
                                  : nullptr;
#pragma unroll
        for (int c = 0; c < BN; c += 16) {
          uint32_t r[16];
          tmem_load16(sy.tmem_base + lane_base + acc * kAccStride + c, r);
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            v[j] = c + j < valid_cols ? __uint_as_float(r[j]) : -__builtin_huge_valf();
          }
          float cm = v[0];
#pragma unroll
          for (int j = 1; j < 16; ++j) cm = max_nan(cm, v[j]);
          const float cr = round_bf16(cm);
          if (cr > best || (cr != cr && best == best)) {
            int first = 15;
#pragma unroll
            for (int j = 15; j >= 0; --j) {
              const float f = round_bf16(v[j]);
              if (f == cr || (f != f && cr != cr)) first = j;
            }
            best = cr;
            best_c = c + first;
          }
          if (lrow != nullptr) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              if (c + j < valid_cols) lrow[c + j] = __float2bfloat16_rn(v[j]);
            }
          }
        }
        if (m < a.m) {
          atomicMax(reinterpret_cast<unsigned long long*>(a.keys + m),
                    static_cast<unsigned long long>(argmax_key(best, n0 + best_c)));
        }
      }
      tc_fence_before();
      mbar_arrive(&sy.tempty[acc]);  // the accumulator may be overwritten
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(sy.tmem_base, kTmemColumns);
}

// Vocabulary rows as the MMA's M (128 per tile), the tokens as its N (a.n_tok, 16 to 256, the
// batch rounded up to 16): for decode-sized batches, where every A tile is 128 real rows of the
// weight and the logits of a token are spread over the TMEM lanes. Each epilogue warp reduces
// its 32 lanes per token with two redux instructions; the four warps meet in shared memory
// (an mbarrier with a bounded wait) and one atomic per token and tile leaves the CTA.
__global__ void __launch_bounds__(kThreads, 1)
    lm_head_argmax_swap_kernel(const __grid_constant__ CUtensorMap map_w,
                               const __grid_constant__ CUtensorMap map_h, const LmHeadArgs a) {
  grid_dependency_sync();
  extern __shared__ uint8_t smem_raw[];
  __shared__ Sync sy;
  __shared__ uint64_t warp_keys[2][4][kMaxTokens];  // per accumulator buffer
  uint8_t* ring = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);

  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x % kWarpSize;
  const int n_tok = a.n_tok;
  const uint32_t stage_bytes = kATileBytes + static_cast<uint32_t>(n_tok) * kBlockK * 2;
  const int64_t tiles = (a.n + kBlockM - 1) / kBlockM;
  const int num_kb = static_cast<int>((a.k + kBlockK - 1) / kBlockK);
  const int stages = a.stages;

  if (threadIdx.x == 0) sync_init(sy, stages);
  if (warp == 1) tmem_alloc(&sy.tmem_base, kTmemColumns);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == 0) {
    if (lane == 0) {
      produce(sy, ring, stages, stage_bytes, &map_w, &map_h, tiles, num_kb,
              [](int64_t t, int32_t& a_row, int32_t& b_row) {
                a_row = static_cast<int32_t>(t * kBlockM);
                b_row = 0;
              },
              a.err);
    }
  } else if (warp == 1) {
    if (lane == 0) mma_loop(sy, ring, stages, stage_bytes, idesc_bf16(kBlockM, n_tok), tiles, num_kb, a.err);
  } else {
    volatile int* abort = &sy.abort;
    const int quarter = warp % 4;
    const int e = threadIdx.x - 2 * kWarpSize;  // 0..127 among the epilogue threads
    const uint32_t lane_base = static_cast<uint32_t>(quarter * kWarpSize) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t epi_phase = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
      const int64_t n = t * kBlockM + quarter * kWarpSize + lane;  // this lane's vocab row
      const bool valid = n < a.n;
      // the warp leaves together: tcgen05.ld below is warp-collective
      if (!__all_sync(0xffffffffu, wait_phase(&sy.tfull[acc], acc_phase, abort, a.err))) break;
      tc_fence_after();
      for (int c = 0; c < n_tok; c += 16) {
        uint32_t r[16];
        tmem_load16(sy.tmem_base + lane_base + acc * kAccStride + c, r);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float f = round_bf16(__uint_as_float(r[j]));
          const uint32_t order = valid ? value_order(f) : 0u;
          const uint32_t hi = __reduce_max_sync(0xffffffffu, order);
          const uint32_t lo = __reduce_max_sync(
              0xffffffffu, valid && order == hi ? 0xFFFFFFFFu - static_cast<uint32_t>(n) : 0u);
          if (lane == 0) warp_keys[acc][quarter][c + j] = (static_cast<uint64_t>(hi) << 32) | lo;
          if (a.logits != nullptr && valid && c + j < a.m) {
            static_cast<__nv_bfloat16*>(a.logits)[(c + j) * a.logits_stride + n] =
                __float2bfloat16_rn(__uint_as_float(r[j]));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&sy.tempty[acc]);  // the accumulator may be overwritten
      // every warp's keys are in shared memory (a bounded wait: a warp that left on an abort
      // must not hold the others); the buffer is rewritten two tiles later, after the next
      // meeting, by when every thread has finished reading it
      mbar_arrive(&sy.epilogue);
      if (!__all_sync(0xffffffffu, wait_phase(&sy.epilogue, epi_phase, abort, a.err))) break;
      epi_phase ^= 1;
      for (int j = e; j < n_tok && j < a.m; j += 4 * kWarpSize) {
        uint64_t key = warp_keys[acc][0][j];
#pragma unroll
        for (int q = 1; q < 4; ++q) {
          key = warp_keys[acc][q][j] > key ? warp_keys[acc][q][j] : key;
        }
        if (key != 0) atomicMax(reinterpret_cast<unsigned long long*>(a.keys + j),
                                static_cast<unsigned long long>(key));
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(sy.tmem_base, kTmemColumns);
}

// ids[m] from the row's key; the key returns to zero for the next call.
__global__ void __launch_bounds__(256) lm_head_argmax_finish_kernel(uint64_t* keys, int64_t m,
                                                                     int64_t* ids) {
  grid_dependency_sync();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < m;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint64_t key = keys[i];
    ids[i] = key == 0 ? 0 : static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(key));
    keys[i] = 0;
  }
}

// ---------------------------------------------------------------------------------------------
// Host side

int ring_stages(uint32_t stage_bytes) {
  const int stages = static_cast<int>(kRingBudget / stage_bytes);
  return stages < kMaxStages ? stages : kMaxStages;
}

template <int BN>
int launch_gemm(const void* hidden, int64_t hidden_stride, const void* weight,
                int64_t weight_stride, LmHeadArgs a, int device, cudaStream_t stream) {
  CUtensorMap map_a, map_b;
  if (!make_map(&map_a, hidden, a.m, a.k, hidden_stride, kBlockM) ||
      !make_map(&map_b, weight, a.n, a.k, weight_stride, BN)) {
    return SVLLM_ERR_UNSUPPORTED;
  }
  const uint32_t stage_bytes = kATileBytes + BN * kBlockK * 2;
  a.stages = ring_stages(stage_bytes);
  const size_t smem = 1024 + static_cast<size_t>(a.stages) * stage_bytes;
  const void* fn = reinterpret_cast<const void*>(lm_head_argmax_kernel<BN>);
  if (blocks_per_sm(fn, kThreads, smem, device) < 1) return SVLLM_ERR_UNSUPPORTED;
  const int64_t tiles = ((a.m + kBlockM - 1) / kBlockM) * ((a.n + BN - 1) / BN);
  const int64_t grid = tiles < sm_count(device) ? tiles : sm_count(device);
  return launch(lm_head_argmax_kernel<BN>, dim3(static_cast<unsigned>(grid)), dim3(kThreads),
                smem, stream, 1, map_a, map_b, a);
}

int launch_swap(const void* hidden, int64_t hidden_stride, const void* weight,
                int64_t weight_stride, LmHeadArgs a, int device, cudaStream_t stream) {
  a.n_tok = static_cast<int>(round_up(a.m, 16));
  CUtensorMap map_w, map_h;
  if (!make_map(&map_w, weight, a.n, a.k, weight_stride, kBlockM) ||
      !make_map(&map_h, hidden, a.m, a.k, hidden_stride, a.n_tok)) {
    return SVLLM_ERR_UNSUPPORTED;
  }
  const uint32_t stage_bytes = kATileBytes + static_cast<uint32_t>(a.n_tok) * kBlockK * 2;
  a.stages = ring_stages(stage_bytes);
  const size_t smem = 1024 + static_cast<size_t>(a.stages) * stage_bytes;
  const void* fn = reinterpret_cast<const void*>(lm_head_argmax_swap_kernel);
  if (blocks_per_sm(fn, kThreads, smem, device) < 1) return SVLLM_ERR_UNSUPPORTED;
  const int64_t tiles = (a.n + kBlockM - 1) / kBlockM;
  const int64_t grid = tiles < sm_count(device) ? tiles : sm_count(device);
  return launch(lm_head_argmax_swap_kernel, dim3(static_cast<unsigned>(grid)), dim3(kThreads),
                smem, stream, 1, map_w, map_h, a);
}

// The N tile whose last wave of tiles is fullest: per-CTA columns = waves * BN, smallest wins.
int pick_bn(int64_t m, int64_t n, int sms) {
  static constexpr int kChoices[] = {256, 224, 208, 192, 160, 128};
  const int64_t m_tiles = (m + kBlockM - 1) / kBlockM;
  int best = kChoices[0];
  int64_t best_cost = INT64_MAX;
  for (const int bn : kChoices) {
    const int64_t tiles = m_tiles * ((n + bn - 1) / bn);
    const int64_t cost = (tiles + sms - 1) / sms * bn;
    if (cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

// Size checks shared by both entry points (SVLLM_OK: the arguments describe a valid call).
int check_lm_head_sizes(int64_t num_rows, int64_t hidden_size, int64_t hidden_stride,
                        int64_t vocab, int64_t weight_stride, const void* logits,
                        int64_t logits_stride) {
  if (num_rows < 0 || hidden_size <= 0 || vocab <= 0 || hidden_stride < hidden_size ||
      weight_stride < hidden_size || vocab >= (int64_t{1} << 31) ||
      num_rows >= (int64_t{1} << 31) || (logits != nullptr && logits_stride < vocab)) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  return SVLLM_OK;
}

// Pointer checks shared by both entry points: present, and the 16-byte aligned bases and row
// strides the tensor maps want.
int check_lm_head_operands(const void* hidden, int64_t hidden_stride, const void* weight,
                           int64_t weight_stride, const int64_t* out_ids) {
  if (hidden == nullptr || weight == nullptr || out_ids == nullptr) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  if (!aligned16(hidden) || !aligned16(weight) || (hidden_stride * 2) % 16 != 0 ||
      (weight_stride * 2) % 16 != 0) {
    return SVLLM_ERR_UNSUPPORTED;
  }
  return SVLLM_OK;
}

// The GEMM with its argmax epilogue into `keys` (num_rows zeroed 8-byte keys), then the kernel
// that turns keys into ids and zeroes them again. Arguments already checked.
int run_lm_head_argmax(const void* hidden, int64_t num_rows, int64_t hidden_size,
                       int64_t hidden_stride, const void* weight, int64_t vocab,
                       int64_t weight_stride, int64_t* out_ids, void* logits,
                       int64_t logits_stride, uint64_t* keys, int device, int* err,
                       cudaStream_t s) {
  LmHeadArgs a{};
  a.m = num_rows;
  a.n = vocab;
  a.k = hidden_size;
  a.keys = keys;
  a.logits = logits;
  a.logits_stride = logits_stride;
  a.err = err;
  int status;
  if (num_rows <= kSwapMaxRows) {
    status = launch_swap(hidden, hidden_stride, weight, weight_stride, a, device, s);
  } else switch (pick_bn(num_rows, vocab, sm_count(device))) {
    case 256: status = launch_gemm<256>(hidden, hidden_stride, weight, weight_stride, a, device, s); break;
    case 224: status = launch_gemm<224>(hidden, hidden_stride, weight, weight_stride, a, device, s); break;
    case 208: status = launch_gemm<208>(hidden, hidden_stride, weight, weight_stride, a, device, s); break;
    case 192: status = launch_gemm<192>(hidden, hidden_stride, weight, weight_stride, a, device, s); break;
    case 160: status = launch_gemm<160>(hidden, hidden_stride, weight, weight_stride, a, device, s); break;
    default: status = launch_gemm<128>(hidden, hidden_stride, weight, weight_stride, a, device, s); break;
  }
  if (status != SVLLM_OK) return status;
  const int64_t blocks = (num_rows + 255) / 256;
  return launch(lm_head_argmax_finish_kernel, dim3(static_cast<unsigned>(blocks < 1024 ? blocks : 1024)),
                dim3(256), 0, s, 1, keys, num_rows, out_ids);
}

}  // namespace
}  // namespace svllm::k

extern "C" int svllm_lm_head_argmax_bf16(const void* hidden, int64_t num_rows,
                                         int64_t hidden_size, int64_t hidden_stride,
                                         const void* weight, int64_t vocab, int64_t weight_stride,
                                         int64_t* out_ids, void* logits, int64_t logits_stride,
                                         void* workspace, int64_t workspace_bytes,
                                         svllm_stream stream) {
  using namespace svllm::k;
  int status = check_lm_head_sizes(num_rows, hidden_size, hidden_stride, vocab, weight_stride,
                                   logits, logits_stride);
  if (status != SVLLM_OK) return status;
  if (num_rows == 0) return SVLLM_OK;
  if (workspace == nullptr || workspace_bytes < num_rows * static_cast<int64_t>(sizeof(uint64_t))) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  status = check_lm_head_operands(hidden, hidden_stride, weight, weight_stride, out_ids);
  if (status != SVLLM_OK) return status;
  if ((reinterpret_cast<uintptr_t>(workspace) & 7u) != 0) return SVLLM_ERR_UNSUPPORTED;  // 8-byte keys
  int device;
  if (current_device(&device) != SVLLM_OK) return SVLLM_ERR_CUDA;
  int* err = library_error_word(device);
  if (err == nullptr) return SVLLM_ERR_CUDA;
  return run_lm_head_argmax(hidden, num_rows, hidden_size, hidden_stride, weight, vocab,
                            weight_stride, out_ids, logits, logits_stride,
                            static_cast<uint64_t*>(workspace), device, err,
                            reinterpret_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------------------------
// The same LM head and greedy sampling without a caller workspace: the per-row keys live in a
// file-scope array of this library. It serves callers that cannot allocate device memory, such
// as a host program driving this C ABI through an FFI (ctypes, cgo, JNI) that has no CUDA
// allocator of its own, or one whose device memory is entirely owned by another allocator.

namespace svllm::k {

// At most this many rows per call: 4096 keys of 8 bytes, 32 KB that every GPU which loads the
// library holds until the process exits.
constexpr int64_t kStaticScratchRows = 4096;

// The keys of svllm_lm_head_argmax_static_bf16. They must be zero when the GEMM starts; each
// call clears the rows it uses first, and its last kernel clears them again.
static __device__ __align__(256) uint64_t g_lm_head_static_keys[kStaticScratchRows];

namespace {

std::atomic<uint64_t*> g_static_keys_address[kMaxDevices];

// The device address of g_lm_head_static_keys on `device` (the current device), looked up once
// per device; null if the lookup fails.
uint64_t* static_keys(int device) {
  uint64_t* p = g_static_keys_address[device].load(std::memory_order_acquire);
  if (p == nullptr) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_lm_head_static_keys) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    p = static_cast<uint64_t*>(addr);
    g_static_keys_address[device].store(p, std::memory_order_release);
  }
  return p;
}

}  // namespace
}  // namespace svllm::k

extern "C" int svllm_lm_head_argmax_static_bf16(const void* hidden, int64_t num_rows,
                                                int64_t hidden_size, int64_t hidden_stride,
                                                const void* weight, int64_t vocab,
                                                int64_t weight_stride, int64_t* out_ids,
                                                void* logits, int64_t logits_stride,
                                                svllm_stream stream) {
  using namespace svllm::k;
  int status = check_lm_head_sizes(num_rows, hidden_size, hidden_stride, vocab, weight_stride,
                                   logits, logits_stride);
  if (status != SVLLM_OK) return status;
  if (num_rows > kStaticScratchRows) return SVLLM_ERR_TOO_LARGE;
  if (num_rows == 0) return SVLLM_OK;
  status = check_lm_head_operands(hidden, hidden_stride, weight, weight_stride, out_ids);
  if (status != SVLLM_OK) return status;
  int device;
  if (current_device(&device) != SVLLM_OK) return SVLLM_ERR_CUDA;
  int* err = library_error_word(device);
  uint64_t* keys = static_keys(device);  // the first call on a device looks it up
  if (err == nullptr || keys == nullptr) return SVLLM_ERR_CUDA;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // The finish kernel leaves every key it read at zero, so after a completed call the rows are
  // clear already. This clear is for the cases where they are not: an earlier call whose kernels
  // stopped early (a wait that timed out) or that overlapped this one on another stream. In a
  // captured decode graph it is one memset node per step, ahead of the GEMM, and it keeps the
  // GEMM from being scheduled early behind the kernel before it.
  if (cudaMemsetAsync(keys, 0, static_cast<size_t>(num_rows) * sizeof(uint64_t), s) !=
      cudaSuccess) {
    cudaGetLastError();
    return SVLLM_ERR_CUDA;
  }
  return run_lm_head_argmax(hidden, num_rows, hidden_size, hidden_stride, weight, vocab,
                            weight_stride, out_ids, logits, logits_stride, keys, device, err, s);
}

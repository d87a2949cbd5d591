// SiLU(gate) * up for bf16 and fp32.
//
// The reference has no kernel (planned at small-vLLM docs/ROADMAP.md:40, "SiLU-and-mul"); the
// formula is Hugging Face's MLP, act_fn(gate_proj(x)) * up_proj(x), evaluated as torch does it:
// silu(g) = g / (1 + exp(-g)) in fp32 with the CUDA math library's accurate expf and an IEEE
// division, rounded to the activation dtype, then multiplied by up and rounded again. On one
// GPU the result therefore equals the torch composite bit for bit.
//
//   * Bulk-copy path: the op is elementwise, so a unit is a chunk of columns. When gate, up and
//     out are all contiguous the whole batch is one flat row and chunks cross row boundaries;
//     otherwise (gate and up as the two halves of one [rows, 2 * inter] tensor, say) chunks stay
//     inside a row. Each warp owns a ring of stages; lane 0 keeps cp.async.bulk loads of the
//     next chunks of gate and up in flight, and the warp writes 16-byte vectors of out.
//   * Table path (bf16, larger batches): a bf16 gate takes only 65536 values, so
//     round(silu(g)) is a function of the gate's 16 bits. A one-time kernel per device evaluates
//     it for every bf16 pattern, with the same expf / IEEE-division code, into a 128 KB table in
//     device memory and then publishes it (a release store of a ready flag). Each CTA of a
//     table-path launch copies the published table into shared memory, then streams with one
//     table load and one packed bf16 multiply per element instead of ~30 instructions of
//     accurate math: identical results, a fraction of the issue slots. A CTA that finds the
//     table not yet published (the build still queued on another stream) computes directly.
//   * Plain path for unaligned or odd-sized rows: grid-stride element loop, still on the GPU.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>

#include "common.cuh"
#include "host_common.h"

namespace svllm::k {
namespace {

struct SiluArgs {
  void* out;
  const void* gate;
  const void* up;
  int64_t rows;          // rows of the chunked view (1 when the batch is flat)
  int64_t cols;          // elements per row of the chunked view
  int64_t out_stride;    // elements
  int64_t gate_stride;
  int64_t up_stride;
  int* err;
  // bulk-copy path
  int64_t chunk;         // elements per unit
  int stages;
  int stage_bytes;       // gate chunk, then up chunk
  int table_offset;      // table path: byte offset of the 65536-entry table
  int interleave;        // unit order (WarpUnits)
  int early_dependents;  // let the next kernel be scheduled at this one's start
  int ring_offset;
};

constexpr int kTableEntries = 65536;  // one per bf16 bit pattern
constexpr int kTableBytes = kTableEntries * 2;
// The table path from this many elements per SM (measured on a B200 at 3072 columns: direct
// math wins at 1024 tokens, 21k elements per SM, 7.5 us; the table at 2048 tokens, 10.1 us
// against 11.9 us direct at 1536; from 4096 tokens on it saves 25-40%).
constexpr int64_t kTableMinElementsPerSm = 24576;

// round(silu(g)) for every bf16 pattern g, two per word (low half: the even pattern), built
// once per device by silu_table_build_kernel; g_silu_table_ready turns 1 when it is complete.
// Read-only after that; it never changes, so every launch on every stream may share it.
__device__ __align__(256) uint32_t g_silu_table[kTableEntries / 2];
__device__ int g_silu_table_ready = 0;

// Whether the table build has been enqueued on each device (host side).
std::atomic<bool> g_silu_table_launched[kMaxDevices];

__device__ __forceinline__ float silu(float g) {
  return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
}

// out = round(round(silu(g)) * u) for one 16-byte vector of gate and of up.
template <class E>
__device__ __forceinline__ uint4 silu_mul_vec(const uint4& g, const uint4& u);

template <>
__device__ __forceinline__ uint4 silu_mul_vec<Bf16>(const uint4& g, const uint4& u) {
  float f[8];
  unpack<Bf16>(g, f);
  uint32_t s[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) s[i] = pack_bf16x2(silu(f[2 * i]), silu(f[2 * i + 1]));
  return make_uint4(bf16x2_mul(s[0], u.x), bf16x2_mul(s[1], u.y), bf16x2_mul(s[2], u.z),
                    bf16x2_mul(s[3], u.w));
}

template <>
__device__ __forceinline__ uint4 silu_mul_vec<F32>(const uint4& g, const uint4& u) {
  float f[4], uf[4];
  unpack<F32>(g, f);
  unpack<F32>(u, uf);
#pragma unroll
  for (int e = 0; e < 4; ++e) f[e] = __fmul_rn(silu(f[e]), uf[e]);
  return pack<F32>(f);
}

// out = round(table[g] * u) for one 16-byte vector, table[g] = round(silu(g)) for bf16 g.
__device__ __forceinline__ uint4 silu_mul_vec_table(const uint4& g, const uint4& u,
                                                    const uint16_t* table) {
  uint32_t y[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w = word(g, i);
    const uint32_t s = static_cast<uint32_t>(table[w & 0xffffu]) |
                       (static_cast<uint32_t>(table[w >> 16]) << 16);
    y[i] = bf16x2_mul(s, word(u, i));
  }
  return make_uint4(y[0], y[1], y[2], y[3]);
}

__device__ __forceinline__ uint32_t silu_table_word(int w) {
  const float g0 = __uint_as_float(static_cast<uint32_t>(2 * w) << 16);
  const float g1 = __uint_as_float(static_cast<uint32_t>(2 * w + 1) << 16);
  return pack_bf16x2(silu(g0), silu(g1));
}

__global__ void __launch_bounds__(1024) silu_table_build_kernel() {
  grid_dependency_sync();
  for (int w = threadIdx.x; w < kTableEntries / 2; w += blockDim.x) {
    g_silu_table[w] = silu_table_word(w);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(&g_silu_table_ready), "r"(1)
                 : "memory");
  }
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <class E, bool kTable>
__global__ void __launch_bounds__(512) silu_bulk_kernel(const SiluArgs a) {
  grid_dependency_wait();
  if (a.early_dependents) allow_dependents();
  using S = typename E::Storage;
  constexpr int kVec = E::kPerVec;
  static_assert(!kTable || sizeof(S) == 2, "the table path is for bf16");
  extern __shared__ __align__(128) uint8_t smem[];

  const int warps = blockDim.x / kWarpSize;
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x % kWarpSize;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * a.stages;
  uint8_t* ring = smem + a.ring_offset + static_cast<size_t>(warp) * a.stages * a.stage_bytes;
  const uint32_t half_stage = static_cast<uint32_t>(a.chunk * sizeof(S));
  const uint16_t* table = reinterpret_cast<const uint16_t*>(smem + a.table_offset);

  if (lane == 0) {
    for (int s = 0; s < a.stages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __shared__ int ready;
  __shared__ __align__(8) uint64_t table_bar;
  bool use_table = false;
  bool table_copy_pending = false;  // a table copy this CTA must see land before it exits
  if constexpr (kTable) {
    // The published table, one bulk copy into shared memory; before it is published, direct
    // math.
    if (threadIdx.x == 0) {
      ready = ld_acquire_gpu(&g_silu_table_ready);
      if (ready) {
        mbar_init(&table_bar, 1);
        fence_mbar_init();
        // the table's generic-proxy writes, acquired above, ordered before the async-proxy read
        asm volatile("fence.proxy.async.global;" ::: "memory");
        mbar_arrive_expect_tx(&table_bar, kTableBytes);
        bulk_load(smem + a.table_offset, g_silu_table, kTableBytes, &table_bar);
      }
    }
    __syncthreads();
    use_table = ready != 0 && __syncthreads_and(mbar_wait_bounded(&table_bar, 0));
    if (ready && !use_table) {
      // the copy did not land in time: direct math, and the copy is waited for before exit
      table_copy_pending = true;
      if (threadIdx.x == 0) raise_error(a.err, kErrWaitTimeout);
    }
  } else {
    __syncwarp();
  }

  const int64_t chunks_per_row = (a.cols + a.chunk - 1) / a.chunk;
  const int64_t num_units = a.rows * chunks_per_row;
  const WarpUnits wu = warp_units(num_units, static_cast<int64_t>(gridDim.x) * warps,
                                  static_cast<int64_t>(blockIdx.x) * warps + warp, a.interleave);
  const int64_t n = wu.count;

  auto unit_of = [&](int64_t u, int64_t& row, int64_t& col, int& len) {
    row = u / chunks_per_row;
    col = (u - row * chunks_per_row) * a.chunk;
    len = static_cast<int>(min(a.chunk, a.cols - col));
  };

  auto issue = [&](int64_t j) {
    const int s = static_cast<int>(j % a.stages);
    uint8_t* st = ring + static_cast<size_t>(s) * a.stage_bytes;
    int64_t row, col;
    int len;
    unit_of(wu.at(j), row, col, len);
    const uint32_t bytes = static_cast<uint32_t>(len) * sizeof(S);
    mbar_arrive_expect_tx(&bars[s], 2 * bytes);
    bulk_load(st, static_cast<const S*>(a.gate) + row * a.gate_stride + col, bytes, &bars[s]);
    bulk_load(st + half_stage, static_cast<const S*>(a.up) + row * a.up_stride + col, bytes,
              &bars[s]);
  };

  if (lane == 0) {
    for (int64_t j = 0; j < min(static_cast<int64_t>(a.stages), n); ++j) issue(j);
  }

  int64_t j = 0;
  for (; j < n; ++j) {
    const int s = static_cast<int>(j % a.stages);
    const uint32_t parity = static_cast<uint32_t>((j / a.stages) & 1);
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bars[s], parity))) break;
    const uint8_t* st = ring + static_cast<size_t>(s) * a.stage_bytes;
    int64_t row, col;
    int len;
    unit_of(wu.at(j), row, col, len);
    S* out = static_cast<S*>(a.out) + row * a.out_stride + col;
    const int nv = len / kVec;
#pragma unroll 2
    for (int v = lane; v < nv; v += kWarpSize) {
      const uint4 g = ld_shared_v4(st + v * 16);
      const uint4 u = ld_shared_v4(st + half_stage + v * 16);
      if (kTable && use_table) {
        st_global_v4(out + v * kVec, silu_mul_vec_table(g, u, table));
      } else {
        st_global_v4(out + v * kVec, silu_mul_vec<E>(g, u));
      }
    }
    __syncwarp();
    if (lane == 0 && j + a.stages < n) {
      fence_proxy_async_smem();
      issue(j + a.stages);
    }
  }

  if (j < n) {
    if (lane == 0) {
      raise_error(a.err, kErrWaitTimeout);
      for (int64_t m = j; m < min(j + a.stages, n); ++m) {
        mbar_wait_bounded(&bars[m % a.stages], static_cast<uint32_t>((m / a.stages) & 1));
      }
    }
    __syncwarp();
  }
  if constexpr (kTable) {
    if (threadIdx.x == 0 && table_copy_pending) mbar_wait_bounded(&table_bar, 0);
  }
}

template <class E>
__global__ void __launch_bounds__(256) silu_plain_kernel(const SiluArgs a) {
  grid_dependency_sync();
  using S = typename E::Storage;
  const int64_t total = a.rows * a.cols;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += step) {
    const int64_t row = i / a.cols;
    const int64_t col = i - row * a.cols;
    const float g = E::to_float(static_cast<const S*>(a.gate)[row * a.gate_stride + col]);
    const float u = E::to_float(static_cast<const S*>(a.up)[row * a.up_stride + col]);
    static_cast<S*>(a.out)[row * a.out_stride + col] =
        E::from_float(__fmul_rn(E::round(silu(g)), u));
  }
}

template <class E>
int launch_silu(void* out, const void* gate, const void* up, int64_t num_rows, int64_t inter,
                int64_t out_stride, int64_t gate_stride, int64_t up_stride, cudaStream_t stream) {
  using S = typename E::Storage;
  constexpr int kVec = E::kPerVec;
  if (num_rows < 0 || inter <= 0 || out_stride < inter || gate_stride < inter ||
      up_stride < inter) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  if (num_rows == 0) return SVLLM_OK;
  if (out == nullptr || gate == nullptr || up == nullptr) return SVLLM_ERR_INVALID_ARGUMENT;

  int device;
  if (current_device(&device) != SVLLM_OK) return SVLLM_ERR_CUDA;
  int* err = library_error_word(device);
  if (err == nullptr) return SVLLM_ERR_CUDA;

  SiluArgs a{};
  a.out = out;
  a.gate = gate;
  a.up = up;
  a.err = err;
  a.interleave = 1;  // measured faster than contiguous shares on B200
  const bool flat = out_stride == inter && gate_stride == inter && up_stride == inter;
  a.rows = flat ? 1 : num_rows;
  a.cols = flat ? num_rows * inter : inter;
  a.out_stride = flat ? 0 : out_stride;
  a.gate_stride = flat ? 0 : gate_stride;
  a.up_stride = flat ? 0 : up_stride;

  const bool bulk_ok = aligned16(out) && aligned16(gate) && aligned16(up) && inter % kVec == 0 &&
                       out_stride % kVec == 0 && gate_stride % kVec == 0 && up_stride % kVec == 0;
  if (bulk_ok) {
    const PipelineShape shape = pipeline_shape(OpId::kSiluAndMul);
    constexpr int64_t kGranule = static_cast<int64_t>(kVec) * kWarpSize;  // one vector per lane
    int64_t chunk = shape.unit_bytes / (2 * static_cast<int64_t>(sizeof(S)));
    // Small batches (decode): shrink the chunk until every SM has its tuned warp count of
    // chunks, so that the SiLU arithmetic of a few thousand elements is spread over many warps
    // instead of serialised in a few.
    const int64_t want_units = static_cast<int64_t>(sm_count(device)) * shape.warps;
    chunk = std::min<int64_t>(chunk, (a.rows * a.cols + want_units - 1) / want_units);
    chunk = std::max<int64_t>(kGranule, chunk / kGranule * kGranule);
    chunk = std::min<int64_t>(chunk, round_up(a.cols, kVec));
    a.chunk = chunk;
    a.stage_bytes = static_cast<int>(round_up(2 * chunk * static_cast<int64_t>(sizeof(S)), 128));
    const bool table = sizeof(S) == 2 &&
                       a.rows * a.cols >= static_cast<int64_t>(sm_count(device)) *
                                              kTableMinElementsPerSm;
    if (table && !g_silu_table_launched[device].exchange(true)) {
      // once per device, on the caller's stream: calls after it on this stream find the table
      // published; calls racing it on other streams compute directly until it is
      if (launch(silu_table_build_kernel, dim3(1), dim3(1024), 0, stream, 1) != SVLLM_OK) {
        g_silu_table_launched[device].store(false);
        return SVLLM_ERR_LAUNCH;
      }
    }
    const int64_t table_bytes = table ? kTableBytes : 0;
    int warps = warps_for(a.rows * ((a.cols + chunk - 1) / chunk), shape.warps, device);
    int stages = shape.stages;
    auto smem_for = [&](int w, int s) {
      return round_up(static_cast<int64_t>(w) * s * 8, 128) + table_bytes +
             static_cast<int64_t>(w) * s * a.stage_bytes;
    };
    while (smem_for(warps, stages) > static_cast<int64_t>(kMaxSmemPerCta) && stages > 2) --stages;
    while (smem_for(warps, stages) > static_cast<int64_t>(kMaxSmemPerCta) && warps > 1) --warps;
    if (smem_for(warps, stages) <= static_cast<int64_t>(kMaxSmemPerCta)) {
      a.stages = stages;
      a.table_offset = static_cast<int>(round_up(static_cast<int64_t>(warps) * stages * 8, 128));
      a.ring_offset = a.table_offset + static_cast<int>(table_bytes);
      const size_t smem = static_cast<size_t>(smem_for(warps, stages));
      const int threads = warps * kWarpSize;
      const auto kernel = table ? silu_bulk_kernel<E, sizeof(S) == 2> : silu_bulk_kernel<E, false>;
      const int per_sm = blocks_per_sm(reinterpret_cast<const void*>(kernel), threads, smem, device);
      if (per_sm > 0) {
        const int64_t units = a.rows * ((a.cols + chunk - 1) / chunk);
        const int64_t grid = persistent_grid((units + warps - 1) / warps, device, per_sm);
        a.early_dependents = early_dependents(a.rows * a.cols * static_cast<int64_t>(sizeof(S)) * 3);
        return launch(kernel, dim3(static_cast<unsigned>(grid)), dim3(threads), smem, stream, 1, a);
      }
    }
  }

  const int64_t grid = persistent_grid((a.rows * a.cols + 255) / 256, device, 8);
  return launch(silu_plain_kernel<E>, dim3(static_cast<unsigned>(grid)), dim3(256), 0, stream, 1,
                a);
}

}  // namespace
}  // namespace svllm::k

using svllm::k::Bf16;
using svllm::k::F32;
using svllm::k::launch_silu;

extern "C" {

int svllm_silu_and_mul_bf16(void* out, const void* gate, const void* up, int64_t num_rows,
                            int64_t inter, int64_t out_row_stride, int64_t gate_row_stride,
                            int64_t up_row_stride, svllm_stream stream) {
  return launch_silu<Bf16>(out, gate, up, num_rows, inter, out_row_stride, gate_row_stride,
                           up_row_stride, reinterpret_cast<cudaStream_t>(stream));
}

int svllm_silu_and_mul_f32(float* out, const float* gate, const float* up, int64_t num_rows,
                           int64_t inter, int64_t out_row_stride, int64_t gate_row_stride,
                           int64_t up_row_stride, svllm_stream stream) {
  return launch_silu<F32>(out, gate, up, num_rows, inter, out_row_stride, gate_row_stride,
                          up_row_stride, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

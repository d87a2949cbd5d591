// RMSNorm and RMSNorm with the fused residual add, for bf16 and fp32 rows.
//
// Reference: small-vLLM src/ops/cuda/rms_norm.cu:62-131 (one CTA per row, two global passes
// over x, block-wide reduction) and src/ops/cpu/rms_norm.cpp:13-44 (the formula, with the
// normalised value rounded to the storage type before the weight multiply). Here each row is
// read from HBM once:
//
//   * Bulk-copy path. Every warp owns a private ring of `stages` shared-memory stages and a
//     contiguous range of row units (a unit is R consecutive rows). Lane 0 keeps `stages`
//     cp.async.bulk loads in flight, each completing on the stage's mbarrier; the warp
//     normalises a landed unit from shared memory into registers and stores 16-byte vectors
//     straight to global memory, then lane 0 refills the stage. A row belongs to G lanes
//     (G = 4..32, a power of two) that hold V 16-byte vectors each, so the sum of squares needs
//     only log2(G) xor shuffles and no block barrier. The weight vector sits in shared memory.
//   * Row-block path, for rows that are not 16-byte aligned, not a multiple of 16 bytes, or
//     longer than the bulk path holds in registers: one CTA per row, two passes over the row
//     (the second hits L1/L2). Still on the GPU.
//
// Summation order. For bf16 the sum of squares is accumulated in exactly the order of the
// reference's CUDA kernel (rms_norm.cu:74-81 with block_sum, :31-56): thread t of a CTA of
// B = min(1024, round_up(units, 32)) threads sums its 8-element vectors (or elements, when the
// rows are not vectorisable) t, t + B, ... in order with fused multiply-adds; each warp reduces
// by xor shuffles with offsets 16..1; the warp sums are then combined by one more 32-lane xor
// tree in which the slots past the last warp hold zero; and the inverse RMS is
// rsqrtf(sum / hidden + eps). The bulk path maps warp w, lane l of that CTA onto vector v = w of
// lane l, keeps one partial per v, and replays the same tree, so the output is bit-identical to
// the reference kernel's, not merely within a rounding step of it.
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>
#include <cstdint>

#include "common.cuh"
#include "host_common.h"

namespace svllm::k {
namespace {

// Rows per SM up to which the row-block kernel runs instead of the bulk-copy pipeline.
constexpr int64_t kRowBlockMaxRowsPerSm = 64;

struct NormArgs {
  void* out;             // rms_norm: output rows; add_rms_norm: x, overwritten in place
  const void* x;         // input rows
  void* residual;        // add_rms_norm only: read, then overwritten with x + residual
  const void* weight;    // [hidden]
  int64_t num_rows;
  int64_t out_stride;    // elements
  int64_t x_stride;
  int64_t res_stride;
  int hidden;
  float eps;
  int* err;
  // bulk-copy path
  int early_dependents;  // let the next kernel be scheduled at this one's start
  int rows_per_unit;     // R
  int interleave;        // unit order (WarpUnits)
  float inv_hidden;      // 1 / hidden when hidden is a power of two, else 0
  int stages;
  int stage_bytes;       // bytes of one stage (x rows, then residual rows)
  int weight_offset;     // byte offsets into dynamic shared memory
  int ring_offset;
};

// Loads `rows` rows starting at row r0 into dst, as one copy when the rows are contiguous.
__device__ __forceinline__ void load_rows(uint8_t* dst, const void* base, int64_t stride_bytes,
                                          int64_t r0, int rows, uint32_t row_bytes,
                                          uint64_t* bar) {
  const uint8_t* src = static_cast<const uint8_t*>(base) + r0 * stride_bytes;
  if (stride_bytes == row_bytes) {
    bulk_load(dst, src, rows * row_bytes, bar);
  } else {
    for (int r = 0; r < rows; ++r) {
      bulk_load(dst + r * row_bytes, src + r * stride_bytes, row_bytes, bar);
    }
  }
}

template <class E, int G, int V, bool kAdd>
__global__ void __launch_bounds__(512) norm_bulk_kernel(const NormArgs a) {
  grid_dependency_wait();
  if (a.early_dependents) allow_dependents();
  using S = typename E::Storage;
  constexpr int kVec = E::kPerVec;
  constexpr int kRowsPerPass = kWarpSize / G;
  // Sums of squares and the scaling by 1/RMS in packed fp32 pairs (bit-identical). Measured on a
  // B200 for plain bf16 rms_norm with an even number of vectors per lane: 1M x 1024 6220 -> 6560
  // GB/s, 16384 x 2048 5890 -> 6300. With the residual add (1M x 1024: 6480 -> 5770) and for one
  // vector per lane (16M x 128: 6410 -> 6040, the scaling alone packed) it was slower; those keep
  // scalar fp32.
  constexpr bool kPacked = std::is_same_v<E, Bf16> && V % 2 == 0 && !kAdd;
  extern __shared__ __align__(128) uint8_t smem[];

  const int warps = blockDim.x / kWarpSize;
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x % kWarpSize;
  const int hidden = a.hidden;
  const int nvec = hidden / kVec;
  const uint32_t row_bytes = static_cast<uint32_t>(hidden) * sizeof(S);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * a.stages;
  uint8_t* wsm = smem + a.weight_offset;
  uint8_t* ring = smem + a.ring_offset + static_cast<size_t>(warp) * a.stages * a.stage_bytes;

  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    *reinterpret_cast<uint4*>(wsm + i * 16) =
        ld_global_nc_v4(static_cast<const uint8_t*>(a.weight) + i * 16);
  }
  if (lane == 0) {
    for (int s = 0; s < a.stages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  const int64_t num_units = (a.num_rows + a.rows_per_unit - 1) / a.rows_per_unit;
  const WarpUnits wu = warp_units(num_units, static_cast<int64_t>(gridDim.x) * warps,
                                  static_cast<int64_t>(blockIdx.x) * warps + warp, a.interleave);
  const int64_t n = wu.count;
  const int64_t x_stride_b = a.x_stride * static_cast<int64_t>(sizeof(S));
  const int64_t r_stride_b = a.res_stride * static_cast<int64_t>(sizeof(S));

  auto issue = [&](int64_t j) {
    const int s = static_cast<int>(j % a.stages);
    uint8_t* st = ring + static_cast<size_t>(s) * a.stage_bytes;
    const int64_t r0 = wu.at(j) * a.rows_per_unit;
    const int rows = static_cast<int>(min(static_cast<int64_t>(a.rows_per_unit), a.num_rows - r0));
    const uint32_t bytes = rows * row_bytes;
    mbar_arrive_expect_tx(&bars[s], kAdd ? 2 * bytes : bytes);
    load_rows(st, a.x, x_stride_b, r0, rows, row_bytes, &bars[s]);
    if constexpr (kAdd) {
      load_rows(st + a.rows_per_unit * row_bytes, a.residual, r_stride_b, r0, rows, row_bytes,
                &bars[s]);
    }
  };

  if (lane == 0) {
    for (int64_t j = 0; j < min(static_cast<int64_t>(a.stages), n); ++j) issue(j);
  }

  const float hidden_f = static_cast<float>(hidden);
  int64_t j = 0;
  for (; j < n; ++j) {
    const int s = static_cast<int>(j % a.stages);
    const uint32_t parity = static_cast<uint32_t>((j / a.stages) & 1);
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bars[s], parity))) break;

    const uint8_t* st = ring + static_cast<size_t>(s) * a.stage_bytes;
    const int64_t r0 = wu.at(j) * a.rows_per_unit;
    const int rows = static_cast<int>(min(static_cast<int64_t>(a.rows_per_unit), a.num_rows - r0));
    const int sub = lane % G;

    for (int pass = 0; pass < a.rows_per_unit / kRowsPerPass; ++pass) {
      const int rl = pass * kRowsPerPass + lane / G;  // row within the unit
      const uint8_t* xs = st + rl * row_bytes;
      uint4 hv[V];
      float part[V];
      if constexpr (kPacked) {
        // vectors v and v + 1 summed side by side in packed fp32 pairs: each running sum keeps
        // its own order and roundings (a vector past the row is zero and leaves its sum +0)
#pragma unroll
        for (int v = 0; v < V; ++v) {
          const int c = sub + G * v;
          hv[v] = make_uint4(0, 0, 0, 0);
          if (c < nvec) {
            uint4 raw = ld_shared_v4(xs + c * 16);
            if constexpr (kAdd) {
              raw = add_vec<E>(raw, ld_shared_v4(xs + a.rows_per_unit * row_bytes + c * 16));
            }
            hv[v] = raw;
          }
        }
#pragma unroll
        for (int v = 0; v < V; v += 2) {
          float f0[kVec], f1[kVec];
          unpack<E>(hv[v], f0);
          unpack<E>(hv[v + 1], f1);
          uint64_t acc = f32x2(0.0f, 0.0f);
#pragma unroll
          for (int e = 0; e < kVec; ++e) {
            const uint64_t p = f32x2(f0[e], f1[e]);
            acc = f32x2_fma(p, p, acc);
          }
          f32x2_split(acc, part[v], part[v + 1]);
        }
      } else {
#pragma unroll
        for (int v = 0; v < V; ++v) {
          const int c = sub + G * v;
          part[v] = 0.0f;
          if (c < nvec) {
            uint4 raw = ld_shared_v4(xs + c * 16);
            if constexpr (kAdd) {
              raw = add_vec<E>(raw, ld_shared_v4(xs + a.rows_per_unit * row_bytes + c * 16));
            }
            hv[v] = raw;
            float f[kVec];
            unpack<E>(raw, f);
#pragma unroll
            for (int e = 0; e < kVec; ++e) part[v] = __fmaf_rn(f[e], f[e], part[v]);
          } else {
            hv[v] = make_uint4(0, 0, 0, 0);
          }
        }
      }
      float total;
      if constexpr (V == 1) {
        total = group_sum<G>(part[0]);
      } else {
        // vector v of every lane is warp v of the reference's CTA: reduce each, then combine
        // the warp sums with the reference's final xor tree (slots past V hold zero)
#pragma unroll
        for (int v = 0; v < V; ++v) part[v] = group_sum<kWarpSize>(part[v]);
#pragma unroll
        for (int off = V / 2; off >= 1; off /= 2) {
#pragma unroll
          for (int i = 0; i < off; ++i) part[i] = __fadd_rn(part[i], part[i + off]);
        }
        total = part[0];
      }
      // sum / hidden; a power-of-two hidden divides exactly as a multiply by its reciprocal
      const float mean = a.inv_hidden != 0.0f ? __fmul_rn(total, a.inv_hidden)
                                              : __fdiv_rn(total, hidden_f);
      const float inv_rms = rsqrtf(__fadd_rn(mean, a.eps));

      if (rl < rows) {
        const int64_t row = r0 + rl;
        S* out_row = static_cast<S*>(a.out) + row * a.out_stride;
        S* res_row = kAdd ? static_cast<S*>(a.residual) + row * a.res_stride : nullptr;
#pragma unroll
        for (int v = 0; v < V; ++v) {
          const int c = sub + G * v;
          if (c < nvec) {
            if constexpr (kAdd) st_global_v4(res_row + c * kVec, hv[v]);
            const uint4 wv = ld_shared_v4(wsm + c * 16);
            if constexpr (kPacked) {
              st_global_v4(out_row + c * kVec, normalize_vec_packed(hv[v], inv_rms, wv));
            } else {
              st_global_v4(out_row + c * kVec, normalize_vec<E>(hv[v], inv_rms, wv));
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0 && j + a.stages < n) {
      fence_proxy_async_smem();
      issue(j + a.stages);
    }
  }

  if (j < n) {
    // A copy did not land in time: report it and give the copies still in flight a bounded
    // chance to finish before the CTA's shared memory goes away.
    if (lane == 0) {
      raise_error(a.err, kErrWaitTimeout);
      for (int64_t k = j; k < min(j + a.stages, n); ++k) {
        mbar_wait_bounded(&bars[k % a.stages], static_cast<uint32_t>((k / a.stages) & 1));
      }
    }
    __syncwarp();
  }
}

// Row-block path: one CTA per row (grid-stride over rows), N elements per load (N = 8 for
// 16-byte bf16 vectors, 4 for fp32, 1 when the rows are not vectorisable), the reference's
// thread-to-element mapping and reduction tree.
template <class E, int N, bool kAdd>
__global__ void __launch_bounds__(1024) norm_rowblock_kernel(const NormArgs a) {
  grid_dependency_sync();
  using S = typename E::Storage;
  struct alignas(sizeof(S) * N) Pack {
    S v[N];
  };
  __shared__ float warp_sums[kWarpSize];
  __shared__ float row_total;
  const int units = a.hidden / N;
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x % kWarpSize;
  const int num_warps = blockDim.x / kWarpSize;
  const Pack* w = static_cast<const Pack*>(a.weight);
  const float hidden_f = static_cast<float>(a.hidden);

  for (int64_t row = blockIdx.x; row < a.num_rows; row += gridDim.x) {
    const Pack* x = reinterpret_cast<const Pack*>(static_cast<const S*>(a.x) + row * a.x_stride);
    Pack* res = kAdd ? reinterpret_cast<Pack*>(static_cast<S*>(a.residual) + row * a.res_stride)
                     : nullptr;
    Pack* out = reinterpret_cast<Pack*>(static_cast<S*>(a.out) + row * a.out_stride);

    float part = 0.0f;
    for (int u = threadIdx.x; u < units; u += blockDim.x) {
      Pack p = x[u];
      if constexpr (kAdd) {
        const Pack r = res[u];
#pragma unroll
        for (int j = 0; j < N; ++j) {
          p.v[j] = E::from_float(__fadd_rn(E::to_float(p.v[j]), E::to_float(r.v[j])));
        }
        res[u] = p;
      }
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const float f = E::to_float(p.v[j]);
        part = __fmaf_rn(f, f, part);
      }
    }
    part = group_sum<kWarpSize>(part);
    if (lane == 0) warp_sums[warp] = part;
    __syncthreads();
    if (warp == 0) {
      float v = lane < num_warps ? warp_sums[lane] : 0.0f;
      v = group_sum<kWarpSize>(v);
      if (lane == 0) row_total = v;
    }
    __syncthreads();
    const float mean = a.inv_hidden != 0.0f ? __fmul_rn(row_total, a.inv_hidden)
                                            : __fdiv_rn(row_total, hidden_f);
    const float inv_rms = rsqrtf(__fadd_rn(mean, a.eps));

    // Each thread re-reads only the units it read (and, for add, wrote) in the first pass.
    for (int u = threadIdx.x; u < units; u += blockDim.x) {
      const Pack p = kAdd ? res[u] : x[u];
      const Pack wv = w[u];
      Pack o;
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const float n = E::round(__fmul_rn(E::to_float(p.v[j]), inv_rms));
        o.v[j] = E::from_float(__fmul_rn(n, E::to_float(wv.v[j])));
      }
      out[u] = o;
    }
    __syncthreads();  // warp_sums and row_total are reused by the next row
  }
}

template <class E, bool kAdd>
using NormKernel = void (*)(NormArgs);

// Picks lanes-per-row G and vectors-per-lane V for a row of nvec 16-byte vectors.
template <class E, bool kAdd>
NormKernel<E, kAdd> pick_bulk_kernel(int nvec, int* lanes_per_row) {
  if (nvec <= 4) { *lanes_per_row = 4; return norm_bulk_kernel<E, 4, 1, kAdd>; }
  if (nvec <= 8) { *lanes_per_row = 8; return norm_bulk_kernel<E, 8, 1, kAdd>; }
  if (nvec <= 16) { *lanes_per_row = 16; return norm_bulk_kernel<E, 16, 1, kAdd>; }
  *lanes_per_row = 32;
  if (nvec <= 32) return norm_bulk_kernel<E, 32, 1, kAdd>;
  if (nvec <= 64) return norm_bulk_kernel<E, 32, 2, kAdd>;
  if (nvec <= 128) return norm_bulk_kernel<E, 32, 4, kAdd>;
  if (nvec <= 256) return norm_bulk_kernel<E, 32, 8, kAdd>;
  if (nvec <= 512) return norm_bulk_kernel<E, 32, 16, kAdd>;
  return nullptr;
}

template <class E, bool kAdd>
int launch_norm(void* out, const void* x, void* residual, const void* weight, int64_t num_rows,
                int64_t hidden, int64_t out_stride, int64_t x_stride, int64_t res_stride,
                float eps, cudaStream_t stream) {
  using S = typename E::Storage;
  if (num_rows < 0 || hidden <= 0 || out_stride < hidden || x_stride < hidden ||
      (kAdd && res_stride < hidden)) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  if (num_rows == 0) return SVLLM_OK;
  if (out == nullptr || x == nullptr || weight == nullptr || (kAdd && residual == nullptr)) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  if (hidden > (1 << 24)) return SVLLM_ERR_TOO_LARGE;

  int device;
  if (current_device(&device) != SVLLM_OK) return SVLLM_ERR_CUDA;
  int* err = library_error_word(device);
  if (err == nullptr) return SVLLM_ERR_CUDA;

  NormArgs a{};
  a.out = out;
  a.x = x;
  a.residual = residual;
  a.weight = weight;
  a.num_rows = num_rows;
  a.out_stride = out_stride;
  a.x_stride = x_stride;
  a.res_stride = kAdd ? res_stride : x_stride;
  a.hidden = static_cast<int>(hidden);
  a.eps = eps;
  a.err = err;
  a.interleave = 1;  // measured faster than contiguous shares on B200
  a.inv_hidden = (hidden & (hidden - 1)) == 0 ? 1.0f / static_cast<float>(hidden) : 0.0f;

  const int64_t row_bytes = hidden * static_cast<int64_t>(sizeof(S));
  const bool bulk_ok = aligned16(out) && aligned16(x) && aligned16(weight) &&
                       (!kAdd || aligned16(residual)) && row_bytes % 16 == 0 &&
                       (out_stride * sizeof(S)) % 16 == 0 && (x_stride * sizeof(S)) % 16 == 0 &&
                       (!kAdd || (res_stride * sizeof(S)) % 16 == 0);
  // Up to ~10k rows (decode and short prefill batches) the row-block kernel's direct loads
  // finish sooner than a bulk-copy pipeline can start: measured on a B200 at 1 to 262144 rows of
  // 1024 bf16 (add_rms_norm: 2.0 vs 3.0 us at one row, 11.4 vs 12.3 us at 8192 rows; from
  // 65536 rows on the pipeline wins, 87 vs 104 us).
  const bool small = num_rows <= kRowBlockMaxRowsPerSm * static_cast<int64_t>(sm_count(device));
  if (bulk_ok && !small) {
    int lanes_per_row = 0;
    const NormKernel<E, kAdd> kernel =
        pick_bulk_kernel<E, kAdd>(static_cast<int>(row_bytes / 16), &lanes_per_row);
    if (kernel != nullptr) {
      const PipelineShape shape = pipeline_shape(kAdd ? OpId::kAddRmsNorm : OpId::kRmsNorm);
      const int rows_per_pass = kWarpSize / lanes_per_row;
      const int64_t unit_row_bytes = row_bytes * (kAdd ? 2 : 1);
      // Short rows (at most 256 bf16) spend more instructions per byte on their reductions and
      // take half again as many warps (rms_norm at 16M rows of 128 on a B200: 5088 -> 6551
      // GB/s with 12 warps instead of 8).
      const int tuned_warps =
          std::min(kMaxBulkWarps, !kAdd && row_bytes <= 512 ? shape.warps * 3 / 2 : shape.warps);
      int64_t rows = std::max<int64_t>(1, shape.unit_bytes / unit_row_bytes);
      rows = std::max<int64_t>(rows_per_pass, rows / rows_per_pass * rows_per_pass);
      rows = std::min<int64_t>(rows, round_up(num_rows, rows_per_pass));
      // Units shrink (down to one pass of rows) until every warp of one CTA per SM has at
      // least 16 of them, so that mid-sized batches keep their pipelines full (rms_norm at
      // 16384 rows of 2048: 4258 -> 5635 GB/s with one-row units instead of two-row ones).
      const int64_t target_units = 16ll * sm_count(device) * tuned_warps;
      rows = std::min<int64_t>(
          rows, std::max<int64_t>(rows_per_pass, num_rows / target_units / rows_per_pass *
                                                     rows_per_pass));
      a.rows_per_unit = static_cast<int>(rows);
      a.stage_bytes = static_cast<int>(round_up(rows * unit_row_bytes, 128));
      int warps = warps_for((num_rows + rows - 1) / rows, tuned_warps, device);
      int stages = shape.stages;
      auto smem_for = [&](int w, int s) {
        return round_up(static_cast<int64_t>(w) * s * 8, 128) + round_up(row_bytes, 128) +
               static_cast<int64_t>(w) * s * a.stage_bytes;
      };
      while (smem_for(warps, stages) > static_cast<int64_t>(kMaxSmemPerCta) && stages > 2) --stages;
      while (smem_for(warps, stages) > static_cast<int64_t>(kMaxSmemPerCta) && warps > 1) --warps;
      if (smem_for(warps, stages) <= static_cast<int64_t>(kMaxSmemPerCta)) {
        a.stages = stages;
        a.weight_offset = static_cast<int>(round_up(static_cast<int64_t>(warps) * stages * 8, 128));
        a.ring_offset = a.weight_offset + static_cast<int>(round_up(row_bytes, 128));
        const size_t smem = static_cast<size_t>(smem_for(warps, stages));
        const int threads = warps * kWarpSize;
        const int per_sm = blocks_per_sm(reinterpret_cast<const void*>(kernel), threads, smem, device);
        if (per_sm > 0) {
          const int64_t num_units = (num_rows + rows - 1) / rows;
          const int64_t grid = persistent_grid((num_units + warps - 1) / warps, device, per_sm);
          a.early_dependents = early_dependents(num_rows * row_bytes * (kAdd ? 4 : 2));
          return launch(kernel, dim3(static_cast<unsigned>(grid)), dim3(threads), smem, stream, 1,
                        a);
        }
      }
    }
  }

  // Row-block path, vectorised exactly when the reference's kernel is (rms_norm.cu:122-127):
  // a row length that is a multiple of the vector and 16-byte aligned base pointers.
  constexpr int kVec = E::kPerVec;
  const bool vec = hidden % kVec == 0 && aligned16(out) && aligned16(x) && aligned16(weight) &&
                   (!kAdd || aligned16(residual)) && out_stride % kVec == 0 &&
                   x_stride % kVec == 0 && (!kAdd || res_stride % kVec == 0);
  const int64_t units = vec ? hidden / kVec : hidden;
  const int threads = static_cast<int>(std::min<int64_t>(1024, round_up(units, kWarpSize)));
  const auto kernel = vec ? norm_rowblock_kernel<E, kVec, kAdd> : norm_rowblock_kernel<E, 1, kAdd>;
  const int per_sm = blocks_per_sm(reinterpret_cast<const void*>(kernel), threads, 0, device);
  const int64_t grid = persistent_grid(num_rows, device, per_sm > 0 ? per_sm : 1);
  return launch(kernel, dim3(static_cast<unsigned>(grid)), dim3(threads), 0, stream, 1, a);
}

}  // namespace
}  // namespace svllm::k

using svllm::k::Bf16;
using svllm::k::F32;
using svllm::k::launch_norm;

extern "C" {

int svllm_rms_norm_bf16(void* out, const void* x, const void* weight, int64_t num_rows,
                        int64_t hidden, int64_t out_row_stride, int64_t x_row_stride, float eps,
                        svllm_stream stream) {
  return launch_norm<Bf16, false>(out, x, nullptr, weight, num_rows, hidden, out_row_stride,
                                  x_row_stride, 0, eps, reinterpret_cast<cudaStream_t>(stream));
}

int svllm_rms_norm_f32(float* out, const float* x, const float* weight, int64_t num_rows,
                       int64_t hidden, int64_t out_row_stride, int64_t x_row_stride, float eps,
                       svllm_stream stream) {
  return launch_norm<F32, false>(out, x, nullptr, weight, num_rows, hidden, out_row_stride,
                                 x_row_stride, 0, eps, reinterpret_cast<cudaStream_t>(stream));
}

int svllm_add_rms_norm_bf16(void* x, void* residual, const void* weight, int64_t num_rows,
                            int64_t hidden, int64_t x_row_stride, int64_t residual_row_stride,
                            float eps, svllm_stream stream) {
  return launch_norm<Bf16, true>(x, x, residual, weight, num_rows, hidden, x_row_stride,
                                 x_row_stride, residual_row_stride, eps,
                                 reinterpret_cast<cudaStream_t>(stream));
}

int svllm_add_rms_norm_f32(float* x, float* residual, const float* weight, int64_t num_rows,
                           int64_t hidden, int64_t x_row_stride, int64_t residual_row_stride,
                           float eps, svllm_stream stream) {
  return launch_norm<F32, true>(x, x, residual, weight, num_rows, hidden, x_row_stride,
                                x_row_stride, residual_row_stride, eps,
                                reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

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
//   * Plain path, for rows that are not 16-byte aligned or not a multiple of 16 bytes: one
//     warp per row, element loads, two passes (the second hits L1/L2). Still on the GPU.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "host_common.h"

namespace svllm::k {
namespace {

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
  int rows_per_unit;     // R
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
__global__ void __launch_bounds__(256) norm_bulk_kernel(const NormArgs a) {
  using S = typename E::Storage;
  constexpr int kVec = E::kPerVec;
  constexpr int kRowsPerPass = kWarpSize / G;
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
  int64_t u0, u1;
  partition(num_units, static_cast<int64_t>(gridDim.x) * warps,
            static_cast<int64_t>(blockIdx.x) * warps + warp, u0, u1);
  const int64_t n = u1 - u0;
  const int64_t x_stride_b = a.x_stride * static_cast<int64_t>(sizeof(S));
  const int64_t r_stride_b = a.res_stride * static_cast<int64_t>(sizeof(S));

  auto issue = [&](int64_t j) {
    const int s = static_cast<int>(j % a.stages);
    uint8_t* st = ring + static_cast<size_t>(s) * a.stage_bytes;
    const int64_t r0 = (u0 + j) * a.rows_per_unit;
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

  const float inv_hidden_div = static_cast<float>(hidden);
  int64_t j = 0;
  for (; j < n; ++j) {
    const int s = static_cast<int>(j % a.stages);
    const uint32_t parity = static_cast<uint32_t>((j / a.stages) & 1);
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bars[s], parity))) break;

    const uint8_t* st = ring + static_cast<size_t>(s) * a.stage_bytes;
    const int64_t r0 = (u0 + j) * a.rows_per_unit;
    const int rows = static_cast<int>(min(static_cast<int64_t>(a.rows_per_unit), a.num_rows - r0));
    const int sub = lane % G;

    for (int pass = 0; pass < a.rows_per_unit / kRowsPerPass; ++pass) {
      const int rl = pass * kRowsPerPass + lane / G;  // row within the unit
      const uint8_t* xs = st + rl * row_bytes;
      uint4 hv[V];
      float ss = 0.0f;
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const int c = sub + G * v;
        if (c < nvec) {
          uint4 raw = ld_shared_v4(xs + c * 16);
          if constexpr (kAdd) {
            const uint4 rr = ld_shared_v4(xs + a.rows_per_unit * row_bytes + c * 16);
            float xf[kVec], rf[kVec];
            unpack<E>(raw, xf);
            unpack<E>(rr, rf);
#pragma unroll
            for (int e = 0; e < kVec; ++e) xf[e] = __fadd_rn(xf[e], rf[e]);
            raw = pack<E>(xf);  // residual + x, rounded to the storage type
          }
          hv[v] = raw;
          float f[kVec];
          unpack<E>(raw, f);
#pragma unroll
          for (int e = 0; e < kVec; ++e) ss = __fmaf_rn(f[e], f[e], ss);
        } else {
          hv[v] = make_uint4(0, 0, 0, 0);
        }
      }
      ss = group_sum<G>(ss);
      const float inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, inv_hidden_div), a.eps)));

      if (rl < rows) {
        const int64_t row = r0 + rl;
        S* out_row = static_cast<S*>(a.out) + row * a.out_stride;
        S* res_row = kAdd ? static_cast<S*>(a.residual) + row * a.res_stride : nullptr;
#pragma unroll
        for (int v = 0; v < V; ++v) {
          const int c = sub + G * v;
          if (c < nvec) {
            if constexpr (kAdd) st_global_v4(res_row + c * kVec, hv[v]);
            float f[kVec], w[kVec];
            unpack<E>(hv[v], f);
            unpack<E>(ld_shared_v4(wsm + c * 16), w);
#pragma unroll
            for (int e = 0; e < kVec; ++e) f[e] = __fmul_rn(E::round(__fmul_rn(f[e], inv_rms)), w[e]);
            st_global_v4(out_row + c * kVec, pack<E>(f));
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

// Plain-load path: one warp per row, grid-stride over rows.
template <class E, bool kAdd>
__global__ void __launch_bounds__(256) norm_plain_kernel(const NormArgs a) {
  using S = typename E::Storage;
  const int lane = threadIdx.x % kWarpSize;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x / kWarpSize);
  const int hidden = a.hidden;
  const S* w = static_cast<const S*>(a.weight);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / kWarpSize) +
                     threadIdx.x / kWarpSize;
       row < a.num_rows; row += warps_total) {
    const S* x = static_cast<const S*>(a.x) + row * a.x_stride;
    S* out = static_cast<S*>(a.out) + row * a.out_stride;
    S* res = kAdd ? static_cast<S*>(a.residual) + row * a.res_stride : nullptr;
    float ss = 0.0f;
    for (int i = lane; i < hidden; i += kWarpSize) {
      float v = E::to_float(x[i]);
      if constexpr (kAdd) {
        v = E::round(__fadd_rn(v, E::to_float(res[i])));
        res[i] = E::from_float(v);
      }
      ss = __fmaf_rn(v, v, ss);
    }
    ss = group_sum<kWarpSize>(ss);
    const float inv_rms =
        __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(hidden)), a.eps)));
    for (int i = lane; i < hidden; i += kWarpSize) {
      // Each lane re-reads only elements it read (and, for add, wrote) itself above.
      const float v = kAdd ? E::to_float(res[i]) : E::to_float(x[i]);
      out[i] = E::from_float(__fmul_rn(E::round(__fmul_rn(v, inv_rms)), E::to_float(w[i])));
    }
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

  const int64_t row_bytes = hidden * static_cast<int64_t>(sizeof(S));
  const bool bulk_ok = aligned16(out) && aligned16(x) && aligned16(weight) &&
                       (!kAdd || aligned16(residual)) && row_bytes % 16 == 0 &&
                       (out_stride * sizeof(S)) % 16 == 0 && (x_stride * sizeof(S)) % 16 == 0 &&
                       (!kAdd || (res_stride * sizeof(S)) % 16 == 0);
  if (bulk_ok) {
    int lanes_per_row = 0;
    const NormKernel<E, kAdd> kernel =
        pick_bulk_kernel<E, kAdd>(static_cast<int>(row_bytes / 16), &lanes_per_row);
    if (kernel != nullptr) {
      const PipelineShape shape = pipeline_shape(kAdd ? OpId::kAddRmsNorm : OpId::kRmsNorm);
      const int rows_per_pass = kWarpSize / lanes_per_row;
      const int64_t unit_row_bytes = row_bytes * (kAdd ? 2 : 1);
      int64_t rows = std::max<int64_t>(1, shape.unit_bytes / unit_row_bytes);
      rows = std::max<int64_t>(rows_per_pass, rows / rows_per_pass * rows_per_pass);
      rows = std::min<int64_t>(rows, round_up(num_rows, rows_per_pass));
      a.rows_per_unit = static_cast<int>(rows);
      a.stage_bytes = static_cast<int>(round_up(rows * unit_row_bytes, 128));
      int warps = shape.warps;
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
          kernel<<<static_cast<unsigned>(grid), threads, smem, stream>>>(a);
          return launch_status();
        }
      }
    }
  }

  constexpr int kThreads = 256;
  const int64_t grid = persistent_grid((num_rows + 7) / 8, device, 8);
  norm_plain_kernel<E, kAdd><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(a);
  return launch_status();
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

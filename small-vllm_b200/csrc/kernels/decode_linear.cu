// A linear layer for decode-sized batches: out[m, n] = bf16(sum_k x[m, k] * W[n, k]) for up to
// 16 token rows, the weight [out_features, in_features] row-major as a checkpoint stores it (the
// projections of the model forward the reference plans in src/model, which calls them through
// at::linear; docs/ROADMAP.md:24-25). At a few tokens such a GEMM is a stream over the weight
// with almost no arithmetic, and what decides its time is how soon every byte of the weight is
// requested: a library GEMM tiled for large M leaves most SMs idle, and a TMA + TMEM pipeline
// (tried first, measured at 5-7 us for the Qwen3-0.6B projections) spends longer on its fixed
// chain (TMEM allocation, mbarriers, a cluster merge of K splits) than on the stream itself.
//
// So the weight goes straight from HBM into mma.sync registers. A CTA of W warps owns 16 weight
// rows (the M of m16n8k16) and splits K between its warps in chunks of 32; lane 4g + t loads 16
// bytes at k = 32c + 8t of rows g and g + 8, which are the A fragments of two k-steps once the
// same permutation of K is applied to the activations (the B fragments: token g, the same 16
// bytes). The first kBuf chunks of weight are loaded before griddepcontrol.wait: they do not
// depend on the kernel before this one, which may still be running (programmatic dependent
// launch), so the whole weight is usually in flight before the activations exist. Then the
// activations (from L2), the MMAs in fp32, and the warps' partial sums meet in shared memory.
// No scratch memory, no waits on other CTAs, one launch.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "host_common.h"

namespace svllm::k {
namespace {

constexpr int kMaxTokens = 16;  // two n-tiles of 8 tokens
constexpr int kChunkK = 32;     // K per lane chunk: 16 bytes each of two rows

struct StreamArgs {
  void* out;
  int64_t out_stride;
  const void* x;
  int64_t x_stride;
  const void* w;
  int64_t w_stride;
  int64_t m, n, k;
};

__device__ __forceinline__ uint4 ld_global_cg_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// NT n-tiles of 8 tokens; W warps per CTA.
template <int NT, int W>
__global__ void __launch_bounds__(W * kWarpSize) decode_linear_kernel(const StreamArgs a) {
  constexpr int kBuf = 8 / NT;  // weight chunks a warp holds in registers at once
  __shared__ float4 red[W][NT][kWarpSize];
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x % kWarpSize;
  const int g = lane >> 2, t = lane & 3;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * 16;
  const int chunks = static_cast<int>((a.k + kChunkK - 1) / kChunkK);
  const int per_warp = (chunks + W - 1) / W;
  const int c_begin = min(chunks, warp * per_warp);
  const int c_end = min(chunks, c_begin + per_warp);
  const bool ok0 = row0 + g < a.n, ok1 = row0 + g + 8 < a.n;
  const uint8_t* w0 = static_cast<const uint8_t*>(a.w) + ((row0 + g) * a.w_stride + 8 * t) * 2;
  const uint8_t* w1 = w0 + 8 * a.w_stride * 2;
  const uint4 zero = make_uint4(0, 0, 0, 0);

  uint4 wlo[kBuf], whi[kBuf];
#pragma unroll
  for (int i = 0; i < kBuf; ++i) {
    const int c = c_begin + i;
    const bool in = c < c_end && kChunkK * c + 8 * t < a.k;  // K % 8 == 0: whole pieces
    wlo[i] = in && ok0 ? ld_global_nc_v4(w0 + 2 * kChunkK * c) : zero;
    whi[i] = in && ok1 ? ld_global_nc_v4(w1 + 2 * kChunkK * c) : zero;
  }
  // the activations are the previous kernel's output, and the output buffer may be memory it
  // still reads: everything below waits for it
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.0f;
  }
  const uint8_t* xb = static_cast<const uint8_t*>(a.x);
  for (int base = c_begin; base < c_end; base += kBuf) {
    uint4 xf[kBuf][NT];  // all of this round's activation fragments in flight together
#pragma unroll
    for (int i = 0; i < kBuf; ++i) {
      const int k = kChunkK * (base + i) + 8 * t;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int64_t tok = 8 * nt + g;
        xf[i][nt] = base + i < c_end && k < a.k && tok < a.m
                        ? ld_global_cg_v4(xb + (tok * a.x_stride + k) * 2)
                        : zero;
      }
    }
#pragma unroll
    for (int i = 0; i < kBuf; ++i) {
      if (base + i < c_end) {  // warp-uniform
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma_16816(acc[nt], wlo[i].x, whi[i].x, wlo[i].y, whi[i].y, xf[i][nt].x, xf[i][nt].y);
          mma_16816(acc[nt], wlo[i].z, whi[i].z, wlo[i].w, whi[i].w, xf[i][nt].z, xf[i][nt].w);
        }
      }
    }
    if (base + kBuf < c_end) {  // the next round's weight
#pragma unroll
      for (int i = 0; i < kBuf; ++i) {
        const int c = base + kBuf + i;
        const bool in = c < c_end && kChunkK * c + 8 * t < a.k;
        wlo[i] = in && ok0 ? ld_global_nc_v4(w0 + 2 * kChunkK * c) : zero;
        whi[i] = in && ok1 ? ld_global_nc_v4(w1 + 2 * kChunkK * c) : zero;
      }
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    red[warp][nt][lane] = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
  }
  __syncthreads();
  if (warp < NT) {  // warp nt adds up n-tile nt: rows g, g + 8 x tokens 8nt + 2t, 8nt + 2t + 1
    float4 sum = red[0][warp][lane];
#pragma unroll
    for (int w = 1; w < W; ++w) {
      const float4 v = red[w][warp][lane];
      sum.x += v.x;
      sum.y += v.y;
      sum.z += v.z;
      sum.w += v.w;
    }
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
    const float vals[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int64_t tok = 8 * warp + 2 * t + (e & 1);
      const int64_t row = row0 + g + (e >> 1) * 8;
      if (tok < a.m && row < a.n) out[tok * a.out_stride + row] = __float2bfloat16_rn(vals[e]);
    }
  }
}

// Warps per CTA: enough that each holds its share of K in one register round where possible
// (all of the weight in flight at once), at most 16.
template <int NT>
int launch_linear(const StreamArgs& a, cudaStream_t stream) {
  const int64_t chunks = (a.k + kChunkK - 1) / kChunkK;
  const int64_t rounds = (chunks + 8 / NT - 1) / (8 / NT);
  const dim3 grid(static_cast<unsigned>((a.n + 15) / 16));
  const dim3 block4(4 * kWarpSize), block8(8 * kWarpSize), block16(16 * kWarpSize);
  if (rounds <= 4) return launch(decode_linear_kernel<NT, 4>, grid, block4, 0, stream, 1, a);
  if (rounds <= 8) return launch(decode_linear_kernel<NT, 8>, grid, block8, 0, stream, 1, a);
  return launch(decode_linear_kernel<NT, 16>, grid, block16, 0, stream, 1, a);
}

}  // namespace
}  // namespace svllm::k

extern "C" int svllm_decode_linear_bf16(void* out, int64_t out_stride, const void* x,
                                        int64_t num_rows, int64_t in_features, int64_t x_stride,
                                        const void* weight, int64_t out_features,
                                        int64_t weight_stride, svllm_stream stream) {
  using namespace svllm::k;
  if (num_rows < 0 || in_features <= 0 || out_features <= 0 || x_stride < in_features ||
      weight_stride < in_features || out_stride < out_features ||
      out_features >= (int64_t{1} << 35) || in_features >= (int64_t{1} << 31)) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  if (num_rows == 0) return SVLLM_OK;
  if (out == nullptr || x == nullptr || weight == nullptr) return SVLLM_ERR_INVALID_ARGUMENT;
  // more rows than a decode batch, or rows the 16-byte loads cannot read: the caller's GEMM
  if (num_rows > kMaxTokens || in_features % 8 != 0 || !aligned16(x) || !aligned16(weight) ||
      (x_stride * 2) % 16 != 0 || (weight_stride * 2) % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(out) & 1u) != 0) {
    return SVLLM_ERR_UNSUPPORTED;
  }
  const StreamArgs a{out, out_stride, x, x_stride, weight, weight_stride, num_rows,
                     out_features, in_features};
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return num_rows <= 8 ? launch_linear<1>(a, s) : launch_linear<2>(a, s);
}

// Qwen3 per-head q/k RMSNorm fused with neox-style rotary embedding, and rotary embedding alone
// (Llama), in place on q and k, for bf16 and fp32.
//
// The reference has no kernel for either: the flags come from small-vLLM src/model/config.h:27-30
// and config.cpp:34-52, and the formulas are Hugging Face's Qwen3RMSNorm followed by
// apply_rotary_pos_emb, with cos/sin rounded to the activation dtype as its rotary embedding
// returns them. One token is one unit: its q row and k row are read from HBM once, normalised
// per head (Qwen3), rotated, and written back.
//
//   * Bulk-copy path (head_dim a multiple of 16 bytes * 2, 16-byte aligned rows): each warp owns
//     a ring of stages and a contiguous range of tokens; lane 0 keeps cp.async.bulk loads of the
//     q and k rows of the next tokens in flight. A head belongs to G = head_dim / (2 * vec) lanes,
//     and lane j of a head holds elements [vec*j, vec*j + vec) and the matching second half, so
//     every rotation pair (i, i + head_dim/2) is in one lane and the head's sum of squares needs
//     log2(G) shuffles. The warp computes the token's head_dim/2 (cos, sin) pairs once (two per
//     lane at head_dim 128), shares them through shared memory, and reuses them for all heads.
//     inv_freq travels in the kernel parameters (constant bank) and is staged in shared memory.
//     The angle is one fp32 multiply fp32(pos) * inv_freq[i], as Hugging Face's fp32 outer
//     product forms it, and cos/sin are the CUDA math library's accurate cosf/sinf (no fast
//     approximations: their error would grow with the angle), the same functions torch's cos and
//     sin kernels call, so on one GPU the result equals the torch composite bit for bit.
//   * Cache variants (qk_norm_rope_cache / rope_cache): the same pass also writes the token's
//     rotated k and its v into a paged KV cache at slot_mapping[t] (the reference's AGENTS.md
//     "slot_mapping": block_id * block_size + offset, so the cache [num_blocks, block_size,
//     num_kv_heads, head_dim] is addressed as [num_slots, num_kv_heads, head_dim]). v rides in
//     the same stage as q and k and is copied from shared memory; a negative slot skips the
//     token (padding), a slot past the cache raises SVLLM_DEVERR_BAD_INDEX and writes nothing.
//   * Plain path for everything else: one warp per token, element loads, still on the GPU.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cmath>
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "host_common.h"

namespace svllm::k {
namespace {

constexpr int kMaxHalfDim = 256;  // head_dim <= 512

struct RopeArgs {
  void* q;
  void* k;
  const void* q_weight;
  const void* k_weight;
  const void* positions;
  int64_t num_tokens;
  int64_t q_stride;  // elements between tokens
  int64_t k_stride;
  int num_heads;
  int num_kv_heads;
  int head_dim;
  int pos_is_i64;
  int norm_vec;  // plain path: the reference would load 8-element vectors
  int interleave;  // token order (WarpUnits)
  int early_dependents;  // let the next kernel be scheduled at this one's start
  float eps;
  int* err;
  // cache variants
  const void* v;
  const int64_t* slots;
  void* k_cache;  // [num_slots, num_kv_heads, head_dim]
  void* v_cache;
  int64_t v_stride;
  int64_t num_slots;
  // bulk-copy path
  int stages;
  int stage_bytes;
  int scratch_offset;  // per-warp cos/sin scratch, then the stage rings
  int ring_offset;
  float inv_freq[kMaxHalfDim];
};

__device__ __forceinline__ float load_position(const void* positions, int is_i64, int64_t t) {
  if (is_i64) {
    return __ll2float_rn(__ldg(static_cast<const long long*>(positions) + t));
  }
  return __int2float_rn(__ldg(static_cast<const int*>(positions) + t));
}

// Rotation of one lane's pair block: lo[e] = x[i], hi[e] = x[i + d/2] for kVec consecutive i,
// in fp32 with the storage type's rounding after every step.
template <class E>
__device__ __forceinline__ void rotate_pairs(float (&lo)[E::kPerVec], float (&hi)[E::kPerVec],
                                       const float (&c)[E::kPerVec],
                                       const float (&s)[E::kPerVec]) {
#pragma unroll
  for (int e = 0; e < E::kPerVec; ++e) {
    const float x1 = lo[e];
    const float x2 = hi[e];
    lo[e] = __fsub_rn(E::round(__fmul_rn(x1, c[e])), E::round(__fmul_rn(x2, s[e])));
    hi[e] = __fadd_rn(E::round(__fmul_rn(x2, c[e])), E::round(__fmul_rn(x1, s[e])));
  }
}

// cos and sin of one lane's kVec rotation pairs, rounded to the storage type (Hugging Face's
// rotary embedding returns them in the activation dtype), kept packed for bf16.
template <class E>
struct LaneTrig;

template <>
struct LaneTrig<Bf16> {
  uint32_t c[4], s[4];
  __device__ __forceinline__ void load(const float* cs, const float* sn) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      c[i] = pack_bf16x2(cs[2 * i], cs[2 * i + 1]);
      s[i] = pack_bf16x2(sn[2 * i], sn[2 * i + 1]);
    }
  }
  // lo = x[i], hi = x[i + d/2]: lo' = round(lo*c) - round(hi*s), hi' = round(hi*c) + round(lo*s)
  __device__ __forceinline__ void rotate(uint4& lo, uint4& hi) const {
    uint32_t l[4], h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t wl = word(lo, i), wh = word(hi, i);
      l[i] = bf16x2_sub(bf16x2_mul(wl, c[i]), bf16x2_mul(wh, s[i]));
      h[i] = bf16x2_add(bf16x2_mul(wh, c[i]), bf16x2_mul(wl, s[i]));
    }
    lo = make_uint4(l[0], l[1], l[2], l[3]);
    hi = make_uint4(h[0], h[1], h[2], h[3]);
  }
};

template <>
struct LaneTrig<F32> {
  float c[4], s[4];
  __device__ __forceinline__ void load(const float* cs, const float* sn) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      c[i] = cs[i];
      s[i] = sn[i];
    }
  }
  __device__ __forceinline__ void rotate(uint4& lo, uint4& hi) const {
    float l[4], h[4];
    unpack<F32>(lo, l);
    unpack<F32>(hi, h);
    rotate_pairs<F32>(l, h, c, s);
    lo = pack<F32>(l);
    hi = pack<F32>(h);
  }
};

// The cache slot of token t, or -1 for "write nothing" (a negative slot is padding; a slot past
// the cache is an error, raised by the caller of this helper).
__device__ __forceinline__ int64_t load_slot(const RopeArgs& a, int64_t t) {
  return __ldg(reinterpret_cast<const long long*>(a.slots) + t);
}

// 16-byte vectors of a token's v row each lane holds in registers (a 2 KB row per warp).
constexpr int kVRegs = 4;

// kPasses > 0: the token's heads take exactly kPasses passes of kWarpSize / G heads and the q heads
// fill whole passes, so the pass loop is unrolled and each pass is all-q or all-k (one weight,
// no per-lane select); the compiler interleaves the passes' independent chains. Measured on a
// B200 at 1M tokens of the Qwen3-0.6B shapes: 6586 GB/s against 6396 for the runtime loop.
// kPasses == 0: a runtime loop over any number of heads.
template <class E, int G, bool kNorm, bool kCache, int kPasses>
__global__ void __launch_bounds__(512) rope_bulk_kernel(const __grid_constant__ RopeArgs a) {
  grid_dependency_wait();
  if (a.early_dependents) allow_dependents();
  using S = typename E::Storage;
  constexpr int kVec = E::kPerVec;
  constexpr int kHalf = kVec * G;  // head_dim / 2
  constexpr int kDim = 2 * kHalf;
  constexpr int kHeadsPerPass = kWarpSize / G;
  extern __shared__ __align__(128) uint8_t smem[];

  const int warps = blockDim.x / kWarpSize;
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x % kWarpSize;
  const int sub = lane % G;
  const int num_heads = a.num_heads;
  const int total_heads = a.num_heads + a.num_kv_heads;
  const uint32_t q_bytes = static_cast<uint32_t>(num_heads) * kDim * sizeof(S);
  const uint32_t k_bytes = static_cast<uint32_t>(a.num_kv_heads) * kDim * sizeof(S);
  const uint32_t v_bytes = kCache ? k_bytes : 0;  // one v row per token, same shape as k

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * a.stages;
  float* inv_sm = reinterpret_cast<float*>(smem + a.scratch_offset);
  float* cos_sm = inv_sm + kHalf + warp * 2 * kHalf;
  float* sin_sm = cos_sm + kHalf;
  uint8_t* ring = smem + a.ring_offset + static_cast<size_t>(warp) * a.stages * a.stage_bytes;

  for (int i = threadIdx.x; i < kHalf; i += blockDim.x) inv_sm[i] = a.inv_freq[i];
  if (lane == 0) {
    for (int s = 0; s < a.stages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }

  // Per-lane norm weights: this lane's block of each half of q_weight and k_weight.
  uint4 qw_lo{}, qw_hi{}, kw_lo{}, kw_hi{};
  if constexpr (kNorm) {
    const uint8_t* qw = static_cast<const uint8_t*>(a.q_weight);
    const uint8_t* kw = static_cast<const uint8_t*>(a.k_weight);
    qw_lo = ld_global_nc_v4(qw + sub * 16);
    qw_hi = ld_global_nc_v4(qw + (kHalf * sizeof(S)) + sub * 16);
    kw_lo = ld_global_nc_v4(kw + sub * 16);
    kw_hi = ld_global_nc_v4(kw + (kHalf * sizeof(S)) + sub * 16);
  }
  __syncthreads();

  const WarpUnits wu = warp_units(a.num_tokens, static_cast<int64_t>(gridDim.x) * warps,
                                  static_cast<int64_t>(blockIdx.x) * warps + warp, a.interleave);
  const int64_t n = wu.count;
  const int64_t q_stride_b = a.q_stride * static_cast<int64_t>(sizeof(S));
  const int64_t k_stride_b = a.k_stride * static_cast<int64_t>(sizeof(S));
  const int64_t v_stride_b = a.v_stride * static_cast<int64_t>(sizeof(S));

  auto issue = [&](int64_t j) {
    const int s = static_cast<int>(j % a.stages);
    uint8_t* st = ring + static_cast<size_t>(s) * a.stage_bytes;
    const int64_t t = wu.at(j);
    mbar_arrive_expect_tx(&bars[s], q_bytes + k_bytes);
    if (q_bytes) bulk_load(st, static_cast<const uint8_t*>(a.q) + t * q_stride_b, q_bytes, &bars[s]);
    if (k_bytes) {
      bulk_load(st + q_bytes, static_cast<const uint8_t*>(a.k) + t * k_stride_b, k_bytes, &bars[s]);
    }
  };

  if (lane == 0) {
    for (int64_t j = 0; j < min(static_cast<int64_t>(a.stages), n); ++j) issue(j);
  }

  // Positions run one token ahead of use, so their load latency hides behind a token's work.
  float pos_next = n > 0 ? load_position(a.positions, a.pos_is_i64, wu.at(0)) : 0.0f;
  int64_t slot_next = kCache && n > 0 ? load_slot(a, wu.at(0)) : -1;

  int64_t j = 0;
  for (; j < n; ++j) {
    const float pos = pos_next;
    if (j + 1 < n) pos_next = load_position(a.positions, a.pos_is_i64, wu.at(j + 1));
    int64_t slot = -1;
    if constexpr (kCache) {
      slot = slot_next;
      if (j + 1 < n) slot_next = load_slot(a, wu.at(j + 1));
      if (slot >= a.num_slots) {
        if (lane == 0) raise_error(a.err, kErrBadIndex);
        slot = -1;
      }
    }

    // The token's v row goes to the cache unchanged: it is loaded into registers here (up to
    // kVRegs vectors per lane) and stored after the heads, so it needs no shared memory and its
    // load latency hides behind the token's work.
    uint4 vr[kVRegs];
    if constexpr (kCache) {
      const uint8_t* vs = static_cast<const uint8_t*>(a.v) + wu.at(j) * v_stride_b;
#pragma unroll
      for (int r = 0; r < kVRegs; ++r) {
        const uint32_t b = (lane + r * kWarpSize) * 16;
        if (slot >= 0 && b < v_bytes) vr[r] = ld_global_nc_v4(vs + b);
      }
    }

    // The token's (cos, sin) table, shared by every head.
    for (int i = lane; i < kHalf; i += kWarpSize) {
      const float angle = __fmul_rn(pos, inv_sm[i]);
      sincosf(angle, &sin_sm[i], &cos_sm[i]);
    }
    __syncwarp();
    LaneTrig<E> trig;
    trig.load(cos_sm + sub * kVec, sin_sm + sub * kVec);

    const int stage = static_cast<int>(j % a.stages);
    const uint32_t parity = static_cast<uint32_t>((j / a.stages) & 1);
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bars[stage], parity))) break;
    const uint8_t* st = ring + static_cast<size_t>(stage) * a.stage_bytes;
    const int64_t t = wu.at(j);

    // One pass: heads h0 .. h0 + kHeadsPerPass - 1, lane / G picking the head. q_pass: the
    // pass is all q heads (kPasses > 0), else each lane checks its own head.
    auto head_pass = [&](int h0, bool q_pass) {
      const int h = h0 + lane / G;
      const bool valid = h < total_heads;
      const uint8_t* hs = st + static_cast<size_t>(valid ? h : 0) * kDim * sizeof(S);
      uint4 lo = ld_shared_v4(hs + sub * 16);
      uint4 hi = ld_shared_v4(hs + kHalf * sizeof(S) + sub * 16);
      const bool is_q = kPasses > 0 ? q_pass : h < num_heads;
      if constexpr (kNorm) {
        // The head's sum of squares in the order of the reference's rms_norm kernel run on the
        // [tokens * heads, head_dim] view: lane j holds that kernel's vectors j (lo) and j + G
        // (hi); its xor tree first adds vector j + G to vector j (offset G), then reduces over
        // the G lanes; at head_dim 512 the two halves are two warps whose sums are added last.
        float lf[kVec], hf[kVec];
        unpack<E>(lo, lf);
        unpack<E>(hi, hf);
        float p_lo = 0.0f, p_hi = 0.0f;
        // bf16: element e of each half as one fp32 pair, so the two running sums and the two
        // scalings take one packed instruction per element (same roundings, same order)
        uint64_t pair[kVec];
        if constexpr (std::is_same_v<E, Bf16>) {
          uint64_t acc = f32x2(0.0f, 0.0f);
#pragma unroll
          for (int e = 0; e < kVec; ++e) {
            pair[e] = f32x2(lf[e], hf[e]);
            acc = f32x2_fma(pair[e], pair[e], acc);
          }
          f32x2_split(acc, p_lo, p_hi);
        } else {
#pragma unroll
          for (int e = 0; e < kVec; ++e) {
            p_lo = __fmaf_rn(lf[e], lf[e], p_lo);
            p_hi = __fmaf_rn(hf[e], hf[e], p_hi);
          }
        }
        float total;
        if constexpr (2 * G <= kWarpSize) {
          total = group_sum<G>(__fadd_rn(p_lo, p_hi));
        } else {
          total = __fadd_rn(group_sum<G>(p_lo), group_sum<G>(p_hi));
        }
        // sum / head_dim: head_dim is a power of two here, so the multiply is exact
        const float inv_rms = rsqrtf(__fadd_rn(__fmul_rn(total, 1.0f / kDim), a.eps));
        if constexpr (std::is_same_v<E, Bf16>) {
          // round(round(x * inv_rms) * w), as normalize_vec computes it
          const uint64_t inv2 = f32x2(inv_rms, inv_rms);
          float nl[kVec], nh[kVec];
#pragma unroll
          for (int e = 0; e < kVec; ++e) f32x2_split(f32x2_mul(pair[e], inv2), nl[e], nh[e]);
          const uint4& wl = is_q ? qw_lo : kw_lo;
          const uint4& wh = is_q ? qw_hi : kw_hi;
          uint32_t rl[4], rh[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            rl[i] = bf16x2_mul(pack_bf16x2(nl[2 * i], nl[2 * i + 1]), word(wl, i));
            rh[i] = bf16x2_mul(pack_bf16x2(nh[2 * i], nh[2 * i + 1]), word(wh, i));
          }
          lo = make_uint4(rl[0], rl[1], rl[2], rl[3]);
          hi = make_uint4(rh[0], rh[1], rh[2], rh[3]);
        } else {
          lo = normalize_vec<E>(lo, inv_rms, is_q ? qw_lo : kw_lo);
          hi = normalize_vec<E>(hi, inv_rms, is_q ? qw_hi : kw_hi);
        }
      }
      trig.rotate(lo, hi);
      if (valid) {
        S* dst = is_q ? static_cast<S*>(a.q) + t * a.q_stride + static_cast<int64_t>(h) * kDim
                      : static_cast<S*>(a.k) + t * a.k_stride +
                            static_cast<int64_t>(h - num_heads) * kDim;
        st_global_v4(dst + sub * kVec, lo);
        st_global_v4(dst + kHalf + sub * kVec, hi);
        if constexpr (kCache) {
          if (!is_q && slot >= 0) {
            S* kc = static_cast<S*>(a.k_cache) + slot * a.num_kv_heads * kDim +
                    static_cast<int64_t>(h - num_heads) * kDim;
            st_global_v4(kc + sub * kVec, lo);
            st_global_v4(kc + kHalf + sub * kVec, hi);
          }
        }
      }
    };
    if constexpr (kPasses > 0) {
#pragma unroll
      for (int p = 0; p < kPasses; ++p) head_pass(p * kHeadsPerPass, p * kHeadsPerPass < num_heads);
    } else {
      for (int h0 = 0; h0 < total_heads; h0 += kHeadsPerPass) head_pass(h0, false);
    }
    if constexpr (kCache) {
      if (slot >= 0) {
        uint8_t* vc = static_cast<uint8_t*>(a.v_cache) + slot * static_cast<int64_t>(v_bytes);
#pragma unroll
        for (int r = 0; r < kVRegs; ++r) {
          const uint32_t b = (lane + r * kWarpSize) * 16;
          if (b < v_bytes) st_global_v4(vc + b, vr[r]);
        }
        // rows longer than the registers hold: the rest copied directly
        const uint8_t* vs = static_cast<const uint8_t*>(a.v) + wu.at(j) * v_stride_b;
        for (uint32_t b = (lane + kVRegs * kWarpSize) * 16; b < v_bytes; b += kWarpSize * 16) {
          st_global_v4(vc + b, ld_global_nc_v4(vs + b));
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
    if (lane == 0) {
      raise_error(a.err, kErrWaitTimeout);
      for (int64_t m = j; m < min(j + a.stages, n); ++m) {
        mbar_wait_bounded(&bars[m % a.stages], static_cast<uint32_t>((m / a.stages) & 1));
      }
    }
    __syncwarp();
  }
}

// 1 / RMS of one head of n values, summed by one warp in the order of the reference's rms_norm
// kernel on that row: a CTA of round_up(units, 32) threads, thread t summing unit t (an 8-element
// vector when vec, else one element), per-warp xor trees, then a final 32-slot xor tree over the
// warp sums with zeros past the last warp. Lane l plays thread l + 32 w of every warp w.
template <class E>
__device__ float reference_order_inv_rms(const typename E::Storage* x, int n, float eps, int vec,
                                         int lane) {
  constexpr int kMaxWarps = 32;
  const int per = vec ? 8 : 1;
  const int units = n / per;
  const int num_warps = (units + kWarpSize - 1) / kWarpSize;
  float slots[kMaxWarps];
  for (int w = 0; w < kMaxWarps; ++w) {
    float p = 0.0f;
    const int u = w * kWarpSize + lane;
    if (w < num_warps && u < units) {
      for (int j = 0; j < per; ++j) {
        const float f = E::to_float(x[u * per + j]);
        p = __fmaf_rn(f, f, p);
      }
    }
    slots[w] = w < num_warps ? group_sum<kWarpSize>(p) : 0.0f;
  }
  for (int off = kMaxWarps / 2; off >= 1; off /= 2) {
    for (int i = 0; i < off; ++i) slots[i] = __fadd_rn(slots[i], slots[i + off]);
  }
  return rsqrtf(__fadd_rn(__fdiv_rn(slots[0], static_cast<float>(n)), eps));
}

// Plain path: one warp per token, any head_dim (even), any alignment.
template <class E, bool kNorm, bool kCache>
__global__ void __launch_bounds__(256) rope_plain_kernel(const __grid_constant__ RopeArgs a) {
  grid_dependency_sync();
  using S = typename E::Storage;
  const int lane = threadIdx.x % kWarpSize;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x / kWarpSize);
  const int dim = a.head_dim;
  const int half = dim / 2;
  const int total_heads = a.num_heads + a.num_kv_heads;
  const S* qw = static_cast<const S*>(a.q_weight);
  const S* kw = static_cast<const S*>(a.k_weight);
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x / kWarpSize) +
                   threadIdx.x / kWarpSize;
       t < a.num_tokens; t += warps_total) {
    const float pos = load_position(a.positions, a.pos_is_i64, t);
    int64_t slot = -1;
    if constexpr (kCache) {
      slot = load_slot(a, t);
      if (slot >= a.num_slots) {
        if (lane == 0) raise_error(a.err, kErrBadIndex);
        slot = -1;
      }
    }
    for (int h = 0; h < total_heads; ++h) {
      const bool is_q = h < a.num_heads;
      S* x = is_q ? static_cast<S*>(a.q) + t * a.q_stride + static_cast<int64_t>(h) * dim
                  : static_cast<S*>(a.k) + t * a.k_stride + static_cast<int64_t>(h - a.num_heads) * dim;
      float inv_rms = 1.0f;
      if constexpr (kNorm) {
        inv_rms = reference_order_inv_rms<E>(x, dim, a.eps, a.norm_vec, lane);
      }
      __syncwarp();
      for (int i = lane; i < half; i += kWarpSize) {
        float lo[E::kPerVec] = {}, hi[E::kPerVec] = {}, c[E::kPerVec] = {}, s[E::kPerVec] = {};
        lo[0] = E::to_float(x[i]);
        hi[0] = E::to_float(x[i + half]);
        if constexpr (kNorm) {
          const S* w = is_q ? qw : kw;
          lo[0] = E::round(__fmul_rn(E::round(__fmul_rn(lo[0], inv_rms)), E::to_float(w[i])));
          hi[0] = E::round(__fmul_rn(E::round(__fmul_rn(hi[0], inv_rms)), E::to_float(w[i + half])));
        }
        const float angle = __fmul_rn(pos, a.inv_freq[i]);
        c[0] = E::round(cosf(angle));
        s[0] = E::round(sinf(angle));
        rotate_pairs<E>(lo, hi, c, s);
        x[i] = E::from_float(lo[0]);
        x[i + half] = E::from_float(hi[0]);
        if constexpr (kCache) {
          if (!is_q && slot >= 0) {
            S* kc = static_cast<S*>(a.k_cache) + (slot * a.num_kv_heads + (h - a.num_heads)) * dim;
            kc[i] = E::from_float(lo[0]);
            kc[i + half] = E::from_float(hi[0]);
          }
        }
      }
      __syncwarp();
    }
    if constexpr (kCache) {
      if (slot >= 0) {
        const S* v = static_cast<const S*>(a.v) + t * a.v_stride;
        S* vc = static_cast<S*>(a.v_cache) + slot * a.num_kv_heads * dim;
        for (int i = lane; i < a.num_kv_heads * dim; i += kWarpSize) vc[i] = v[i];
      }
    }
  }
}

using RopeKernel = void (*)(RopeArgs);

template <class E, bool kNorm, bool kCache>
RopeKernel pick_bulk_kernel(int head_dim, int num_heads, int num_kv_heads) {
  constexpr int kVec = E::kPerVec;
  if (head_dim % (2 * kVec) != 0) return nullptr;
  const int g = head_dim / (2 * kVec);
  const int per_pass = g > 0 && g <= kWarpSize ? kWarpSize / g : 0;
  const int total = num_heads + num_kv_heads;
  // unrolled kernels for the head layouts of the Qwen3 (24 or 40 heads of 128) and Llama-3.2
  // (40 heads of 64) families: bf16, q heads filling whole passes
  const bool whole = per_pass > 0 && num_heads % per_pass == 0 && total % per_pass == 0;
  const int passes = whole ? total / per_pass : 0;
  if constexpr (sizeof(typename E::Storage) == 2) {
    if (g == 8 && passes == 6) return rope_bulk_kernel<E, 8, kNorm, kCache, 6>;
    if (g == 8 && passes == 10) return rope_bulk_kernel<E, 8, kNorm, kCache, 10>;
    if (g == 4 && passes == 5) return rope_bulk_kernel<E, 4, kNorm, kCache, 5>;
  }
  switch (g) {
    case 2: return rope_bulk_kernel<E, 2, kNorm, kCache, 0>;
    case 4: return rope_bulk_kernel<E, 4, kNorm, kCache, 0>;
    case 8: return rope_bulk_kernel<E, 8, kNorm, kCache, 0>;
    case 16: return rope_bulk_kernel<E, 16, kNorm, kCache, 0>;
    case 32: return rope_bulk_kernel<E, 32, kNorm, kCache, 0>;
    default: return nullptr;
  }
}

// The paged-KV destination of the cache variants (all null / zero without one).
struct CacheTarget {
  const void* v = nullptr;
  const int64_t* slots = nullptr;
  void* k_cache = nullptr;
  void* v_cache = nullptr;
  int64_t v_stride = 0;
  int64_t num_slots = 0;
};

template <class E, bool kNorm, bool kCache>
int launch_rope(void* q, void* k, const void* q_weight, const void* k_weight,
                const void* positions, int pos_type, int64_t num_tokens, int64_t num_heads,
                int64_t num_kv_heads, int64_t head_dim, int64_t q_stride, int64_t k_stride,
                float eps, const float* inv_freq, const CacheTarget& cache, cudaStream_t stream) {
  using S = typename E::Storage;
  if (kCache && (num_kv_heads <= 0 || cache.num_slots < 0 ||
                 cache.v_stride < num_kv_heads * head_dim)) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  if (num_tokens < 0 || num_heads < 0 || num_kv_heads < 0 || head_dim <= 0 || head_dim % 2 != 0 ||
      head_dim > 2 * kMaxHalfDim || (pos_type != SVLLM_INDEX_I32 && pos_type != SVLLM_INDEX_I64) ||
      (num_heads > 0 && q_stride < num_heads * head_dim) ||
      (num_kv_heads > 0 && k_stride < num_kv_heads * head_dim) || inv_freq == nullptr) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  if (num_tokens == 0 || num_heads + num_kv_heads == 0) return SVLLM_OK;
  if (positions == nullptr || (num_heads > 0 && q == nullptr) ||
      (num_kv_heads > 0 && k == nullptr) ||
      (kNorm && ((num_heads > 0 && q_weight == nullptr) ||
                 (num_kv_heads > 0 && k_weight == nullptr)))) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  if (kCache && (cache.v == nullptr || cache.slots == nullptr || cache.k_cache == nullptr ||
                 cache.v_cache == nullptr)) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  if (kCache && (reinterpret_cast<uintptr_t>(cache.slots) & 7u) != 0) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  if (num_heads + num_kv_heads > (1 << 16)) return SVLLM_ERR_TOO_LARGE;

  int device;
  if (current_device(&device) != SVLLM_OK) return SVLLM_ERR_CUDA;
  int* err = library_error_word(device);
  if (err == nullptr) return SVLLM_ERR_CUDA;

  RopeArgs a{};
  a.q = q;
  a.k = k;
  // A missing weight is never read: its heads do not exist. Point it at the other one so the
  // kernel's unconditional per-lane weight loads stay in bounds.
  a.q_weight = q_weight != nullptr ? q_weight : k_weight;
  a.k_weight = k_weight != nullptr ? k_weight : q_weight;
  a.positions = positions;
  a.num_tokens = num_tokens;
  a.q_stride = q_stride;
  a.k_stride = k_stride;
  a.num_heads = static_cast<int>(num_heads);
  a.num_kv_heads = static_cast<int>(num_kv_heads);
  a.head_dim = static_cast<int>(head_dim);
  a.pos_is_i64 = pos_type == SVLLM_INDEX_I64;
  a.interleave = 1;  // measured faster than contiguous shares on B200
  a.eps = eps;
  a.err = err;
  a.v = cache.v;
  a.slots = cache.slots;
  a.k_cache = cache.k_cache;
  a.v_cache = cache.v_cache;
  a.v_stride = cache.v_stride;
  a.num_slots = cache.num_slots;
  std::memcpy(a.inv_freq, inv_freq, sizeof(float) * (head_dim / 2));
  a.norm_vec = sizeof(S) == 2 && head_dim % 8 == 0 && aligned16(q) && aligned16(k) &&
               (q_stride * sizeof(S)) % 16 == 0 && (k_stride * sizeof(S)) % 16 == 0 &&
               (!kNorm || (aligned16(a.q_weight) && aligned16(a.k_weight)));

  const int64_t head_bytes = head_dim * static_cast<int64_t>(sizeof(S));
  const int64_t q_bytes = num_heads * head_bytes;
  const int64_t k_bytes = num_kv_heads * head_bytes;
  const int64_t v_bytes = kCache ? k_bytes : 0;
  const bool bulk_ok =
      (num_heads == 0 || (aligned16(q) && (q_stride * sizeof(S)) % 16 == 0)) &&
      (num_kv_heads == 0 || (aligned16(k) && (k_stride * sizeof(S)) % 16 == 0)) &&
      (!kNorm || (aligned16(a.q_weight) && aligned16(a.k_weight))) &&
      (!kCache || (aligned16(cache.v) && (cache.v_stride * sizeof(S)) % 16 == 0 &&
                   aligned16(cache.k_cache) && aligned16(cache.v_cache)));
  const RopeKernel kernel =
      bulk_ok ? pick_bulk_kernel<E, kNorm, kCache>(static_cast<int>(head_dim),
                                                   static_cast<int>(num_heads),
                                                   static_cast<int>(num_kv_heads))
              : nullptr;
  if (kernel != nullptr) {
    const PipelineShape shape = pipeline_shape(kNorm ? OpId::kQkNormRope : OpId::kRope);
    a.stage_bytes = static_cast<int>(round_up(q_bytes + k_bytes, 128));  // v is not staged
    int warps = warps_for(num_tokens, shape.warps, device);
    int stages = shape.stages;
    const int64_t half = head_dim / 2;
    auto smem_for = [&](int w, int s) {
      return round_up(static_cast<int64_t>(w) * s * 8, 128) +
             round_up((half + static_cast<int64_t>(w) * 2 * half) * 4, 128) +
             static_cast<int64_t>(w) * s * a.stage_bytes;
    };
    while (smem_for(warps, stages) > static_cast<int64_t>(kMaxSmemPerCta) && stages > 2) --stages;
    while (smem_for(warps, stages) > static_cast<int64_t>(kMaxSmemPerCta) && warps > 1) --warps;
    if (smem_for(warps, stages) <= static_cast<int64_t>(kMaxSmemPerCta) &&
        q_bytes + k_bytes + v_bytes < (1 << 20)) {
      a.stages = stages;
      a.scratch_offset = static_cast<int>(round_up(static_cast<int64_t>(warps) * stages * 8, 128));
      a.ring_offset = a.scratch_offset +
                      static_cast<int>(round_up((half + static_cast<int64_t>(warps) * 2 * half) * 4, 128));
      const size_t smem = static_cast<size_t>(smem_for(warps, stages));
      const int threads = warps * kWarpSize;
      const int per_sm = blocks_per_sm(reinterpret_cast<const void*>(kernel), threads, smem, device);
      if (per_sm > 0) {
        const int64_t grid = persistent_grid((num_tokens + warps - 1) / warps, device, per_sm);
        a.early_dependents = early_dependents(num_tokens * (2 * (q_bytes + k_bytes) + 3 * v_bytes));
        return launch(kernel, dim3(static_cast<unsigned>(grid)), dim3(threads), smem, stream, 1,
                      a);
      }
    }
  }

  const int64_t grid = persistent_grid((num_tokens + 7) / 8, device, 8);
  return launch(rope_plain_kernel<E, kNorm, kCache>, dim3(static_cast<unsigned>(grid)), dim3(256),
                0, stream, 1, a);
}

}  // namespace
}  // namespace svllm::k

using svllm::k::Bf16;
using svllm::k::F32;
using svllm::k::launch_rope;

extern "C" {

int svllm_qk_norm_rope_bf16(void* q, void* k, const void* q_weight, const void* k_weight,
                            const void* positions, int pos_type, int64_t num_tokens,
                            int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                            int64_t q_row_stride, int64_t k_row_stride, float eps,
                            const float* inv_freq, svllm_stream stream) {
  return launch_rope<Bf16, true, false>(q, k, q_weight, k_weight, positions, pos_type,
                                        num_tokens, num_heads, num_kv_heads, head_dim,
                                        q_row_stride, k_row_stride, eps, inv_freq, {},
                                        reinterpret_cast<cudaStream_t>(stream));
}

int svllm_qk_norm_rope_f32(float* q, float* k, const float* q_weight, const float* k_weight,
                           const void* positions, int pos_type, int64_t num_tokens,
                           int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                           int64_t q_row_stride, int64_t k_row_stride, float eps,
                           const float* inv_freq, svllm_stream stream) {
  return launch_rope<F32, true, false>(q, k, q_weight, k_weight, positions, pos_type,
                                       num_tokens, num_heads, num_kv_heads, head_dim,
                                       q_row_stride, k_row_stride, eps, inv_freq, {},
                                       reinterpret_cast<cudaStream_t>(stream));
}

int svllm_rope_bf16(void* q, void* k, const void* positions, int pos_type, int64_t num_tokens,
                    int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                    int64_t q_row_stride, int64_t k_row_stride, const float* inv_freq,
                    svllm_stream stream) {
  return launch_rope<Bf16, false, false>(q, k, nullptr, nullptr, positions, pos_type,
                                         num_tokens, num_heads, num_kv_heads, head_dim,
                                         q_row_stride, k_row_stride, 0.0f, inv_freq, {},
                                         reinterpret_cast<cudaStream_t>(stream));
}

int svllm_rope_f32(float* q, float* k, const void* positions, int pos_type, int64_t num_tokens,
                   int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                   int64_t q_row_stride, int64_t k_row_stride, const float* inv_freq,
                   svllm_stream stream) {
  return launch_rope<F32, false, false>(q, k, nullptr, nullptr, positions, pos_type,
                                        num_tokens, num_heads, num_kv_heads, head_dim,
                                        q_row_stride, k_row_stride, 0.0f, inv_freq, {},
                                        reinterpret_cast<cudaStream_t>(stream));
}

namespace {

svllm::k::CacheTarget cache_target(const void* v, const int64_t* slot_mapping, void* k_cache,
                                   void* v_cache, int64_t num_slots, int64_t v_row_stride) {
  svllm::k::CacheTarget c;
  c.v = v;
  c.slots = slot_mapping;
  c.k_cache = k_cache;
  c.v_cache = v_cache;
  c.num_slots = num_slots;
  c.v_stride = v_row_stride;
  return c;
}

}  // namespace

int svllm_qk_norm_rope_cache_bf16(void* q, void* k, const void* v, const void* q_weight,
                                  const void* k_weight, const void* positions, int pos_type,
                                  const int64_t* slot_mapping, void* k_cache, void* v_cache,
                                  int64_t num_slots, int64_t num_tokens, int64_t num_heads,
                                  int64_t num_kv_heads, int64_t head_dim, int64_t q_row_stride,
                                  int64_t k_row_stride, int64_t v_row_stride, float eps,
                                  const float* inv_freq, svllm_stream stream) {
  return launch_rope<Bf16, true, true>(
      q, k, q_weight, k_weight, positions, pos_type, num_tokens, num_heads, num_kv_heads,
      head_dim, q_row_stride, k_row_stride, eps, inv_freq,
      cache_target(v, slot_mapping, k_cache, v_cache, num_slots, v_row_stride),
      reinterpret_cast<cudaStream_t>(stream));
}

int svllm_qk_norm_rope_cache_f32(float* q, float* k, const float* v, const float* q_weight,
                                 const float* k_weight, const void* positions, int pos_type,
                                 const int64_t* slot_mapping, float* k_cache, float* v_cache,
                                 int64_t num_slots, int64_t num_tokens, int64_t num_heads,
                                 int64_t num_kv_heads, int64_t head_dim, int64_t q_row_stride,
                                 int64_t k_row_stride, int64_t v_row_stride, float eps,
                                 const float* inv_freq, svllm_stream stream) {
  return launch_rope<F32, true, true>(
      q, k, q_weight, k_weight, positions, pos_type, num_tokens, num_heads, num_kv_heads,
      head_dim, q_row_stride, k_row_stride, eps, inv_freq,
      cache_target(v, slot_mapping, k_cache, v_cache, num_slots, v_row_stride),
      reinterpret_cast<cudaStream_t>(stream));
}

int svllm_rope_cache_bf16(void* q, void* k, const void* v, const void* positions, int pos_type,
                          const int64_t* slot_mapping, void* k_cache, void* v_cache,
                          int64_t num_slots, int64_t num_tokens, int64_t num_heads,
                          int64_t num_kv_heads, int64_t head_dim, int64_t q_row_stride,
                          int64_t k_row_stride, int64_t v_row_stride, const float* inv_freq,
                          svllm_stream stream) {
  return launch_rope<Bf16, false, true>(
      q, k, nullptr, nullptr, positions, pos_type, num_tokens, num_heads, num_kv_heads, head_dim,
      q_row_stride, k_row_stride, 0.0f, inv_freq,
      cache_target(v, slot_mapping, k_cache, v_cache, num_slots, v_row_stride),
      reinterpret_cast<cudaStream_t>(stream));
}

int svllm_rope_cache_f32(float* q, float* k, const float* v, const void* positions, int pos_type,
                         const int64_t* slot_mapping, float* k_cache, float* v_cache,
                         int64_t num_slots, int64_t num_tokens, int64_t num_heads,
                         int64_t num_kv_heads, int64_t head_dim, int64_t q_row_stride,
                         int64_t k_row_stride, int64_t v_row_stride, const float* inv_freq,
                         svllm_stream stream) {
  return launch_rope<F32, false, true>(
      q, k, nullptr, nullptr, positions, pos_type, num_tokens, num_heads, num_kv_heads, head_dim,
      q_row_stride, k_row_stride, 0.0f, inv_freq,
      cache_target(v, slot_mapping, k_cache, v_cache, num_slots, v_row_stride),
      reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

extern "C" int svllm_rope_inv_freq(double theta, int64_t head_dim,
                                   const svllm_llama3_scaling* scaling, float* inv_freq) {
  // Hugging Face's fp32 formula, one fp32 operation per step. torch evaluates `scalar / tensor`
  // as reciprocal(tensor) * scalar and `tensor / scalar` as a true division; so does this.
  if (!(theta > 0.0) || head_dim <= 0 || head_dim % 2 != 0 || inv_freq == nullptr) {
    return SVLLM_ERR_INVALID_ARGUMENT;
  }
  const int64_t half = head_dim / 2;
  const float base = static_cast<float>(theta);
  for (int64_t i = 0; i < half; ++i) {
    const float e = static_cast<float>(2 * i) / static_cast<float>(head_dim);
    inv_freq[i] = 1.0f / powf(base, e);
  }
  if (scaling != nullptr) {
    const svllm_llama3_scaling& s = *scaling;
    if (!(s.factor > 0.0) || !(s.high_freq_factor > s.low_freq_factor) ||
        !(s.low_freq_factor > 0.0) || s.original_max_position_embeddings <= 0) {
      return SVLLM_ERR_INVALID_ARGUMENT;
    }
    const float factor = static_cast<float>(s.factor);
    const float low = static_cast<float>(s.low_freq_factor);
    const float old_len = static_cast<float>(s.original_max_position_embeddings);
    const float low_wavelen =
        static_cast<float>(static_cast<double>(s.original_max_position_embeddings) / s.low_freq_factor);
    const float high_wavelen =
        static_cast<float>(static_cast<double>(s.original_max_position_embeddings) / s.high_freq_factor);
    const float two_pi = static_cast<float>(2.0 * 3.14159265358979323846);
    const float span = static_cast<float>(s.high_freq_factor - s.low_freq_factor);
    for (int64_t i = 0; i < half; ++i) {
      const float inv = inv_freq[i];
      const float wavelen = (1.0f / inv) * two_pi;
      const float scaled = wavelen > low_wavelen ? inv / factor : inv;
      const float smooth = ((1.0f / wavelen) * old_len - low) / span;
      const float smoothed = (1.0f - smooth) * scaled / factor + smooth * scaled;
      const bool medium = !(wavelen < high_wavelen) && !(wavelen > low_wavelen);
      inv_freq[i] = medium ? smoothed : scaled;
    }
  }
  return SVLLM_OK;
}

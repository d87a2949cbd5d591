// OpenMP kernel of ops::rope and ops::qk_norm_rope for CPU tensors, on torch's thread pool.
#include <ATen/Parallel.h>
#include <c10/util/BFloat16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

#include "ops/rope_kernels.h"

namespace svllm::ops::cpu_impl {
namespace {

inline float bf16_round(float v) { return static_cast<float>(static_cast<at::BFloat16>(v)); }

// Qwen3RMSNorm of one head in place.
void norm_head(at::BFloat16* x, const at::BFloat16* w, int64_t dim, float eps) {
  float sum_sq = 0.0f;
  for (int64_t i = 0; i < dim; ++i) {
    const float v = static_cast<float>(x[i]);
    sum_sq += v * v;
  }
  const float inv_rms = 1.0f / std::sqrt(sum_sq / static_cast<float>(dim) + eps);
  for (int64_t i = 0; i < dim; ++i) {
    const float normed = bf16_round(static_cast<float>(x[i]) * inv_rms);
    x[i] = static_cast<at::BFloat16>(normed * static_cast<float>(w[i]));
  }
}

// apply_rotary_pos_emb on one head in place, cos/sin already rounded to bf16.
void rotate_head(at::BFloat16* x, const float* c, const float* s, int64_t half) {
  for (int64_t i = 0; i < half; ++i) {
    const float x1 = static_cast<float>(x[i]);
    const float x2 = static_cast<float>(x[i + half]);
    x[i] = static_cast<at::BFloat16>(bf16_round(x1 * c[i]) - bf16_round(x2 * s[i]));
    x[i + half] = static_cast<at::BFloat16>(bf16_round(x2 * c[i]) + bf16_round(x1 * s[i]));
  }
}

}  // namespace

void rope(const at::Tensor& q, const at::Tensor& k, const at::Tensor& q_weight,
          const at::Tensor& k_weight, const at::Tensor& positions, double eps,
          const float* inv_freq) {
  const int64_t num_tokens = q.size(0);
  const int64_t num_heads = q.size(1);
  const int64_t num_kv_heads = k.size(1);
  const int64_t dim = q.size(2);
  const int64_t half = dim / 2;
  const int64_t q_stride = q.stride(0);
  const int64_t k_stride = k.stride(0);
  auto* qp = q.mutable_data_ptr<at::BFloat16>();
  auto* kp = k.mutable_data_ptr<at::BFloat16>();
  const bool norm = q_weight.defined();
  const at::BFloat16* qw = norm ? q_weight.const_data_ptr<at::BFloat16>() : nullptr;
  const at::BFloat16* kw = norm ? k_weight.const_data_ptr<at::BFloat16>() : nullptr;
  const bool pos64 = positions.scalar_type() == at::kLong;
  const void* pos = positions.const_data_ptr();
  const float eps_f = static_cast<float>(eps);

  at::parallel_for(0, num_tokens, 16, [&](int64_t begin, int64_t end) {
    std::vector<float> c(static_cast<size_t>(half));
    std::vector<float> s(static_cast<size_t>(half));
    for (int64_t t = begin; t < end; ++t) {
      const float p = pos64 ? static_cast<float>(static_cast<const int64_t*>(pos)[t])
                            : static_cast<float>(static_cast<const int32_t*>(pos)[t]);
      for (int64_t i = 0; i < half; ++i) {
        const float angle = p * inv_freq[i];
        c[i] = bf16_round(std::cos(angle));
        s[i] = bf16_round(std::sin(angle));
      }
      for (int64_t h = 0; h < num_heads; ++h) {
        at::BFloat16* x = qp + t * q_stride + h * dim;
        if (norm) norm_head(x, qw, dim, eps_f);
        rotate_head(x, c.data(), s.data(), half);
      }
      for (int64_t h = 0; h < num_kv_heads; ++h) {
        at::BFloat16* x = kp + t * k_stride + h * dim;
        if (norm) norm_head(x, kw, dim, eps_f);
        rotate_head(x, c.data(), s.data(), half);
      }
    }
  });
}

int64_t write_kv_cache(const at::Tensor& k, const at::Tensor& v, const at::Tensor& slot_mapping,
                       const at::Tensor& k_cache, const at::Tensor& v_cache) {
  const int64_t num_tokens = k.size(0);
  const int64_t row = k.size(1) * k.size(2);  // elements of one slot
  const int64_t num_slots = k_cache.size(0);
  const auto* slots = slot_mapping.const_data_ptr<int64_t>();
  const auto* kp = k.const_data_ptr<at::BFloat16>();
  const auto* vp = v.const_data_ptr<at::BFloat16>();
  auto* kc = k_cache.mutable_data_ptr<at::BFloat16>();
  auto* vc = v_cache.mutable_data_ptr<at::BFloat16>();
  int64_t bad = 0;
  for (int64_t t = 0; t < num_tokens; ++t) {
    const int64_t s = slots[t];
    if (s < 0) continue;
    if (s >= num_slots) {
      ++bad;
      continue;
    }
    std::copy(kp + t * k.stride(0), kp + t * k.stride(0) + row, kc + s * row);
    std::copy(vp + t * v.stride(0), vp + t * v.stride(0) + row, vc + s * row);
  }
  return bad;
}

}  // namespace svllm::ops::cpu_impl

#pragma once

// Per-device kernels behind ops::rope and ops::qk_norm_rope, which validate the inputs; include
// this only from the dispatch and the kernels themselves.

#include <ATen/core/Tensor.h>

namespace svllm::ops {

// q [num_tokens, num_heads, head_dim] and k [num_tokens, num_kv_heads, head_dim] views (heads
// and head_dim contiguous); q_weight / k_weight undefined for rope alone; inv_freq is a host
// array of head_dim / 2 floats.
// The cache variants take v [num_tokens, num_kv_heads, head_dim] (token stride free), int64
// slot_mapping [num_tokens] and contiguous caches viewed as [num_slots, num_kv_heads, head_dim].
namespace cpu_impl {
void rope(const at::Tensor& q, const at::Tensor& k, const at::Tensor& q_weight,
          const at::Tensor& k_weight, const at::Tensor& positions, double eps,
          const float* inv_freq);
// Returns the number of slots past the cache (their tokens write nothing).
int64_t write_kv_cache(const at::Tensor& k, const at::Tensor& v, const at::Tensor& slot_mapping,
                       const at::Tensor& k_cache, const at::Tensor& v_cache);
}  // namespace cpu_impl

namespace cuda_impl {
void rope(const at::Tensor& q, const at::Tensor& k, const at::Tensor& q_weight,
          const at::Tensor& k_weight, const at::Tensor& positions, double eps,
          const float* inv_freq);
void rope_cache(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                const at::Tensor& q_weight, const at::Tensor& k_weight,
                const at::Tensor& positions, const at::Tensor& slot_mapping,
                const at::Tensor& k_cache, const at::Tensor& v_cache, double eps,
                const float* inv_freq);
}  // namespace cuda_impl

}  // namespace svllm::ops

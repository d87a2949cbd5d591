#pragma once

// Per-device kernels behind ops::rope and ops::qk_norm_rope, which validate the inputs; include
// this only from the dispatch and the kernels themselves.

#include <ATen/core/Tensor.h>

namespace svllm::ops {

// q [num_tokens, num_heads, head_dim] and k [num_tokens, num_kv_heads, head_dim] views (heads
// and head_dim contiguous); q_weight / k_weight undefined for rope alone; inv_freq is a host
// array of head_dim / 2 floats.
namespace cpu_impl {
void rope(const at::Tensor& q, const at::Tensor& k, const at::Tensor& q_weight,
          const at::Tensor& k_weight, const at::Tensor& positions, double eps,
          const float* inv_freq);
}

namespace cuda_impl {
void rope(const at::Tensor& q, const at::Tensor& k, const at::Tensor& q_weight,
          const at::Tensor& k_weight, const at::Tensor& positions, double eps,
          const float* inv_freq);
}

}  // namespace svllm::ops

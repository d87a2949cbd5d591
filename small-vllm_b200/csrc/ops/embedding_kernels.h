#pragma once

// Per-device kernels behind ops::embedding; ids is flat [num_tokens], out [num_tokens, hidden].

#include <ATen/core/Tensor.h>

namespace svllm::ops {

namespace cpu_impl {
// Returns the number of ids outside [0, vocab); their rows are zero.
int64_t embedding(const at::Tensor& out, const at::Tensor& ids, const at::Tensor& table);
}

namespace cuda_impl {
void embedding(const at::Tensor& out, const at::Tensor& ids, const at::Tensor& table);
}

}  // namespace svllm::ops

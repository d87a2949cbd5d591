#pragma once

// Per-device kernels behind ops::silu_and_mul; gate, up and out are [rows, intermediate] views
// with contiguous rows.

#include <ATen/core/Tensor.h>

namespace svllm::ops {

namespace cpu_impl {
void silu_and_mul(const at::Tensor& out, const at::Tensor& gate, const at::Tensor& up);
}

namespace cuda_impl {
void silu_and_mul(const at::Tensor& out, const at::Tensor& gate, const at::Tensor& up);
}

}  // namespace svllm::ops

#pragma once

// Per-device kernels behind ops::argmax: logits [rows, vocab] with contiguous rows (any row
// stride), out int64 [rows].

#include <ATen/core/Tensor.h>

namespace svllm::ops {

namespace cpu_impl {
void argmax(const at::Tensor& out, const at::Tensor& logits);
}

namespace cuda_impl {
void argmax(const at::Tensor& out, const at::Tensor& logits);
}

}  // namespace svllm::ops

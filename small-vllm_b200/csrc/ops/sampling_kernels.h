#pragma once

// Per-device kernels behind ops::argmax (logits [rows, vocab] with contiguous rows, any row
// stride; out int64 [rows]) and ops::greedy_sample.

#include <ATen/core/Tensor.h>

namespace svllm::ops {

namespace cpu_impl {
void argmax(const at::Tensor& out, const at::Tensor& logits);
}

namespace cuda_impl {
void argmax(const at::Tensor& out, const at::Tensor& logits);
// The LM head fused with argmax (bf16, hidden [rows, H] and weight [vocab, H] with contiguous
// rows); false when the fused kernel does not take these operands (alignment), nothing run.
bool lm_head_argmax(const at::Tensor& out, const at::Tensor& hidden, const at::Tensor& weight);
}

}  // namespace svllm::ops

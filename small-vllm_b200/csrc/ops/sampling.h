#pragma once

#include <ATen/core/Tensor.h>

namespace svllm::ops {

// Definition: Greedy sampling, the index of the largest logit along the last dimension.
// Formula:    out[...] = argmax_j logits[..., j], the first index of the maximum; a NaN counts
//             as larger than any number (torch.argmax semantics).
// Domain:     logits [..., vocab] bf16 or fp32 with a contiguous last dimension (2-D inputs may
//             have any row stride), vocab > 0.
// Returns:    A new int64 tensor [...] on logits' device.
// Throws:     c10::Error on dtype or layout mismatches, or an unsupported device.
// The step after the final norm and the LM head (docs/design-spec.md:28-29, sampling on GPU).
at::Tensor argmax(const at::Tensor& logits);

// Definition: The model's last steps for greedy decoding with a tied (or any) LM head:
//             logits = hidden @ lm_head_weight^T, then argmax over the vocabulary. hidden is
//             the final norm's output. On CUDA (bf16) one fused tcgen05 kernel computes the
//             GEMM in fp32, rounds each logit to bf16 as a bf16 matmul stores it and takes the
//             argmax without storing the logits; it can differ from matmul-then-argmax only
//             where a logit tied for the maximum rounds differently under the two GEMMs'
//             accumulation orders. Elsewhere: torch::matmul, then argmax.
// Domain:     hidden [..., H] and lm_head_weight [vocab, H] (the embedding table when
//             tie_word_embeddings, src/model/config.h:28), same dtype and device.
// Returns:    int64 token ids [...].
at::Tensor greedy_sample(const at::Tensor& hidden, const at::Tensor& lm_head_weight);

}  // namespace svllm::ops

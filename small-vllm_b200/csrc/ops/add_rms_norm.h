#pragma once

#include <ATen/core/Tensor.h>

namespace svllm::ops {

// Definition: The residual add of a decoder layer fused with the RMSNorm that follows it, in
//             place, as Hugging Face's Qwen3 / Llama decoder layers compute it.
// Formula:    residual <- bf16(x + residual); x <- bf16(bf16(residual * rsqrt(mean(residual^2)
//             + eps)) * weight), the sum of squares in fp32.
// Domain:     x and residual [..., hidden], weight [hidden]; contiguous bf16 on one device.
// Returns:    Nothing; x holds the normalized rows and residual the updated residual stream.
// Throws:     c10::Error on dtype, shape, contiguity or device mismatches, or an unsupported
//             device.
// New op in the reference's op convention (planned at docs/design-spec.md:28).
void add_rms_norm(const at::Tensor& x, const at::Tensor& residual, const at::Tensor& weight,
                  double eps);

}  // namespace svllm::ops

#pragma once

#include <ATen/core/Tensor.h>

namespace svllm::ops {

// Definition: Root-mean-square normalization over the last dimension, scaled by a weight.
// Formula:    out = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * weight), the sum of squares in fp32.
// Domain:     x [..., hidden] and weight [hidden], contiguous bf16 on one device; hidden > 0.
// Returns:    A new bf16 tensor shaped like x, on x's device.
// Throws:     c10::Error if x or weight is not bf16, their shapes don't match, either is not
//             contiguous, they are on different devices, or x's device has no kernel.
// The signature and contract are the reference's (src/ops/rms_norm.h:7-13); on CUDA the work
// runs in the sm_100a kernel behind svllm_rms_norm_bf16.
at::Tensor rms_norm(const at::Tensor& x, const at::Tensor& weight, double eps);

}  // namespace svllm::ops

#pragma once

#include <ATen/core/Tensor.h>

namespace svllm::ops {

// Definition: The gated activation of a Qwen3 / Llama MLP, act_fn(gate) * up with act_fn = SiLU.
// Formula:    out = bf16(bf16(gate / (1 + exp(-gate))) * up), evaluated in fp32.
// Domain:     gate and up bf16 with equal shapes [..., intermediate] on one device; the last
//             dimension contiguous; 2-D inputs may have any row stride (so gate and up can be the
//             two halves of one [rows, 2 * intermediate] projection), higher ranks must be
//             contiguous.
// Returns:    A new contiguous bf16 tensor shaped like gate.
// Throws:     c10::Error on dtype, shape, layout or device mismatches, or an unsupported device.
// New op in the reference's op convention (docs/ROADMAP.md:40, "SiLU-and-mul").
at::Tensor silu_and_mul(const at::Tensor& gate, const at::Tensor& up);

// Definition: silu_and_mul on one concatenated gate_up projection, [..., 2 * intermediate] with
//             gate the first half and up the second (the fused-weight layout of
//             docs/ROADMAP.md:40, #48). No copy: the halves are passed as strided views.
// Returns:    A new contiguous bf16 tensor [..., intermediate].
// Throws:     As silu_and_mul, or if the last dimension is odd.
at::Tensor silu_and_mul(const at::Tensor& gate_up);

}  // namespace svllm::ops

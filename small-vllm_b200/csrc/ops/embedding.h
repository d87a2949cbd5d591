#pragma once

#include <ATen/core/Tensor.h>

namespace svllm::ops {

// Definition: The token-embedding gather at the bottom of the model.
// Formula:    out[..., :] = table[ids[...], :], a bit-exact row copy.
// Domain:     ids int32 (as the tokenizer returns them) or int64, any shape, contiguous;
//             table [vocab, hidden] bf16 with a contiguous last dimension; one device.
// Returns:    A new contiguous bf16 tensor [*ids.shape, hidden].
// Throws:     c10::Error on dtype, shape, layout or device mismatches, an unsupported device,
//             or (CPU only) ids outside [0, vocab). On CUDA an id outside [0, vocab) zeroes its
//             row and raises a bit in the device error word (read_device_error) without a host
//             sync, so the op stays graph-capturable.
// The table is model.embed_tokens.weight (reference tests/cpp/safetensors_test.cpp:161-162).
at::Tensor embedding(const at::Tensor& ids, const at::Tensor& table);

// Definition: Reads, and with reset clears, the device error word the kernels raise bits in
//             (1 = an embedding id out of range, 2 = a kernel's bulk copy timed out).
// Returns:    The word. Synchronises the device; for validation, not the hot path.
int64_t read_device_error(int64_t device_index, bool reset);

}  // namespace svllm::ops

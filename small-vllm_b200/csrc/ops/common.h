#pragma once

// Shared helpers of the op layer: the CUDA stream an op runs on and the C-ABI status check.

#include <ATen/core/Tensor.h>
#include <c10/util/Exception.h>

#include "svllm_kernels.h"

namespace svllm::ops::detail {

// Throws c10::Error naming the op when a C-ABI call returns an error status.
inline void check_status(const char* op, int status) {
  TORCH_CHECK(status == SVLLM_OK, op, ": ", svllm_status_string(status), " (status ", status, ")");
}

}  // namespace svllm::ops::detail

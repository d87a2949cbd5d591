// CUDA side of ops::argmax: a thin LibTorch -> C ABI shim.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "ops/common.h"
#include "ops/sampling_kernels.h"

namespace svllm::ops::cuda_impl {

void argmax(const at::Tensor& out, const at::Tensor& logits) {
  if (logits.size(0) == 0) {
    return;
  }
  const c10::cuda::CUDAGuard device_guard(logits.device());
  const auto stream = reinterpret_cast<svllm_stream>(c10::cuda::getCurrentCUDAStream().stream());
  auto* ids = out.mutable_data_ptr<int64_t>();
  const int status =
      logits.scalar_type() == at::kBFloat16
          ? svllm_argmax_bf16(logits.const_data_ptr(), logits.size(0), logits.size(1),
                              logits.stride(0), ids, stream)
          : svllm_argmax_f32(logits.const_data_ptr<float>(), logits.size(0), logits.size(1),
                             logits.stride(0), ids, stream);
  detail::check_status("argmax", status);
}

}  // namespace svllm::ops::cuda_impl

// CUDA side of ops::argmax and ops::greedy_sample: thin LibTorch -> C ABI shims.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <ATen/ATen.h>

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

bool lm_head_argmax(const at::Tensor& out, const at::Tensor& hidden, const at::Tensor& weight) {
  const c10::cuda::CUDAGuard device_guard(hidden.device());
  const auto stream = reinterpret_cast<svllm_stream>(c10::cuda::getCurrentCUDAStream().stream());
  // zeroed per call, so calls on different streams never share one
  const at::Tensor workspace = at::zeros({hidden.size(0)}, hidden.options().dtype(at::kLong));
  const int status = svllm_lm_head_argmax_bf16(
      hidden.const_data_ptr(), hidden.size(0), hidden.size(1), hidden.stride(0),
      weight.const_data_ptr(), weight.size(0), weight.stride(0), out.mutable_data_ptr<int64_t>(),
      nullptr, 0, workspace.mutable_data_ptr(), workspace.numel() * 8, stream);
  if (status == SVLLM_ERR_UNSUPPORTED) return false;
  detail::check_status("greedy_sample", status);
  return true;
}

}  // namespace svllm::ops::cuda_impl

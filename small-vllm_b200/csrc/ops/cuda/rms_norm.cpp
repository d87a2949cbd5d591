// CUDA side of ops::rms_norm and ops::add_rms_norm: a thin LibTorch -> C ABI shim. The kernels
// are the sm_100a bulk-copy pipelines in libsvllm_kernels.so; nothing here computes.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "ops/common.h"
#include "ops/rms_norm_kernels.h"

namespace svllm::ops::cuda_impl {

void rms_norm(const at::Tensor& out, const at::Tensor& x, const at::Tensor& weight, double eps) {
  const int64_t hidden = x.size(-1);
  const int64_t num_rows = x.numel() / hidden;
  if (num_rows == 0) {
    return;
  }
  const c10::cuda::CUDAGuard device_guard(x.device());
  const auto stream = reinterpret_cast<svllm_stream>(c10::cuda::getCurrentCUDAStream().stream());
  detail::check_status("rms_norm",
                       svllm_rms_norm_bf16(out.mutable_data_ptr(), x.const_data_ptr(),
                                           weight.const_data_ptr(), num_rows, hidden, hidden,
                                           hidden, static_cast<float>(eps), stream));
}

void add_rms_norm(const at::Tensor& x, const at::Tensor& residual, const at::Tensor& weight,
                  double eps) {
  const int64_t hidden = x.size(-1);
  const int64_t num_rows = x.numel() / hidden;
  if (num_rows == 0) {
    return;
  }
  const c10::cuda::CUDAGuard device_guard(x.device());
  const auto stream = reinterpret_cast<svllm_stream>(c10::cuda::getCurrentCUDAStream().stream());
  detail::check_status("add_rms_norm",
                       svllm_add_rms_norm_bf16(x.mutable_data_ptr(), residual.mutable_data_ptr(),
                                               weight.const_data_ptr(), num_rows, hidden, hidden,
                                               hidden, static_cast<float>(eps), stream));
}

}  // namespace svllm::ops::cuda_impl

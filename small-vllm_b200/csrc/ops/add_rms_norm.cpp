#include "ops/add_rms_norm.h"

#include <c10/util/Exception.h>

#include "ops/rms_norm_kernels.h"

namespace svllm::ops {

void add_rms_norm(const at::Tensor& x, const at::Tensor& residual, const at::Tensor& weight,
                  double eps) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && residual.scalar_type() == at::kBFloat16 &&
                  weight.scalar_type() == at::kBFloat16,
              "add_rms_norm: expected bf16 x, residual and weight, got ", x.scalar_type(), ", ",
              residual.scalar_type(), " and ", weight.scalar_type());
  TORCH_CHECK(x.dim() >= 1 && x.sizes() == residual.sizes() && weight.dim() == 1 &&
                  weight.size(0) > 0 && x.size(-1) == weight.size(0),
              "add_rms_norm: x of shape ", x.sizes(), ", residual of shape ", residual.sizes(),
              " and weight of shape ", weight.sizes(), " do not match");
  TORCH_CHECK(x.is_contiguous() && residual.is_contiguous() && weight.is_contiguous(),
              "add_rms_norm: x, residual and weight must be contiguous");
  TORCH_CHECK(x.device() == residual.device() && x.device() == weight.device(),
              "add_rms_norm: x is on ", x.device(), " but residual is on ", residual.device(),
              " and weight is on ", weight.device());

  switch (x.device().type()) {
    case c10::DeviceType::CPU:
      cpu_impl::add_rms_norm(x, residual, weight, eps);
      break;
    case c10::DeviceType::CUDA:
      cuda_impl::add_rms_norm(x, residual, weight, eps);
      break;
    default:
      TORCH_CHECK(false, "add_rms_norm: unsupported device ", x.device());
  }
}

}  // namespace svllm::ops

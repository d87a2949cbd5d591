#include "ops/sampling.h"

#include <ATen/ATen.h>
#include <c10/util/Exception.h>

#include <vector>

#include "ops/sampling_kernels.h"

namespace svllm::ops {

at::Tensor argmax(const at::Tensor& logits) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 || logits.scalar_type() == at::kFloat,
              "argmax: expected bf16 or fp32 logits, got ", logits.scalar_type());
  TORCH_CHECK(logits.dim() >= 1 && logits.size(-1) > 0, "argmax: logits of shape ",
              logits.sizes(), " have no vocabulary dimension");
  TORCH_CHECK(logits.stride(-1) == 1 && (logits.dim() <= 2 || logits.is_contiguous()),
              "argmax: logits must have a contiguous last dimension (and be contiguous beyond "
              "two dimensions)");

  const std::vector<int64_t> shape(logits.sizes().begin(), logits.sizes().end() - 1);
  at::Tensor out = at::empty(shape, logits.options().dtype(at::kLong));
  const at::Tensor rows = logits.dim() == 1   ? logits.unsqueeze(0)
                          : logits.dim() == 2 ? logits
                                              : logits.view({-1, logits.size(-1)});
  const at::Tensor flat_out = out.view({-1});
  switch (logits.device().type()) {
    case c10::DeviceType::CPU:
      cpu_impl::argmax(flat_out, rows);
      break;
    case c10::DeviceType::CUDA:
      cuda_impl::argmax(flat_out, rows);
      break;
    default:
      TORCH_CHECK(false, "argmax: unsupported device ", logits.device());
  }
  return out;
}

at::Tensor greedy_sample(const at::Tensor& hidden, const at::Tensor& lm_head_weight) {
  TORCH_CHECK(lm_head_weight.dim() == 2 && hidden.dim() >= 1 &&
                  hidden.size(-1) == lm_head_weight.size(1),
              "greedy_sample: hidden of shape ", hidden.sizes(),
              " does not match lm_head_weight of shape ", lm_head_weight.sizes());
  TORCH_CHECK(hidden.scalar_type() == lm_head_weight.scalar_type() &&
                  hidden.device() == lm_head_weight.device(),
              "greedy_sample: hidden and lm_head_weight must share dtype and device");
  if (hidden.is_cuda() && hidden.scalar_type() == at::kBFloat16 && hidden.numel() > 0 &&
      hidden.stride(-1) == 1 && lm_head_weight.stride(1) == 1 &&
      (hidden.dim() <= 2 || hidden.is_contiguous())) {
    // the LM-head GEMM and the argmax in one pass, the logits never stored
    const at::Tensor rows = hidden.dim() == 1 ? hidden.unsqueeze(0)
                            : hidden.dim() == 2 ? hidden
                                                : hidden.view({-1, hidden.size(-1)});
    const std::vector<int64_t> shape(hidden.sizes().begin(), hidden.sizes().end() - 1);
    at::Tensor out = at::empty(shape, hidden.options().dtype(at::kLong));
    if (cuda_impl::lm_head_argmax(out.view({-1}), rows, lm_head_weight)) return out;
  }
  return svllm::ops::argmax(at::matmul(hidden, lm_head_weight.t()));
}

}  // namespace svllm::ops

// CUDA side of ops::rope and ops::qk_norm_rope: a thin LibTorch -> C ABI shim.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "ops/common.h"
#include "ops/rope_kernels.h"

namespace svllm::ops::cuda_impl {

void rope(const at::Tensor& q, const at::Tensor& k, const at::Tensor& q_weight,
          const at::Tensor& k_weight, const at::Tensor& positions, double eps,
          const float* inv_freq) {
  const int64_t num_tokens = q.size(0);
  if (num_tokens == 0) {
    return;
  }
  const c10::cuda::CUDAGuard device_guard(q.device());
  const auto stream = reinterpret_cast<svllm_stream>(c10::cuda::getCurrentCUDAStream().stream());
  const int pos_type = positions.scalar_type() == at::kLong ? SVLLM_INDEX_I64 : SVLLM_INDEX_I32;
  if (q_weight.defined()) {
    detail::check_status(
        "qk_norm_rope",
        svllm_qk_norm_rope_bf16(q.mutable_data_ptr(), k.mutable_data_ptr(),
                                q_weight.const_data_ptr(), k_weight.const_data_ptr(),
                                positions.const_data_ptr(), pos_type, num_tokens, q.size(1),
                                k.size(1), q.size(2), q.stride(0), k.stride(0),
                                static_cast<float>(eps), inv_freq, stream));
  } else {
    detail::check_status(
        "rope", svllm_rope_bf16(q.mutable_data_ptr(), k.mutable_data_ptr(),
                                positions.const_data_ptr(), pos_type, num_tokens, q.size(1),
                                k.size(1), q.size(2), q.stride(0), k.stride(0), inv_freq, stream));
  }
}

void rope_cache(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                const at::Tensor& q_weight, const at::Tensor& k_weight,
                const at::Tensor& positions, const at::Tensor& slot_mapping,
                const at::Tensor& k_cache, const at::Tensor& v_cache, double eps,
                const float* inv_freq) {
  const int64_t num_tokens = q.size(0);
  if (num_tokens == 0) {
    return;
  }
  const c10::cuda::CUDAGuard device_guard(q.device());
  const auto stream = reinterpret_cast<svllm_stream>(c10::cuda::getCurrentCUDAStream().stream());
  const int pos_type = positions.scalar_type() == at::kLong ? SVLLM_INDEX_I64 : SVLLM_INDEX_I32;
  const auto* slots = slot_mapping.const_data_ptr<int64_t>();
  if (q_weight.defined()) {
    detail::check_status(
        "qk_norm_rope_cache",
        svllm_qk_norm_rope_cache_bf16(
            q.mutable_data_ptr(), k.mutable_data_ptr(), v.const_data_ptr(),
            q_weight.const_data_ptr(), k_weight.const_data_ptr(), positions.const_data_ptr(),
            pos_type, slots, k_cache.mutable_data_ptr(), v_cache.mutable_data_ptr(),
            k_cache.size(0), num_tokens, q.size(1), k.size(1), q.size(2), q.stride(0),
            k.stride(0), v.stride(0), static_cast<float>(eps), inv_freq, stream));
  } else {
    detail::check_status(
        "rope_cache",
        svllm_rope_cache_bf16(q.mutable_data_ptr(), k.mutable_data_ptr(), v.const_data_ptr(),
                              positions.const_data_ptr(), pos_type, slots,
                              k_cache.mutable_data_ptr(), v_cache.mutable_data_ptr(),
                              k_cache.size(0), num_tokens, q.size(1), k.size(1), q.size(2),
                              q.stride(0), k.stride(0), v.stride(0), inv_freq, stream));
  }
}

}  // namespace svllm::ops::cuda_impl

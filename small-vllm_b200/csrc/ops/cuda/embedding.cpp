// CUDA side of ops::embedding: a thin LibTorch -> C ABI shim.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "ops/common.h"
#include "ops/embedding_kernels.h"

namespace svllm::ops::cuda_impl {

void embedding(const at::Tensor& out, const at::Tensor& ids, const at::Tensor& table) {
  const c10::cuda::CUDAGuard device_guard(ids.device());
  const auto stream = reinterpret_cast<svllm_stream>(c10::cuda::getCurrentCUDAStream().stream());
  const int id_type = ids.scalar_type() == at::kLong ? SVLLM_INDEX_I64 : SVLLM_INDEX_I32;
  detail::check_status(
      "embedding",
      svllm_embedding_bf16(out.mutable_data_ptr(), ids.const_data_ptr(), id_type,
                           table.const_data_ptr(), ids.numel(), table.size(0), table.size(1),
                           out.stride(0), table.stride(0), nullptr, stream));
}

}  // namespace svllm::ops::cuda_impl

// CUDA side of ops::silu_and_mul: a thin LibTorch -> C ABI shim.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "ops/common.h"
#include "ops/silu_and_mul_kernels.h"

namespace svllm::ops::cuda_impl {

void silu_and_mul(const at::Tensor& out, const at::Tensor& gate, const at::Tensor& up) {
  const c10::cuda::CUDAGuard device_guard(gate.device());
  const auto stream = reinterpret_cast<svllm_stream>(c10::cuda::getCurrentCUDAStream().stream());
  detail::check_status(
      "silu_and_mul",
      svllm_silu_and_mul_bf16(out.mutable_data_ptr(), gate.const_data_ptr(), up.const_data_ptr(),
                              gate.size(0), gate.size(1), out.stride(0), gate.stride(0),
                              up.stride(0), stream));
}

}  // namespace svllm::ops::cuda_impl

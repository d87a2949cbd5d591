#pragma once

// Per-device kernels behind ops::rms_norm and ops::add_rms_norm, which validate the inputs (and
// allocate out); include this only from the dispatch and the kernels themselves.

#include <ATen/core/Tensor.h>

namespace svllm::ops {

// Definition: The OpenMP kernels, writing into out (rms_norm) or in place (add_rms_norm).
// Domain:     Inputs already validated by the op; contiguous bf16.
namespace cpu_impl {
void rms_norm(const at::Tensor& out, const at::Tensor& x, const at::Tensor& weight, double eps);
void add_rms_norm(const at::Tensor& x, const at::Tensor& residual, const at::Tensor& weight,
                  double eps);
}  // namespace cpu_impl

// Definition: The CUDA kernels, enqueued on the current stream through the C ABI.
// Throws:     c10::Error if the C ABI reports an error (bad size, launch failure).
namespace cuda_impl {
void rms_norm(const at::Tensor& out, const at::Tensor& x, const at::Tensor& weight, double eps);
void add_rms_norm(const at::Tensor& x, const at::Tensor& residual, const at::Tensor& weight,
                  double eps);
}  // namespace cuda_impl

}  // namespace svllm::ops

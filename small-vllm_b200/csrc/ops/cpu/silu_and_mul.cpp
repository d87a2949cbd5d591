// OpenMP kernel of ops::silu_and_mul for CPU tensors, on torch's thread pool.
#include <ATen/Parallel.h>
#include <c10/util/BFloat16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "ops/silu_and_mul_kernels.h"

namespace svllm::ops::cpu_impl {

// Elements per parallel_for chunk, so a decode step's few rows run inline without a fork.
constexpr int64_t kGrainElems = 32768;

void silu_and_mul(const at::Tensor& out, const at::Tensor& gate, const at::Tensor& up) {
  const int64_t rows = gate.size(0);
  const int64_t inter = gate.size(1);
  const auto* gp = gate.const_data_ptr<at::BFloat16>();
  const auto* up_p = up.const_data_ptr<at::BFloat16>();
  auto* op = out.mutable_data_ptr<at::BFloat16>();
  const int64_t gs = gate.stride(0);
  const int64_t us = up.stride(0);
  const int64_t os = out.stride(0);
  const int64_t grain = std::max<int64_t>(1, kGrainElems / inter);
  at::parallel_for(0, rows, grain, [&](int64_t begin, int64_t end) {
    for (int64_t r = begin; r < end; ++r) {
      for (int64_t i = 0; i < inter; ++i) {
        const float g = static_cast<float>(gp[r * gs + i]);
        const at::BFloat16 act = g / (1.0f + std::exp(-g));
        op[r * os + i] = static_cast<float>(act) * static_cast<float>(up_p[r * us + i]);
      }
    }
  });
}

}  // namespace svllm::ops::cpu_impl

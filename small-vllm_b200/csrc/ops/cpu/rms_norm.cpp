// OpenMP kernels of ops::rms_norm and ops::add_rms_norm for CPU tensors, on torch's thread pool.
#include <ATen/Parallel.h>
#include <c10/util/BFloat16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

#include "ops/rms_norm_kernels.h"

namespace svllm::ops::cpu_impl {

// Elements per parallel_for chunk, so a decode step's few rows run inline without a fork.
constexpr int64_t kGrainElems = 32768;
namespace {

// Normalises one row of n values already in `row` (fp32 copies of bf16) into out.
void normalize_row(at::BFloat16* out, const float* row, const at::BFloat16* weight, int64_t n,
                   float eps) {
  float sum_sq = 0.0f;
#pragma omp simd reduction(+ : sum_sq)
  for (int64_t i = 0; i < n; ++i) sum_sq += row[i] * row[i];
  const float inv_rms = 1.0f / std::sqrt(sum_sq / static_cast<float>(n) + eps);
  for (int64_t i = 0; i < n; ++i) {
    // bf16 rounding of the normalised value before the weight, as Hugging Face does
    const float normed = static_cast<float>(static_cast<at::BFloat16>(row[i] * inv_rms));
    out[i] = static_cast<at::BFloat16>(normed * static_cast<float>(weight[i]));
  }
}

template <class RowFn>
void for_rows(int64_t num_rows, int64_t hidden, const RowFn& fn) {
  const int64_t grain = std::max<int64_t>(1, kGrainElems / hidden);
  at::parallel_for(0, num_rows, grain, [&](int64_t begin, int64_t end) {
    std::vector<float> row(static_cast<size_t>(hidden));
    for (int64_t r = begin; r < end; ++r) fn(r, row.data());
  });
}

}  // namespace

void rms_norm(const at::Tensor& out, const at::Tensor& x, const at::Tensor& weight, double eps) {
  const int64_t hidden = x.size(-1);
  const int64_t num_rows = x.numel() / hidden;
  const auto* xp = x.const_data_ptr<at::BFloat16>();
  const auto* wp = weight.const_data_ptr<at::BFloat16>();
  auto* op = out.mutable_data_ptr<at::BFloat16>();
  const float eps_f = static_cast<float>(eps);
  for_rows(num_rows, hidden, [&](int64_t r, float* row) {
    const at::BFloat16* xr = xp + r * hidden;
    for (int64_t i = 0; i < hidden; ++i) row[i] = static_cast<float>(xr[i]);
    normalize_row(op + r * hidden, row, wp, hidden, eps_f);
  });
}

void add_rms_norm(const at::Tensor& x, const at::Tensor& residual, const at::Tensor& weight,
                  double eps) {
  const int64_t hidden = x.size(-1);
  const int64_t num_rows = x.numel() / hidden;
  auto* xp = x.mutable_data_ptr<at::BFloat16>();
  auto* rp = residual.mutable_data_ptr<at::BFloat16>();
  const auto* wp = weight.const_data_ptr<at::BFloat16>();
  const float eps_f = static_cast<float>(eps);
  for_rows(num_rows, hidden, [&](int64_t r, float* row) {
    at::BFloat16* xr = xp + r * hidden;
    at::BFloat16* rr = rp + r * hidden;
    for (int64_t i = 0; i < hidden; ++i) {
      const at::BFloat16 sum = static_cast<float>(xr[i]) + static_cast<float>(rr[i]);
      rr[i] = sum;
      row[i] = static_cast<float>(sum);
    }
    normalize_row(xr, row, wp, hidden, eps_f);
  });
}

}  // namespace svllm::ops::cpu_impl

// OpenMP kernel of ops::argmax for CPU tensors, on torch's thread pool.
#include <ATen/Parallel.h>
#include <c10/util/BFloat16.h>

#include <cmath>
#include <cstdint>

#include "ops/sampling_kernels.h"

namespace svllm::ops::cpu_impl {
namespace {

template <class T>
void argmax_rows(int64_t* out, const T* x, int64_t rows, int64_t vocab, int64_t stride) {
  at::parallel_for(0, rows, 1, [&](int64_t begin, int64_t end) {
    for (int64_t r = begin; r < end; ++r) {
      const T* row = x + r * stride;
      int64_t best = 0;
      float best_v = static_cast<float>(row[0]);
      for (int64_t j = 1; j < vocab && !std::isnan(best_v); ++j) {
        const float v = static_cast<float>(row[j]);
        if (std::isnan(v) || v > best_v) {  // the first NaN, else the first maximum
          best = j;
          best_v = v;
        }
      }
      out[r] = best;
    }
  });
}

}  // namespace

void argmax(const at::Tensor& out, const at::Tensor& logits) {
  auto* o = out.mutable_data_ptr<int64_t>();
  if (logits.scalar_type() == at::kBFloat16) {
    argmax_rows(o, logits.const_data_ptr<at::BFloat16>(), logits.size(0), logits.size(1),
                logits.stride(0));
  } else {
    argmax_rows(o, logits.const_data_ptr<float>(), logits.size(0), logits.size(1),
                logits.stride(0));
  }
}

}  // namespace svllm::ops::cpu_impl

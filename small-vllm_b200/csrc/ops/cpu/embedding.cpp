// Kernel of ops::embedding for CPU tensors: row copies on torch's thread pool.
#include <ATen/Parallel.h>

#include <atomic>
#include <cstdint>
#include <cstring>

#include "ops/embedding_kernels.h"

namespace svllm::ops::cpu_impl {

int64_t embedding(const at::Tensor& out, const at::Tensor& ids, const at::Tensor& table) {
  const int64_t num_tokens = ids.numel();
  const int64_t vocab = table.size(0);
  const int64_t row_bytes = table.size(1) * static_cast<int64_t>(table.element_size());
  const int64_t table_stride = table.stride(0) * static_cast<int64_t>(table.element_size());
  const bool ids64 = ids.scalar_type() == at::kLong;
  const void* id_p = ids.const_data_ptr();
  const auto* tp = static_cast<const char*>(table.const_data_ptr());
  auto* op = static_cast<char*>(out.mutable_data_ptr());
  std::atomic<int64_t> bad{0};
  at::parallel_for(0, num_tokens, 64, [&](int64_t begin, int64_t end) {
    int64_t local_bad = 0;
    for (int64_t t = begin; t < end; ++t) {
      const int64_t id = ids64 ? static_cast<const int64_t*>(id_p)[t]
                               : static_cast<int64_t>(static_cast<const int32_t*>(id_p)[t]);
      if (id < 0 || id >= vocab) {
        std::memset(op + t * row_bytes, 0, static_cast<size_t>(row_bytes));
        ++local_bad;
      } else {
        std::memcpy(op + t * row_bytes, tp + id * table_stride, static_cast<size_t>(row_bytes));
      }
    }
    bad += local_bad;
  });
  return bad.load();
}

}  // namespace svllm::ops::cpu_impl

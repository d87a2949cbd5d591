#include "ops/embedding.h"

#include <ATen/Functions.h>
#include <c10/util/Exception.h>

#include <vector>

#include "ops/common.h"
#include "ops/embedding_kernels.h"

namespace svllm::ops {

at::Tensor embedding(const at::Tensor& ids, const at::Tensor& table) {
  TORCH_CHECK(ids.scalar_type() == at::kInt || ids.scalar_type() == at::kLong,
              "embedding: expected int32 or int64 ids, got ", ids.scalar_type());
  TORCH_CHECK(table.scalar_type() == at::kBFloat16, "embedding: expected a bf16 table, got ",
              table.scalar_type());
  TORCH_CHECK(table.dim() == 2 && table.size(0) > 0 && table.size(1) > 0,
              "embedding: table must be [vocab, hidden], got shape ", table.sizes());
  TORCH_CHECK(ids.is_contiguous() && table.stride(1) == 1,
              "embedding: ids must be contiguous and table rows contiguous");
  TORCH_CHECK(ids.device() == table.device(), "embedding: ids are on ", ids.device(),
              " but table is on ", table.device());

  std::vector<int64_t> out_shape(ids.sizes().begin(), ids.sizes().end());
  out_shape.push_back(table.size(1));
  at::Tensor out = at::empty(out_shape, table.options().memory_format(at::MemoryFormat::Contiguous));
  const at::Tensor flat_ids = ids.reshape({-1});
  const at::Tensor flat_out = out.view({-1, table.size(1)});

  switch (ids.device().type()) {
    case c10::DeviceType::CPU: {
      const int64_t bad = flat_ids.numel() ? cpu_impl::embedding(flat_out, flat_ids, table) : 0;
      TORCH_CHECK(bad == 0, "embedding: ", bad, " ids outside [0, ", table.size(0), ")");
      break;
    }
    case c10::DeviceType::CUDA:
      if (flat_ids.numel()) cuda_impl::embedding(flat_out, flat_ids, table);
      break;
    default:
      TORCH_CHECK(false, "embedding: unsupported device ", ids.device());
  }
  return out;
}

int64_t read_device_error(int64_t device_index, bool reset) {
  int flags = 0;
  detail::check_status("read_device_error",
                       svllm_read_device_error(static_cast<int>(device_index), reset ? 1 : 0, &flags));
  return flags;
}

}  // namespace svllm::ops

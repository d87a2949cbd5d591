#include "ops/silu_and_mul.h"

#include <ATen/Functions.h>
#include <c10/util/Exception.h>

#include <vector>

#include "ops/silu_and_mul_kernels.h"

namespace svllm::ops {
namespace {

// A [rows, intermediate] view with contiguous rows, without copying.
at::Tensor rows_view(const at::Tensor& t) {
  if (t.dim() == 2) {
    return t;
  }
  if (t.dim() == 1) {
    return t.unsqueeze(0);
  }
  return t.view({-1, t.size(-1)});
}

}  // namespace

at::Tensor silu_and_mul(const at::Tensor& gate, const at::Tensor& up) {
  TORCH_CHECK(gate.scalar_type() == at::kBFloat16 && up.scalar_type() == at::kBFloat16,
              "silu_and_mul: expected bf16 gate and up, got ", gate.scalar_type(), " and ",
              up.scalar_type());
  TORCH_CHECK(gate.dim() >= 1 && gate.sizes() == up.sizes() && gate.size(-1) > 0,
              "silu_and_mul: gate of shape ", gate.sizes(), " does not match up of shape ",
              up.sizes());
  TORCH_CHECK(gate.stride(-1) == 1 && up.stride(-1) == 1 &&
                  (gate.dim() <= 2 || (gate.is_contiguous() && up.is_contiguous())),
              "silu_and_mul: gate and up must have a contiguous last dimension (and be contiguous "
              "beyond two dimensions)");
  TORCH_CHECK(gate.device() == up.device(), "silu_and_mul: gate is on ", gate.device(),
              " but up is on ", up.device());

  at::Tensor out = at::empty(gate.sizes(), gate.options().memory_format(at::MemoryFormat::Contiguous));
  if (out.numel() == 0) {
    TORCH_CHECK(gate.device().type() == c10::DeviceType::CPU ||
                    gate.device().type() == c10::DeviceType::CUDA,
                "silu_and_mul: unsupported device ", gate.device());
    return out;
  }

  switch (gate.device().type()) {
    case c10::DeviceType::CPU:
      cpu_impl::silu_and_mul(rows_view(out), rows_view(gate), rows_view(up));
      break;
    case c10::DeviceType::CUDA:
      cuda_impl::silu_and_mul(rows_view(out), rows_view(gate), rows_view(up));
      break;
    default:
      TORCH_CHECK(false, "silu_and_mul: unsupported device ", gate.device());
  }
  return out;
}

at::Tensor silu_and_mul(const at::Tensor& gate_up) {
  TORCH_CHECK(gate_up.dim() >= 1 && gate_up.size(-1) % 2 == 0,
              "silu_and_mul: gate_up must have an even last dimension, got shape ",
              gate_up.sizes());
  TORCH_CHECK(gate_up.dim() <= 2 || gate_up.is_contiguous(),
              "silu_and_mul: gate_up must be contiguous beyond two dimensions");
  const at::Tensor rows = gate_up.dim() == 1 ? gate_up.unsqueeze(0)
                          : gate_up.dim() == 2 ? gate_up
                                               : gate_up.view({-1, gate_up.size(-1)});
  const int64_t inter = rows.size(1) / 2;
  at::Tensor out = silu_and_mul(rows.narrow(1, 0, inter), rows.narrow(1, inter, inter));
  std::vector<int64_t> shape(gate_up.sizes().begin(), gate_up.sizes().end());
  shape.back() = inter;
  return out.view(shape);
}

}  // namespace svllm::ops

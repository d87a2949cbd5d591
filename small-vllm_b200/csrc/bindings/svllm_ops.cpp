// pybind11 module svllm_ops: the reference's binding (bindings/svllm_ops.cpp:11-29) with its
// attributes and rms_norm signature unchanged, plus the five fused layer ops added in the same
// style. The reference's Tokenizer class sits outside the layer-op path and is not bound here.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include <optional>

#include "model/config.h"
#include "ops/add_rms_norm.h"
#include "ops/embedding.h"
#include "ops/rms_norm.h"
#include "ops/rope.h"
#include "ops/sampling.h"
#include "ops/silu_and_mul.h"

namespace py = pybind11;

PYBIND11_MODULE(svllm_ops, m) {
  m.attr("__version__") = SVLLM_VERSION;
#ifdef SVLLM_CUDA
  m.attr("built_with_cuda") = true;
#else
  m.attr("built_with_cuda") = false;
#endif

  py::class_<svllm::Llama3RopeScaling>(m, "Llama3RopeScaling")
      .def(py::init([](double factor, double low_freq_factor, double high_freq_factor,
                       int64_t original_max_position_embeddings) {
             return svllm::Llama3RopeScaling{factor, low_freq_factor, high_freq_factor,
                                             original_max_position_embeddings};
           }),
           py::arg("factor"), py::arg("low_freq_factor"), py::arg("high_freq_factor"),
           py::arg("original_max_position_embeddings"))
      .def_readwrite("factor", &svllm::Llama3RopeScaling::factor)
      .def_readwrite("low_freq_factor", &svllm::Llama3RopeScaling::low_freq_factor)
      .def_readwrite("high_freq_factor", &svllm::Llama3RopeScaling::high_freq_factor)
      .def_readwrite("original_max_position_embeddings",
                     &svllm::Llama3RopeScaling::original_max_position_embeddings);

  m.def("rms_norm", &svllm::ops::rms_norm, py::arg("x"), py::arg("weight"), py::arg("eps"));
  m.def("add_rms_norm", &svllm::ops::add_rms_norm, py::arg("x"), py::arg("residual"),
        py::arg("weight"), py::arg("eps"));
  m.def("qk_norm_rope", &svllm::ops::qk_norm_rope, py::arg("q"), py::arg("k"),
        py::arg("q_weight"), py::arg("k_weight"), py::arg("positions"), py::arg("eps"),
        py::arg("theta"), py::arg("rope_scaling") = std::nullopt);
  m.def("rope", &svllm::ops::rope, py::arg("q"), py::arg("k"), py::arg("positions"),
        py::arg("theta"), py::arg("rope_scaling") = std::nullopt);
  m.def("qk_norm_rope_cache", &svllm::ops::qk_norm_rope_cache, py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("q_weight"), py::arg("k_weight"), py::arg("positions"),
        py::arg("slot_mapping"), py::arg("k_cache"), py::arg("v_cache"), py::arg("eps"),
        py::arg("theta"), py::arg("rope_scaling") = std::nullopt);
  m.def("rope_cache", &svllm::ops::rope_cache, py::arg("q"), py::arg("k"), py::arg("v"),
        py::arg("positions"), py::arg("slot_mapping"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("theta"), py::arg("rope_scaling") = std::nullopt);
  m.def("rope_inv_freq", &svllm::ops::rope_inv_freq, py::arg("theta"), py::arg("head_dim"),
        py::arg("rope_scaling") = std::nullopt);
  m.def("silu_and_mul",
        py::overload_cast<const at::Tensor&, const at::Tensor&>(&svllm::ops::silu_and_mul),
        py::arg("gate"), py::arg("up"));
  m.def("silu_and_mul", py::overload_cast<const at::Tensor&>(&svllm::ops::silu_and_mul),
        py::arg("gate_up"));
  m.def("embedding", &svllm::ops::embedding, py::arg("ids"), py::arg("table"));
  m.def("argmax", &svllm::ops::argmax, py::arg("logits"));
  m.def("greedy_sample", &svllm::ops::greedy_sample, py::arg("hidden"),
        py::arg("lm_head_weight"));
  m.def("read_device_error", &svllm::ops::read_device_error, py::arg("device_index"),
        py::arg("reset") = true);
}

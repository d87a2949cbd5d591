// pybind11 module svllm_ops: the reference's binding (bindings/svllm_ops.cpp:11-29) with its
// attributes and rms_norm signature unchanged, plus the fused layer ops added in the same style,
// and the model forward that calls them (ModelConfig, Model, DecodeGraphs). The reference's
// Tokenizer class sits outside the layer-op path and is not bound here.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include <optional>

#include "model/config.h"
#include "model/qwen3.h"
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

  using svllm::ModelConfig;
  py::class_<ModelConfig>(m, "ModelConfig")
      .def(py::init([](int64_t vocab_size, int64_t hidden_size, int64_t intermediate_size,
                       int64_t num_layers, int64_t num_heads, int64_t num_kv_heads,
                       int64_t head_dim, double rms_norm_eps, double rope_theta,
                       bool tie_word_embeddings, bool qk_norm,
                       std::optional<svllm::Llama3RopeScaling> rope_scaling) {
             return ModelConfig{vocab_size,   hidden_size,  intermediate_size, num_layers,
                                num_heads,    num_kv_heads, head_dim,          rms_norm_eps,
                                rope_theta,   tie_word_embeddings, qk_norm,    rope_scaling};
           }),
           py::arg("vocab_size"), py::arg("hidden_size"), py::arg("intermediate_size"),
           py::arg("num_layers"), py::arg("num_heads"), py::arg("num_kv_heads"),
           py::arg("head_dim"), py::arg("rms_norm_eps"), py::arg("rope_theta"),
           py::arg("tie_word_embeddings"), py::arg("qk_norm"),
           py::arg("rope_scaling") = std::nullopt)
      .def_readwrite("vocab_size", &ModelConfig::vocab_size)
      .def_readwrite("hidden_size", &ModelConfig::hidden_size)
      .def_readwrite("intermediate_size", &ModelConfig::intermediate_size)
      .def_readwrite("num_layers", &ModelConfig::num_layers)
      .def_readwrite("num_heads", &ModelConfig::num_heads)
      .def_readwrite("num_kv_heads", &ModelConfig::num_kv_heads)
      .def_readwrite("head_dim", &ModelConfig::head_dim)
      .def_readwrite("rms_norm_eps", &ModelConfig::rms_norm_eps)
      .def_readwrite("rope_theta", &ModelConfig::rope_theta)
      .def_readwrite("tie_word_embeddings", &ModelConfig::tie_word_embeddings)
      .def_readwrite("qk_norm", &ModelConfig::qk_norm)
      .def_readwrite("rope_scaling", &ModelConfig::rope_scaling);

  using svllm::model::Model;
  py::class_<Model, std::shared_ptr<Model>>(m, "Model")
      .def(py::init<const ModelConfig&, const std::unordered_map<std::string, at::Tensor>&>(),
           py::arg("config"), py::arg("weights"))
      .def("allocate_kv_cache", &Model::allocate_kv_cache, py::arg("num_blocks"),
           py::arg("block_size"))
      .def(
          "forward",
          [](Model& self, const at::Tensor& ids, const at::Tensor& positions,
             const at::Tensor& slot_mapping, const at::Tensor& block_tables,
             const at::Tensor& seq_lens, const at::Tensor& query_start_loc) {
            return self.forward(ids, positions,
                                {slot_mapping, block_tables, seq_lens, query_start_loc});
          },
          py::arg("ids"), py::arg("positions"), py::arg("slot_mapping"), py::arg("block_tables"),
          py::arg("seq_lens"), py::arg("query_start_loc"))
      .def("logits", &Model::logits, py::arg("hidden"))
      .def("greedy", &Model::greedy, py::arg("hidden"))
      .def("decode", &Model::decode, py::arg("ids"), py::arg("positions"),
           py::arg("slot_mapping"), py::arg("block_tables"), py::arg("seq_lens"))
      .def_property_readonly("config", &Model::config)
      .def_property_readonly("block_size", &Model::block_size)
      .def_property_readonly("num_blocks", &Model::num_blocks)
      .def_property_readonly("k_cache", &Model::k_cache)
      .def_property_readonly("v_cache", &Model::v_cache);

  using svllm::model::DecodeGraphs;
  py::class_<DecodeGraphs>(m, "DecodeGraphs")
      .def(py::init<std::shared_ptr<Model>, int64_t, int64_t, std::vector<int64_t>>(),
           py::arg("model"), py::arg("max_num_seqs"), py::arg("max_blocks_per_seq"),
           py::arg("batch_sizes") = std::vector<int64_t>{})
      .def("step", &DecodeGraphs::step, py::arg("ids"), py::arg("positions"),
           py::arg("slot_mapping"), py::arg("block_tables"), py::arg("seq_lens"))
      .def_property_readonly("batch_sizes", &DecodeGraphs::batch_sizes);
}

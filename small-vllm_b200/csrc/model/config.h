#pragma once

#include <cstdint>
#include <optional>

namespace svllm {

// RoPE frequency scaling with rope_type "llama3". The same fields, in the same order, as the
// reference's src/model/config.h:10-15, so its ModelConfig::rope_scaling passes straight through
// to ops::rope and ops::qk_norm_rope.
struct Llama3RopeScaling {
  double factor;
  double low_freq_factor;
  double high_freq_factor;
  int64_t original_max_position_embeddings;
};

// Sizes and architecture flags of a Qwen3 or Llama checkpoint: the reference's ModelConfig
// (src/model/config.h:18-31), field for field, so a config it loads drives this forward as is.
struct ModelConfig {
  int64_t vocab_size;
  int64_t hidden_size;
  int64_t intermediate_size;
  int64_t num_layers;
  int64_t num_heads;
  int64_t num_kv_heads;
  int64_t head_dim;
  double rms_norm_eps;
  double rope_theta;
  bool tie_word_embeddings;
  bool qk_norm;  // Qwen3 normalises q and k per head before RoPE; Llama does not
  std::optional<Llama3RopeScaling> rope_scaling;
};

}  // namespace svllm

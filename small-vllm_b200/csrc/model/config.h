#pragma once

#include <cstdint>

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

}  // namespace svllm

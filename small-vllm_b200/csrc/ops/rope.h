#pragma once

#include <ATen/core/Tensor.h>

#include <optional>

#include "model/config.h"

namespace svllm::ops {

// Definition: Neox-style rotary position embedding, in place on q and k.
// Formula:    For each head and i < head_dim/2, with a = fp32(pos) * inv_freq[i],
//             c = bf16(cos a), s = bf16(sin a):
//               x[i]            <- bf16(bf16(x[i] * c) - bf16(x[i + head_dim/2] * s))
//               x[i + head_dim/2] <- bf16(bf16(x[i + head_dim/2] * c) + bf16(x[i] * s))
//             i.e. Hugging Face's apply_rotary_pos_emb with bf16 cos/sin. inv_freq is
//             rope_inv_freq(theta, head_dim, rope_scaling).
// Domain:     q [num_tokens, num_heads, head_dim] and k [num_tokens, num_kv_heads, head_dim]
//             bf16 (any leading dims that collapse into num_tokens; heads and head_dim
//             contiguous, tokens at any stride, so q and k may be views of a fused qkv tensor);
//             positions [num_tokens] int32 or int64, contiguous; head_dim even, <= 512; one
//             device.
// Returns:    Nothing; q and k hold the rotated heads.
// Throws:     c10::Error on dtype, shape, layout or device mismatches, or an unsupported device.
// Parameters come from the reference's ModelConfig (src/model/config.h:27,30: rope_theta,
// rope_scaling); Llama 3.2 has no q/k norm (config.h:29).
void rope(const at::Tensor& q, const at::Tensor& k, const at::Tensor& positions, double theta,
          const std::optional<Llama3RopeScaling>& rope_scaling);

// Definition: Qwen3's per-head q/k RMSNorm followed by rotary embedding, in one pass, in place.
// Formula:    Per head h = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w) with w = q_weight for q
//             heads and k_weight for k heads (Qwen3RMSNorm over head_dim), then rope() on h.
// Domain:     As rope(); q_weight and k_weight [head_dim] contiguous bf16 on the same device.
// Returns:    Nothing; q and k hold the normalised, rotated heads.
// Throws:     As rope().
// The qk_norm flag is the reference's src/model/config.h:29.
void qk_norm_rope(const at::Tensor& q, const at::Tensor& k, const at::Tensor& q_weight,
                  const at::Tensor& k_weight, const at::Tensor& positions, double eps,
                  double theta, const std::optional<Llama3RopeScaling>& rope_scaling);

// Definition: qk_norm_rope (Qwen3) or rope (Llama, when q_weight is undefined) fused with the
//             paged-KV cache write that follows it in a decoder layer.
// Formula:    q and k as qk_norm_rope / rope; then for every token t with s = slot_mapping[t]
//             >= 0: k_cache[s] = the rotated k[t], v_cache[s] = v[t] (the reference's
//             slot_mapping: block_id * block_size + offset, AGENTS.md "Names").
// Domain:     As rope(); v like k ([num_tokens, num_kv_heads, head_dim], tokens at any stride);
//             k_cache and v_cache contiguous [..., num_kv_heads, head_dim] of the same dtype
//             (e.g. [num_blocks, block_size, num_kv_heads, head_dim]); slot_mapping
//             [num_tokens] int64, contiguous; one device.
// Returns:    Nothing; q, k, and the cache slots hold the results. A negative slot skips its
//             token (padding).
// Throws:     As rope(), or on cache shape / dtype mismatches. A slot past the cache throws on
//             CPU; on CUDA it writes nothing and raises a bit of the device error word.
void qk_norm_rope_cache(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                        const at::Tensor& q_weight, const at::Tensor& k_weight,
                        const at::Tensor& positions, const at::Tensor& slot_mapping,
                        const at::Tensor& k_cache, const at::Tensor& v_cache, double eps,
                        double theta, const std::optional<Llama3RopeScaling>& rope_scaling);

void rope_cache(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                const at::Tensor& positions, const at::Tensor& slot_mapping,
                const at::Tensor& k_cache, const at::Tensor& v_cache, double theta,
                const std::optional<Llama3RopeScaling>& rope_scaling);

// Definition: The inverse-frequency table rope() uses, computed on the CPU with torch's own fp32
//             ops in Hugging Face's order (_compute_default_rope_parameters, and
//             _compute_llama3_parameters when rope_scaling is given), so it equals Hugging Face's
//             table bit for bit. Cached per parameter set.
// Returns:    A new fp32 CPU tensor [head_dim / 2].
// Throws:     c10::Error if theta <= 0, head_dim is not a positive even number, or the scaling
//             parameters are invalid.
at::Tensor rope_inv_freq(double theta, int64_t head_dim,
                         const std::optional<Llama3RopeScaling>& rope_scaling);

}  // namespace svllm::ops

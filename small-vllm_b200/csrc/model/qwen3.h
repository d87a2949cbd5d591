#pragma once

// The model-forward call sites of the fused layer ops: a Qwen3 / Llama decoder stack on LibTorch
// tensors (the reference's planned src/model forward, docs/ROADMAP.md:24-25), with a paged KV
// cache, greedy sampling, and decode steps replayed from CUDA graphs captured at bucketed batch
// sizes (docs/ROADMAP.md:42: 1, 2, 4, 8, then every 8 up to max_num_seqs; batches padded up).
//
// Per layer: add_rms_norm -> one qkv GEMM -> qk_norm_rope_cache (Qwen3) or rope_cache (Llama),
// which also writes k and v into the paged cache -> attention over the cache -> o GEMM ->
// add_rms_norm -> one gate_up GEMM -> silu_and_mul -> down GEMM. GEMMs are torch::linear
// (cuBLAS on GPU, as the reference plans, docs/ROADMAP.md:16), except for batches of up to 16
// token rows on CUDA, which take this library's decode-linear kernel. Attention: on CUDA
// decode steps the paged decode-attention kernel reads the cache in place; otherwise (prefill,
// mixed steps, CPU) a LibTorch composite over the gathered cache.

#include <ATen/ATen.h>

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "model/config.h"

namespace svllm::model {

// What one forward step attends over, in the reference's names (AGENTS.md "Names"):
//   slot_mapping     [T] int64    per token, the KV slot it writes: block_id * block_size +
//                                 offset; negative = padding (writes nothing)
//   block_tables     [S, B] int32 per request, its KV block ids in order (unused entries any
//                                 valid block id, e.g. 0)
//   seq_lens         [S] int32    per request, tokens in the KV cache including this step's
//   query_start_loc  [S+1] int32  prefix sums of the per-request query lengths
// Token i of request s (query_start_loc[s] <= i < query_start_loc[s+1]) sits at position
// seq_lens[s] - query_len + (i - query_start_loc[s]) and sees the cache up to and including it.
struct AttentionMetadata {
  at::Tensor slot_mapping;
  at::Tensor block_tables;
  at::Tensor seq_lens;
  at::Tensor query_start_loc;
  bool decode = false;  // every request has one query token (query_start_loc = 0..S)
};

// A decoder-only Qwen3 or Llama model. Weights are taken by their Hugging Face names; q/k/v and
// gate/up projections are concatenated at load into one qkv and one gate_up matrix (the
// reference's planned load-time fusion, docs/ROADMAP.md "Fused ops", #48).
class Model {
 public:
  Model(const ModelConfig& config, const std::unordered_map<std::string, at::Tensor>& weights);

  // Allocates a zeroed paged KV cache of num_blocks blocks of block_size tokens per layer,
  // [num_blocks, block_size, num_kv_heads, head_dim] each, on the weights' device.
  void allocate_kv_cache(int64_t num_blocks, int64_t block_size);

  // The final-norm hidden states [T, hidden] of the tokens ids [T] at positions [T]; writes
  // every token's k and v into the cache first.
  at::Tensor forward(const at::Tensor& ids, const at::Tensor& positions,
                     const AttentionMetadata& meta);

  // Logits [rows, vocab] of hidden rows (the tied embedding or lm_head).
  at::Tensor logits(const at::Tensor& hidden) const;

  // Greedy next tokens [rows] of hidden rows: argmax over logits, first maximum.
  at::Tensor greedy(const at::Tensor& hidden) const;

  // One decode step: every request has one query token (query_start_loc = 0..S). Returns the
  // next token id of every request, [S] int64.
  at::Tensor decode(const at::Tensor& ids, const at::Tensor& positions,
                    const at::Tensor& slot_mapping, const at::Tensor& block_tables,
                    const at::Tensor& seq_lens);

  const ModelConfig& config() const { return config_; }
  int64_t block_size() const { return block_size_; }
  int64_t num_blocks() const { return num_blocks_; }
  const std::vector<at::Tensor>& k_cache() const { return k_cache_; }
  const std::vector<at::Tensor>& v_cache() const { return v_cache_; }

 private:
  struct Layer {
    at::Tensor input_norm;  // [H]
    at::Tensor qkv;         // [(Hq + 2 Hk) D, H]
    at::Tensor q_norm;      // [D] (Qwen3) or undefined
    at::Tensor k_norm;
    at::Tensor o_proj;      // [H, Hq D]
    at::Tensor post_norm;   // [H]
    at::Tensor gate_up;     // [2 I, H]
    at::Tensor down;        // [H, I]
  };

  // Per token, the cache slot of every context position it may see, and which of them it does.
  struct AttentionPlan {
    at::Tensor slots;  // [T, L] int64, L = blocks per request * block_size
    at::Tensor mask;   // [T, 1, 1, L]: 0 where visible, -inf elsewhere
  };
  AttentionPlan plan_attention(int64_t tokens, const AttentionMetadata& meta) const;
  at::Tensor attention(const at::Tensor& q, int64_t layer, const AttentionPlan& plan) const;
  // Decode steps on CUDA: the paged decode-attention kernel straight from the cache.
  bool paged_decode_ok(const AttentionMetadata& meta) const;
  at::Tensor paged_decode_attention(const at::Tensor& q, int64_t layer,
                                    const AttentionMetadata& meta) const;

  ModelConfig config_;
  at::Tensor embed_;       // [V, H]
  at::Tensor lm_head_;     // [V, H]: embed_ when tied
  at::Tensor final_norm_;  // [H]
  std::vector<Layer> layers_;
  std::vector<at::Tensor> k_cache_;
  std::vector<at::Tensor> v_cache_;
  int64_t block_size_ = 0;
  int64_t num_blocks_ = 0;
};

// Decode steps replayed from CUDA graphs, one per batch-size bucket. Each graph is captured once
// (after one eager warm-up) over static input buffers of the bucket's size; a step copies its
// inputs in, pads the batch up to the bucket (padding tokens: id 0, position 0, slot -1 so they
// write no cache, one visible token), replays, and returns the first S next-token ids. The
// model's KV cache must be allocated first and stay in place.
class DecodeGraphs {
 public:
  // batch_sizes empty: 1, 2, 4, 8, then every 8 up to max_num_seqs.
  DecodeGraphs(std::shared_ptr<Model> model, int64_t max_num_seqs, int64_t max_blocks_per_seq,
               std::vector<int64_t> batch_sizes = {});
  ~DecodeGraphs();

  at::Tensor step(const at::Tensor& ids, const at::Tensor& positions,
                  const at::Tensor& slot_mapping, const at::Tensor& block_tables,
                  const at::Tensor& seq_lens);

  const std::vector<int64_t>& batch_sizes() const { return sizes_; }

 private:
  struct Impl;
  std::shared_ptr<Model> model_;
  std::vector<int64_t> sizes_;
  std::unique_ptr<Impl> impl_;
};

}  // namespace svllm::model

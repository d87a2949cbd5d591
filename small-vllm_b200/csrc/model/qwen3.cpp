#include "model/qwen3.h"

#include <c10/util/Exception.h>

#include <algorithm>
#include <cmath>
#include <limits>
#include <utility>

#include "ops/add_rms_norm.h"
#include "ops/embedding.h"
#include "ops/rms_norm.h"
#include "ops/rope.h"
#include "ops/sampling.h"
#include "ops/silu_and_mul.h"

#include "svllm_kernels.h"

#ifdef SVLLM_CUDA
#include <ATen/cuda/CUDAContext.h>
#include <ATen/cuda/CUDAGraph.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#endif

namespace svllm::model {
namespace {

at::Tensor weight(const std::unordered_map<std::string, at::Tensor>& weights,
                  const std::string& name, at::IntArrayRef shape) {
  const auto it = weights.find(name);
  TORCH_CHECK(it != weights.end(), "Model: missing weight ", name);
  TORCH_CHECK(it->second.sizes() == shape, "Model: ", name, " has shape ", it->second.sizes(),
              ", the config needs ", shape);
  return it->second;
}

// x [T, K] . w [N, K]^T. Decode-sized batches (up to 16 rows) in bf16 on CUDA take the
// decode-linear kernel, which streams the weight over every SM; larger batches, other dtypes,
// the CPU and shapes that kernel does not take go through at::linear (cuBLAS on GPU).
at::Tensor project(const at::Tensor& x, const at::Tensor& w) {
#ifdef SVLLM_CUDA
  if (x.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
      x.dim() == 2 && w.dim() == 2 && x.size(0) <= 16 && x.stride(1) == 1 && w.stride(1) == 1) {
    at::Tensor out = at::empty({x.size(0), w.size(0)}, x.options());
    const c10::cuda::CUDAGuard device_guard(x.device());
    const int status = svllm_decode_linear_bf16(
        out.data_ptr(), out.stride(0), x.data_ptr(), x.size(0), x.size(1), x.stride(0),
        w.data_ptr(), w.size(0), w.stride(0),
        reinterpret_cast<svllm_stream>(c10::cuda::getCurrentCUDAStream().stream()));
    if (status == SVLLM_OK) return out;
    TORCH_CHECK(status == SVLLM_ERR_UNSUPPORTED, "Model: decode linear: ",
                svllm_status_string(status));
  }
#endif
  return at::linear(x, w);
}

}  // namespace

Model::Model(const ModelConfig& config,
             const std::unordered_map<std::string, at::Tensor>& weights)
    : config_(config) {
  const int64_t H = config.hidden_size, V = config.vocab_size, I = config.intermediate_size;
  const int64_t Hq = config.num_heads, Hk = config.num_kv_heads, D = config.head_dim;
  TORCH_CHECK(H > 0 && V > 0 && I > 0 && Hq > 0 && Hk > 0 && D > 0 && Hq % Hk == 0 &&
                  config.num_layers > 0,
              "Model: invalid config (hidden ", H, ", vocab ", V, ", intermediate ", I,
              ", heads ", Hq, "/", Hk, ", head_dim ", D, ", layers ", config.num_layers, ")");
  embed_ = weight(weights, "model.embed_tokens.weight", {V, H}).contiguous();
  lm_head_ = config.tie_word_embeddings ? embed_
                                        : weight(weights, "lm_head.weight", {V, H}).contiguous();
  final_norm_ = weight(weights, "model.norm.weight", {H}).contiguous();
  layers_.reserve(config.num_layers);
  for (int64_t l = 0; l < config.num_layers; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    Layer layer;
    layer.input_norm = weight(weights, p + "input_layernorm.weight", {H}).contiguous();
    layer.qkv = at::cat({weight(weights, p + "self_attn.q_proj.weight", {Hq * D, H}),
                         weight(weights, p + "self_attn.k_proj.weight", {Hk * D, H}),
                         weight(weights, p + "self_attn.v_proj.weight", {Hk * D, H})},
                        0)
                    .contiguous();
    if (config.qk_norm) {
      layer.q_norm = weight(weights, p + "self_attn.q_norm.weight", {D}).contiguous();
      layer.k_norm = weight(weights, p + "self_attn.k_norm.weight", {D}).contiguous();
    }
    layer.o_proj = weight(weights, p + "self_attn.o_proj.weight", {H, Hq * D}).contiguous();
    layer.post_norm = weight(weights, p + "post_attention_layernorm.weight", {H}).contiguous();
    layer.gate_up = at::cat({weight(weights, p + "mlp.gate_proj.weight", {I, H}),
                             weight(weights, p + "mlp.up_proj.weight", {I, H})},
                            0)
                        .contiguous();
    layer.down = weight(weights, p + "mlp.down_proj.weight", {H, I}).contiguous();
    layers_.push_back(std::move(layer));
  }
}

void Model::allocate_kv_cache(int64_t num_blocks, int64_t block_size) {
  TORCH_CHECK(num_blocks > 0 && block_size > 0, "allocate_kv_cache: num_blocks ", num_blocks,
              " and block_size ", block_size, " must be positive");
  k_cache_.clear();
  v_cache_.clear();
  for (int64_t l = 0; l < config_.num_layers; ++l) {
    const auto shape = {num_blocks, block_size, config_.num_kv_heads, config_.head_dim};
    k_cache_.push_back(at::zeros(shape, embed_.options()));
    v_cache_.push_back(at::zeros(shape, embed_.options()));
  }
  num_blocks_ = num_blocks;
  block_size_ = block_size;
}

Model::AttentionPlan Model::plan_attention(int64_t tokens, const AttentionMetadata& meta) const {
  const at::TensorOptions i64 = at::TensorOptions().dtype(at::kLong).device(embed_.device());
  const int64_t requests = meta.seq_lens.size(0);
  const at::Tensor qsl = meta.query_start_loc.to(at::kLong);
  const at::Tensor tok = at::arange(tokens, i64);
  // the request of each token: the first whose query end lies beyond it
  const at::Tensor req = at::searchsorted(qsl.narrow(0, 1, requests), tok, false, true);
  const at::Tensor start = qsl.index_select(0, req);
  const at::Tensor query_len = qsl.index_select(0, req + 1) - start;
  const at::Tensor seq = meta.seq_lens.to(at::kLong).index_select(0, req);
  const at::Tensor visible = seq - query_len + (tok - start) + 1;  // causal: up to itself
  const at::Tensor tables = meta.block_tables.to(at::kLong).index_select(0, req);
  const int64_t length = meta.block_tables.size(1) * block_size_;
  const at::Tensor slots =
      (tables.unsqueeze(2) * block_size_ + at::arange(block_size_, i64)).view({tokens, length});
  // additive mask in the activations' dtype, built once per step for every layer (a boolean
  // mask would be converted again by every attention call)
  const at::Tensor hidden_pos = at::arange(length, i64).unsqueeze(0) >= visible.unsqueeze(1);
  const at::Tensor mask = at::zeros({tokens, length}, embed_.options())
                              .masked_fill_(hidden_pos, -std::numeric_limits<float>::infinity());
  return AttentionPlan{slots, mask.view({tokens, 1, 1, length})};
}

at::Tensor Model::attention(const at::Tensor& q, int64_t layer, const AttentionPlan& plan) const {
  const int64_t T = q.size(0), Hq = config_.num_heads, Hk = config_.num_kv_heads;
  const int64_t D = config_.head_dim, L = plan.slots.size(1);
  const at::Tensor idx = plan.slots.reshape({-1});
  const at::Tensor k = k_cache_[layer].view({-1, Hk, D}).index_select(0, idx).view({T, L, Hk, D});
  const at::Tensor v = v_cache_[layer].view({-1, Hk, D}).index_select(0, idx).view({T, L, Hk, D});
  const at::Tensor out = at::scaled_dot_product_attention(
      q.unsqueeze(2), k.transpose(1, 2), v.transpose(1, 2), plan.mask, 0.0, false,
      std::pow(static_cast<double>(D), -0.5), /*enable_gqa=*/Hq != Hk);
  return out.reshape({T, Hq * D});
}

bool Model::paged_decode_ok(const AttentionMetadata& meta) const {
#ifdef SVLLM_CUDA
  const int64_t group = config_.num_heads / config_.num_kv_heads;
  return meta.decode && embed_.is_cuda() && embed_.scalar_type() == at::kBFloat16 &&
         (config_.head_dim == 64 || config_.head_dim == 128) && group <= 8 &&
         (group & (group - 1)) == 0;
#else
  (void)meta;
  return false;
#endif
}

at::Tensor Model::paged_decode_attention(const at::Tensor& q, int64_t layer,
                                         const AttentionMetadata& meta) const {
  const int64_t S = q.size(0), Hq = config_.num_heads, D = config_.head_dim;
#ifdef SVLLM_CUDA
  const at::Tensor tables = meta.block_tables.to(at::kInt).contiguous();
  const at::Tensor lens = meta.seq_lens.to(at::kInt).contiguous();
  at::Tensor out = at::empty({S, Hq, D}, q.options());
  const c10::cuda::CUDAGuard device_guard(q.device());
  const int status = svllm_paged_decode_attention_bf16(
      out.data_ptr(), q.data_ptr(), q.stride(0), k_cache_[layer].data_ptr(),
      v_cache_[layer].data_ptr(), num_blocks_, block_size_, tables.const_data_ptr<int32_t>(),
      tables.size(1), lens.const_data_ptr<int32_t>(), S, Hq, config_.num_kv_heads, D,
      tables.size(1) * block_size_, static_cast<float>(std::pow(static_cast<double>(D), -0.5)),
      reinterpret_cast<svllm_stream>(c10::cuda::getCurrentCUDAStream().stream()));
  TORCH_CHECK(status == SVLLM_OK, "Model: paged decode attention: ", svllm_status_string(status));
  return out.view({S, Hq * D});
#else
  (void)layer;
  (void)meta;
  TORCH_CHECK(false, "Model: paged decode attention needs CUDA");
  return at::Tensor();
#endif
}

at::Tensor Model::forward(const at::Tensor& ids, const at::Tensor& positions,
                          const AttentionMetadata& meta) {
  TORCH_CHECK(!k_cache_.empty(), "Model::forward: allocate_kv_cache first");
  TORCH_CHECK(ids.dim() == 1 && positions.dim() == 1 && positions.size(0) == ids.size(0) &&
                  meta.slot_mapping.dim() == 1 && meta.slot_mapping.size(0) == ids.size(0),
              "Model::forward: ids ", ids.sizes(), ", positions ", positions.sizes(),
              " and slot_mapping ", meta.slot_mapping.sizes(), " must be [tokens]");
  TORCH_CHECK(meta.block_tables.dim() == 2 && meta.seq_lens.dim() == 1 &&
                  meta.query_start_loc.dim() == 1 &&
                  meta.block_tables.size(0) == meta.seq_lens.size(0) &&
                  meta.query_start_loc.size(0) == meta.seq_lens.size(0) + 1,
              "Model::forward: block_tables ", meta.block_tables.sizes(), ", seq_lens ",
              meta.seq_lens.sizes(), " and query_start_loc ", meta.query_start_loc.sizes(),
              " must be [S, blocks], [S] and [S + 1]");
  const int64_t T = ids.size(0);
  const int64_t Hq = config_.num_heads, Hk = config_.num_kv_heads, D = config_.head_dim;
  const double eps = config_.rms_norm_eps;
  const bool paged = paged_decode_ok(meta);
  const AttentionPlan plan = paged ? AttentionPlan{} : plan_attention(T, meta);

  at::Tensor hidden = ops::embedding(ids, embed_);
  at::Tensor residual;
  for (size_t l = 0; l < layers_.size(); ++l) {
    const Layer& layer = layers_[l];
    if (l == 0) {
      residual = hidden;
      hidden = ops::rms_norm(residual, layer.input_norm, eps);
    } else {
      ops::add_rms_norm(hidden, residual, layer.input_norm, eps);
    }
    const at::Tensor qkv = project(hidden, layer.qkv);  // [T, (Hq + 2 Hk) D]
    const at::Tensor q = qkv.narrow(1, 0, Hq * D).view({T, Hq, D});
    const at::Tensor k = qkv.narrow(1, Hq * D, Hk * D).view({T, Hk, D});
    const at::Tensor v = qkv.narrow(1, (Hq + Hk) * D, Hk * D).view({T, Hk, D});
    if (config_.qk_norm) {
      ops::qk_norm_rope_cache(q, k, v, layer.q_norm, layer.k_norm, positions, meta.slot_mapping,
                              k_cache_[l], v_cache_[l], eps, config_.rope_theta,
                              config_.rope_scaling);
    } else {
      ops::rope_cache(q, k, v, positions, meta.slot_mapping, k_cache_[l], v_cache_[l],
                      config_.rope_theta, config_.rope_scaling);
    }
    const at::Tensor attn = paged ? paged_decode_attention(q, static_cast<int64_t>(l), meta)
                                  : attention(q, static_cast<int64_t>(l), plan);
    hidden = project(attn, layer.o_proj);
    ops::add_rms_norm(hidden, residual, layer.post_norm, eps);
    hidden = project(ops::silu_and_mul(project(hidden, layer.gate_up)), layer.down);
  }
  ops::add_rms_norm(hidden, residual, final_norm_, eps);
  return hidden;
}

at::Tensor Model::logits(const at::Tensor& hidden) const { return at::linear(hidden, lm_head_); }

at::Tensor Model::greedy(const at::Tensor& hidden) const {
  return ops::greedy_sample(hidden, lm_head_);
}

at::Tensor Model::decode(const at::Tensor& ids, const at::Tensor& positions,
                         const at::Tensor& slot_mapping, const at::Tensor& block_tables,
                         const at::Tensor& seq_lens) {
  const at::Tensor qsl = at::arange(
      ids.size(0) + 1, at::TensorOptions().dtype(at::kInt).device(ids.device()));
  return greedy(forward(ids, positions, {slot_mapping, block_tables, seq_lens, qsl, true}));
}

#ifdef SVLLM_CUDA

struct DecodeGraphs::Impl {
  at::Tensor ids, positions, slots, tables, seq_lens;  // static inputs, the largest bucket
  std::vector<std::unique_ptr<at::cuda::CUDAGraph>> graphs;
  std::vector<at::Tensor> outs;
};

DecodeGraphs::DecodeGraphs(std::shared_ptr<Model> model, int64_t max_num_seqs,
                           int64_t max_blocks_per_seq, std::vector<int64_t> batch_sizes)
    : model_(std::move(model)), sizes_(std::move(batch_sizes)), impl_(std::make_unique<Impl>()) {
  TORCH_CHECK(model_ != nullptr && !model_->k_cache().empty(),
              "DecodeGraphs: the model needs its KV cache allocated first");
  const at::Device device = model_->k_cache()[0].device();
  TORCH_CHECK(device.is_cuda(), "DecodeGraphs: CUDA graphs need a model on a CUDA device");
  TORCH_CHECK(max_num_seqs > 0 && max_blocks_per_seq > 0, "DecodeGraphs: max_num_seqs ",
              max_num_seqs, " and max_blocks_per_seq ", max_blocks_per_seq, " must be positive");
  if (sizes_.empty()) {
    for (int64_t b : {1, 2, 4, 8}) {
      if (b <= max_num_seqs) sizes_.push_back(b);
    }
    for (int64_t b = 16; b <= max_num_seqs; b += 8) sizes_.push_back(b);
    if (sizes_.back() < max_num_seqs) sizes_.push_back(max_num_seqs);
  }
  std::sort(sizes_.begin(), sizes_.end());
  sizes_.erase(std::unique(sizes_.begin(), sizes_.end()), sizes_.end());
  TORCH_CHECK(sizes_.front() > 0, "DecodeGraphs: batch sizes must be positive");
  const int64_t max_b = sizes_.back();

  c10::cuda::CUDAGuard device_guard(device);
  const auto i64 = at::TensorOptions().dtype(at::kLong).device(device);
  const auto i32 = at::TensorOptions().dtype(at::kInt).device(device);
  Impl& s = *impl_;
  s.ids = at::zeros({max_b}, i64);
  s.positions = at::zeros({max_b}, i64);
  s.slots = at::full({max_b}, -1, i64);
  s.tables = at::zeros({max_b, max_blocks_per_seq}, i32);
  s.seq_lens = at::ones({max_b}, i32);
  s.graphs.resize(sizes_.size());
  s.outs.resize(sizes_.size());

  // Capture on a side stream, the largest bucket first so the shared pool fits every graph.
  const at::cuda::MempoolId_t pool = at::cuda::graph_pool_handle();
  const c10::cuda::CUDAStream stream = c10::cuda::getStreamFromPool(false, device.index());
  const c10::cuda::CUDAStreamGuard stream_guard(stream);
  for (int64_t k = static_cast<int64_t>(sizes_.size()) - 1; k >= 0; --k) {
    const int64_t b = sizes_[k];
    const auto run = [&] {
      return model_->decode(s.ids.narrow(0, 0, b), s.positions.narrow(0, 0, b),
                            s.slots.narrow(0, 0, b), s.tables.narrow(0, 0, b),
                            s.seq_lens.narrow(0, 0, b));
    };
    run();  // warm-up: the op layer's one-time set-up happens outside the capture
    stream.synchronize();
    auto graph = std::make_unique<at::cuda::CUDAGraph>();
    graph->capture_begin(pool);
    s.outs[k] = run();
    graph->capture_end();
    s.graphs[k] = std::move(graph);
  }
  stream.synchronize();
}

DecodeGraphs::~DecodeGraphs() = default;

at::Tensor DecodeGraphs::step(const at::Tensor& ids, const at::Tensor& positions,
                              const at::Tensor& slot_mapping, const at::Tensor& block_tables,
                              const at::Tensor& seq_lens) {
  Impl& s = *impl_;
  const int64_t n = ids.size(0);
  TORCH_CHECK(n >= 1 && n <= sizes_.back(), "DecodeGraphs::step: ", n,
              " requests; the largest captured batch is ", sizes_.back());
  TORCH_CHECK(positions.size(0) == n && slot_mapping.size(0) == n && seq_lens.size(0) == n &&
                  block_tables.dim() == 2 && block_tables.size(0) == n &&
                  block_tables.size(1) <= s.tables.size(1),
              "DecodeGraphs::step: inputs for ", n, " requests with block tables of at most ",
              s.tables.size(1), " blocks expected, got block_tables ", block_tables.sizes());
  const size_t k = std::lower_bound(sizes_.begin(), sizes_.end(), n) - sizes_.begin();
  const int64_t b = sizes_[k];
  const int64_t blocks = block_tables.size(1);
  const c10::cuda::CUDAGuard device_guard(s.ids.device());
  s.ids.narrow(0, 0, n).copy_(ids);
  s.positions.narrow(0, 0, n).copy_(positions);
  s.slots.narrow(0, 0, n).copy_(slot_mapping);
  s.tables.narrow(0, 0, n).narrow(1, 0, blocks).copy_(block_tables);
  if (blocks < s.tables.size(1)) {
    s.tables.narrow(0, 0, n).narrow(1, blocks, s.tables.size(1) - blocks).zero_();
  }
  s.seq_lens.narrow(0, 0, n).copy_(seq_lens);
  if (b > n) {
    // padding requests: no cache write, one visible token of block 0
    s.ids.narrow(0, n, b - n).zero_();
    s.positions.narrow(0, n, b - n).zero_();
    s.slots.narrow(0, n, b - n).fill_(-1);
    s.tables.narrow(0, n, b - n).zero_();
    s.seq_lens.narrow(0, n, b - n).fill_(1);
  }
  s.graphs[k]->replay();
  return s.outs[k].narrow(0, 0, n).clone();
}

#else

struct DecodeGraphs::Impl {};

DecodeGraphs::DecodeGraphs(std::shared_ptr<Model>, int64_t, int64_t, std::vector<int64_t>) {
  TORCH_CHECK(false, "DecodeGraphs: built without CUDA");
}
DecodeGraphs::~DecodeGraphs() = default;
at::Tensor DecodeGraphs::step(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                              const at::Tensor&, const at::Tensor&) {
  TORCH_CHECK(false, "DecodeGraphs: built without CUDA");
}

#endif

}  // namespace svllm::model

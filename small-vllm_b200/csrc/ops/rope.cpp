#include "ops/rope.h"

#include <ATen/ATen.h>
#include <c10/util/Exception.h>

#include <cmath>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "ops/rope_kernels.h"

namespace svllm::ops {
namespace {

constexpr int64_t kMaxHeadDim = 512;
constexpr double kTwoPi = 2.0 * 3.141592653589793;  // Python's 2 * math.pi

using InvFreqKey = std::tuple<double, int64_t, bool, double, double, double, int64_t>;

// The table for one parameter set, built once (torch CPU ops are not free at decode rates).
const std::vector<float>& cached_inv_freq(double theta, int64_t head_dim,
                                          const std::optional<Llama3RopeScaling>& scaling) {
  static std::mutex mutex;
  static std::map<InvFreqKey, std::vector<float>> cache;
  const InvFreqKey key{theta,
                       head_dim,
                       scaling.has_value(),
                       scaling ? scaling->factor : 0.0,
                       scaling ? scaling->low_freq_factor : 0.0,
                       scaling ? scaling->high_freq_factor : 0.0,
                       scaling ? scaling->original_max_position_embeddings : 0};
  const std::lock_guard<std::mutex> lock(mutex);
  auto it = cache.find(key);
  if (it == cache.end()) {
    const at::Tensor table = rope_inv_freq(theta, head_dim, scaling).contiguous();
    const float* p = table.const_data_ptr<float>();
    it = cache.emplace(key, std::vector<float>(p, p + table.numel())).first;
  }
  return it->second;
}

// Collapses the leading dims into tokens without copying: [num_tokens, heads, head_dim].
at::Tensor token_view(const char* op, const char* name, const at::Tensor& t) {
  TORCH_CHECK(t.dim() >= 2, op, ": ", name, " must be [..., heads, head_dim], got shape ",
              t.sizes());
  const int64_t heads = t.size(-2);
  const int64_t head_dim = t.size(-1);
  TORCH_CHECK(t.stride(-1) == 1 && (heads <= 1 || t.stride(-2) == head_dim), op, ": ", name,
              " must have contiguous heads and head_dim, got strides ", t.strides());
  if (t.dim() == 2) {
    return t.unsqueeze(0);
  }
  if (t.dim() == 3) {
    return t;
  }
  // view() fails (without copying) if the leading dims do not collapse to one token stride
  return t.view({-1, heads, head_dim});
}

// Cache-write operands of the *_cache ops (all undefined for plain rope / qk_norm_rope).
struct KvCacheArgs {
  at::Tensor v;
  at::Tensor slot_mapping;
  at::Tensor k_cache;
  at::Tensor v_cache;
};

void check_and_run(const char* op, const at::Tensor& q, const at::Tensor& k,
                   const at::Tensor& q_weight, const at::Tensor& k_weight,
                   const at::Tensor& positions, double eps, double theta,
                   const std::optional<Llama3RopeScaling>& rope_scaling,
                   const KvCacheArgs& cache = {}) {
  const bool norm = q_weight.defined();
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 &&
                  (!norm || (q_weight.scalar_type() == at::kBFloat16 &&
                             k_weight.scalar_type() == at::kBFloat16)),
              op, ": expected bf16 q, k", norm ? " and norm weights" : "", ", got ",
              q.scalar_type(), " and ", k.scalar_type());
  TORCH_CHECK(positions.scalar_type() == at::kInt || positions.scalar_type() == at::kLong, op,
              ": expected int32 or int64 positions, got ", positions.scalar_type());
  const at::Tensor q3 = token_view(op, "q", q);
  const at::Tensor k3 = token_view(op, "k", k);
  const int64_t head_dim = q3.size(2);
  TORCH_CHECK(k3.size(2) == head_dim && q3.size(0) == k3.size(0), op, ": q of shape ", q.sizes(),
              " and k of shape ", k.sizes(), " do not match");
  TORCH_CHECK(head_dim > 0 && head_dim % 2 == 0 && head_dim <= kMaxHeadDim, op,
              ": head_dim must be even and at most ", kMaxHeadDim, ", got ", head_dim);
  TORCH_CHECK(positions.numel() == q3.size(0), op, ": ", positions.numel(),
              " positions for ", q3.size(0), " tokens");
  TORCH_CHECK(positions.is_contiguous(), op, ": positions must be contiguous");
  if (norm) {
    TORCH_CHECK(q_weight.dim() == 1 && k_weight.dim() == 1 && q_weight.size(0) == head_dim &&
                    k_weight.size(0) == head_dim,
                op, ": q_weight of shape ", q_weight.sizes(), " and k_weight of shape ",
                k_weight.sizes(), " do not match head_dim ", head_dim);
    TORCH_CHECK(q_weight.is_contiguous() && k_weight.is_contiguous(), op,
                ": q_weight and k_weight must be contiguous");
  }
  const bool same_device = k.device() == q.device() && positions.device() == q.device() &&
                           (!norm || (q_weight.device() == q.device() &&
                                      k_weight.device() == q.device()));
  TORCH_CHECK(same_device, op, ": q is on ", q.device(), " but k, positions",
              norm ? " or the weights are" : " are", " elsewhere (k on ", k.device(),
              ", positions on ", positions.device(), ")");

  const bool with_cache = cache.v.defined();
  at::Tensor v3, kc, vc;
  if (with_cache) {
    TORCH_CHECK(cache.v.scalar_type() == q.scalar_type() &&
                    cache.k_cache.scalar_type() == q.scalar_type() &&
                    cache.v_cache.scalar_type() == q.scalar_type(),
                op, ": expected bf16 v, k_cache and v_cache");
    v3 = token_view(op, "v", cache.v);
    TORCH_CHECK(v3.sizes() == k3.sizes(), op, ": v of shape ", cache.v.sizes(),
                " does not match k of shape ", k.sizes());
    const int64_t kv_heads = k3.size(1);
    for (const at::Tensor* c : {&cache.k_cache, &cache.v_cache}) {
      TORCH_CHECK(c->dim() >= 2 && c->size(-1) == head_dim && c->size(-2) == kv_heads &&
                      c->is_contiguous(),
                  op, ": caches must be contiguous [..., num_kv_heads, head_dim] = [..., ",
                  kv_heads, ", ", head_dim, "], got shape ", c->sizes());
    }
    TORCH_CHECK(cache.k_cache.sizes() == cache.v_cache.sizes(), op, ": k_cache of shape ",
                cache.k_cache.sizes(), " does not match v_cache of shape ",
                cache.v_cache.sizes());
    TORCH_CHECK(cache.slot_mapping.scalar_type() == at::kLong &&
                    cache.slot_mapping.is_contiguous() &&
                    cache.slot_mapping.numel() == q3.size(0),
                op, ": slot_mapping must be contiguous int64 with one slot per token");
    const bool cache_same_device = cache.v.device() == q.device() &&
                                   cache.slot_mapping.device() == q.device() &&
                                   cache.k_cache.device() == q.device() &&
                                   cache.v_cache.device() == q.device();
    TORCH_CHECK(cache_same_device, op, ": q is on ", q.device(),
                " but v, slot_mapping or a cache is elsewhere");
    kc = cache.k_cache.view({-1, kv_heads, head_dim});
    vc = cache.v_cache.view({-1, kv_heads, head_dim});
  }

  const std::vector<float>& inv_freq = cached_inv_freq(theta, head_dim, rope_scaling);

  switch (q.device().type()) {
    case c10::DeviceType::CPU: {
      cpu_impl::rope(q3, k3, q_weight, k_weight, positions, eps, inv_freq.data());
      if (with_cache) {
        const int64_t bad = cpu_impl::write_kv_cache(k3, v3, cache.slot_mapping, kc, vc);
        TORCH_CHECK(bad == 0, op, ": ", bad, " slots past the cache's ", kc.size(0));
      }
      break;
    }
    case c10::DeviceType::CUDA:
      if (with_cache) {
        cuda_impl::rope_cache(q3, k3, v3, q_weight, k_weight, positions, cache.slot_mapping, kc,
                              vc, eps, inv_freq.data());
      } else {
        cuda_impl::rope(q3, k3, q_weight, k_weight, positions, eps, inv_freq.data());
      }
      break;
    default:
      TORCH_CHECK(false, op, ": unsupported device ", q.device());
  }
}

}  // namespace

at::Tensor rope_inv_freq(double theta, int64_t head_dim,
                         const std::optional<Llama3RopeScaling>& rope_scaling) {
  TORCH_CHECK(theta > 0.0, "rope_inv_freq: theta must be positive, got ", theta);
  TORCH_CHECK(head_dim > 0 && head_dim % 2 == 0, "rope_inv_freq: head_dim must be positive and ",
              "even, got ", head_dim);

  // Hugging Face: inv_freq = 1.0 / (base ** (arange(0, dim, 2).float() / dim)). Python evaluates
  // `scalar ** t` as pow(scalar, t) and `scalar / t` as reciprocal(t) * scalar.
  const at::Tensor exponent =
      at::arange(0, head_dim, 2, at::TensorOptions().dtype(at::kLong)).to(at::kFloat) /
      static_cast<double>(head_dim);
  at::Tensor inv_freq = at::reciprocal(at::pow(theta, exponent)) * 1.0;
  if (!rope_scaling) {
    return inv_freq;
  }

  // Hugging Face's _compute_llama3_parameters, operation for operation.
  const Llama3RopeScaling& s = *rope_scaling;
  TORCH_CHECK(s.factor > 0.0 && s.low_freq_factor > 0.0 && s.high_freq_factor > s.low_freq_factor &&
                  s.original_max_position_embeddings > 0,
              "rope_inv_freq: invalid llama3 rope scaling (factor ", s.factor, ", low ",
              s.low_freq_factor, ", high ", s.high_freq_factor, ", original max positions ",
              s.original_max_position_embeddings, ")");
  const double old_context_len = static_cast<double>(s.original_max_position_embeddings);
  const double low_freq_wavelen = old_context_len / s.low_freq_factor;
  const double high_freq_wavelen = old_context_len / s.high_freq_factor;
  const at::Tensor wavelen = at::reciprocal(inv_freq) * kTwoPi;
  at::Tensor inv_freq_llama = at::where(wavelen > low_freq_wavelen, inv_freq / s.factor, inv_freq);
  const at::Tensor smooth_factor = (at::reciprocal(wavelen) * old_context_len - s.low_freq_factor) /
                                   (s.high_freq_factor - s.low_freq_factor);
  const at::Tensor smoothed_inv_freq =
      (1 - smooth_factor) * inv_freq_llama / s.factor + smooth_factor * inv_freq_llama;
  const at::Tensor is_medium_freq =
      at::logical_not(wavelen < high_freq_wavelen) * at::logical_not(wavelen > low_freq_wavelen);
  return at::where(is_medium_freq, smoothed_inv_freq, inv_freq_llama);
}

void rope(const at::Tensor& q, const at::Tensor& k, const at::Tensor& positions, double theta,
          const std::optional<Llama3RopeScaling>& rope_scaling) {
  check_and_run("rope", q, k, at::Tensor(), at::Tensor(), positions, 0.0, theta, rope_scaling);
}

void qk_norm_rope(const at::Tensor& q, const at::Tensor& k, const at::Tensor& q_weight,
                  const at::Tensor& k_weight, const at::Tensor& positions, double eps,
                  double theta, const std::optional<Llama3RopeScaling>& rope_scaling) {
  TORCH_CHECK(q_weight.defined() && k_weight.defined(),
              "qk_norm_rope: q_weight and k_weight are required");
  check_and_run("qk_norm_rope", q, k, q_weight, k_weight, positions, eps, theta, rope_scaling);
}

void qk_norm_rope_cache(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                        const at::Tensor& q_weight, const at::Tensor& k_weight,
                        const at::Tensor& positions, const at::Tensor& slot_mapping,
                        const at::Tensor& k_cache, const at::Tensor& v_cache, double eps,
                        double theta, const std::optional<Llama3RopeScaling>& rope_scaling) {
  TORCH_CHECK(q_weight.defined() && k_weight.defined(),
              "qk_norm_rope_cache: q_weight and k_weight are required");
  check_and_run("qk_norm_rope_cache", q, k, q_weight, k_weight, positions, eps, theta,
                rope_scaling, {v, slot_mapping, k_cache, v_cache});
}

void rope_cache(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                const at::Tensor& positions, const at::Tensor& slot_mapping,
                const at::Tensor& k_cache, const at::Tensor& v_cache, double theta,
                const std::optional<Llama3RopeScaling>& rope_scaling) {
  check_and_run("rope_cache", q, k, at::Tensor(), at::Tensor(), positions, 0.0, theta,
                rope_scaling, {v, slot_mapping, k_cache, v_cache});
}

}  // namespace svllm::ops

/*
 * svllm_kernels.h - C ABI of the sm_100a layer-op kernels (libsvllm_kernels.so).
 *
 * These are the memory-bound, token-row-parallel ops around every GEMM of a Qwen3 / Llama
 * decoder layer: RMSNorm, RMSNorm with the fused residual add, Qwen3's per-head q/k RMSNorm
 * fused with rotary embedding, rotary embedding alone (plain theta or Llama-3 frequency
 * scaling), SiLU(gate) * up, and the token-embedding gather.
 *
 * Conventions (every entry point):
 *   - Plain pointers and sizes only. Tensor pointers are DEVICE pointers on the current CUDA
 *     device; `stream` is a cudaStream_t (NULL = the legacy default stream). Work is enqueued
 *     on `stream` and the call returns without synchronising: no host sync, no allocation, so
 *     every entry point may be captured in a CUDA graph.
 *   - Rows are `num_rows` (or `num_tokens`) rows of `hidden` elements; a row stride is given in
 *     elements and must be >= the row length. The last dimension is always contiguous.
 *   - bf16 is IEEE bfloat16 (2 bytes); the *_f32 variants take fp32. Arithmetic is fp32.
 *   - The return value is an svllm_status; svllm_status_string() names it. A call that returns
 *     an error has enqueued nothing. No entry point throws.
 *   - 16-byte aligned pointers and strides with a row length that is a multiple of 16 bytes take
 *     the bulk-copy (TMA) path; anything else takes a plain-load path on the GPU. There is no
 *     CPU path behind these functions.
 *   - `err` (optional, may be NULL) is a device int the kernel ORs SVLLM_DEVERR_* bits into.
 *     With NULL the library's own per-device word is used; svllm_read_device_error reads it.
 *   - No launch setting can be changed through this ABI: each op's pipeline shape (bytes per
 *     stage, stages, warps per CTA) is a tuned constant. For tuning sweeps the environment
 *     variable SVLLM_PIPELINE="op=unit_bytes:stages:warps[,...]" (op: rms_norm, add_rms_norm,
 *     qk_norm_rope, rope, silu_and_mul, embedding; unit_bytes a multiple of 16, stages 2-16,
 *     warps 1-16; 0 keeps a value) is read once, at the process's first launch; entries that
 *     do not parse or are out of range are ignored. Results do not depend on the shape.
 *
 * Reference interfaces these replace or extend (small-vLLM, paths within its project):
 *   src/ops/rms_norm.h:13            at::Tensor svllm::ops::rms_norm(x, weight, eps)
 *   src/ops/rms_norm_kernels.h:38-40 svllm::ops::cuda_impl::rms_norm(out, x, weight, eps)
 *   src/ops/cuda/rms_norm.cu:103-131 the CUDA launcher this library's calls stand in for
 *   bindings/svllm_ops.cpp:18        the Python binding the op layer above this ABI keeps
 *   src/model/config.h:10-15         Llama3RopeScaling, mirrored by svllm_llama3_scaling
 * The other five ops have no implementation in the reference; they are added in its op
 * convention (one op per src/ops/<op>.{h,cpp}, docs/design-spec.md:28 "Fused CUDA kernels",
 * docs/ROADMAP.md:40 "RoPE with QK-norm", "SiLU-and-mul").
 */
#ifndef SVLLM_KERNELS_H_
#define SVLLM_KERNELS_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without including the CUDA headers. */
struct CUstream_st;
typedef struct CUstream_st* svllm_stream;

typedef enum svllm_status {
  SVLLM_OK = 0,
  SVLLM_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, stride or dtype */
  SVLLM_ERR_TOO_LARGE = 2,        /* sizes exceed the kernel's index range */
  SVLLM_ERR_UNSUPPORTED = 3,      /* a shape the library has no kernel for */
  SVLLM_ERR_LAUNCH = 4,           /* the kernel launch failed */
  SVLLM_ERR_CUDA = 5              /* another CUDA runtime call failed */
} svllm_status;

/* Bits of the device error word. */
#define SVLLM_DEVERR_BAD_INDEX 1    /* an embedding id outside [0, vocab) (its row is zeroed) or a
                                       KV slot past the cache (nothing written) */
#define SVLLM_DEVERR_WAIT_TIMEOUT 2 /* a bulk copy did not land in time: the kernel stopped */

/* Index dtype of positions / token ids. */
typedef enum svllm_index_type { SVLLM_INDEX_I32 = 0, SVLLM_INDEX_I64 = 1 } svllm_index_type;

/* Llama-3 RoPE frequency scaling (rope_type "llama3"); mirrors src/model/config.h:10-15. */
typedef struct svllm_llama3_scaling {
  double factor;
  double low_freq_factor;
  double high_freq_factor;
  int64_t original_max_position_embeddings;
} svllm_llama3_scaling;

/* Returns a static, human-readable name for a status code. */
const char* svllm_status_string(int status);

/* Library version, "0.1.0" (the reference's pyproject.toml:3 version). */
const char* svllm_version(void);

/*
 * RMSNorm.  out = round(round(x * rsqrt(mean(x^2) + eps)) * weight), fp32 sum of squares,
 * round() being the output dtype's rounding (identity for fp32), i.e. the reference's
 * src/ops/cuda/rms_norm.cu:62-95 and src/ops/cpu/rms_norm.cpp:13-44 formula.
 * x, out: [num_rows, hidden] with row strides; weight: [hidden] contiguous.
 * Replaces: svllm::ops::cuda_impl::rms_norm (src/ops/rms_norm_kernels.h:38-40).
 */
int svllm_rms_norm_bf16(void* out, const void* x, const void* weight, int64_t num_rows,
                        int64_t hidden, int64_t out_row_stride, int64_t x_row_stride, float eps,
                        svllm_stream stream);
int svllm_rms_norm_f32(float* out, const float* x, const float* weight, int64_t num_rows,
                       int64_t hidden, int64_t out_row_stride, int64_t x_row_stride, float eps,
                       svllm_stream stream);

/*
 * RMSNorm with the fused residual add, in place (Hugging Face decoder-layer semantics):
 *   residual <- round(x + residual);   x <- rms_norm(residual, weight, eps)
 * x, residual: [num_rows, hidden] with row strides; weight: [hidden].
 * New op in the reference's convention (planned at docs/design-spec.md:28).
 */
int svllm_add_rms_norm_bf16(void* x, void* residual, const void* weight, int64_t num_rows,
                            int64_t hidden, int64_t x_row_stride, int64_t residual_row_stride,
                            float eps, svllm_stream stream);
int svllm_add_rms_norm_f32(float* x, float* residual, const float* weight, int64_t num_rows,
                           int64_t hidden, int64_t x_row_stride, int64_t residual_row_stride,
                           float eps, svllm_stream stream);

/*
 * Qwen3 per-head q/k RMSNorm fused with neox-style rotary embedding, in place.
 *   q: [num_tokens, num_heads, head_dim] (token row stride q_row_stride, heads contiguous)
 *   k: [num_tokens, num_kv_heads, head_dim] (token row stride k_row_stride)
 *   q_weight, k_weight: [head_dim]; positions: [num_tokens] of pos_type.
 *   inv_freq: HOST array of head_dim/2 fp32 inverse frequencies (see svllm_rope_inv_freq); it
 *   is passed to the kernel by value, so the caller may free it when the call returns.
 * Per head: h = round(round(x * rsqrt(mean(x^2) + eps)) * w); then for i < head_dim/2, with
 * a = fp32(pos) * inv_freq[i], c = round(cos a), s = round(sin a):
 *   out[i] = round(round(h[i] * c) - round(h[i + d/2] * s))
 *   out[i + d/2] = round(round(h[i + d/2] * c) + round(h[i] * s))
 * which is Qwen3RMSNorm followed by apply_rotary_pos_emb with bf16 cos/sin. head_dim must be
 * even and at most 512. Flags: src/model/config.h:29 (qk_norm), config.h:27 (rope_theta).
 */
int svllm_qk_norm_rope_bf16(void* q, void* k, const void* q_weight, const void* k_weight,
                            const void* positions, int pos_type, int64_t num_tokens,
                            int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                            int64_t q_row_stride, int64_t k_row_stride, float eps,
                            const float* inv_freq, svllm_stream stream);
int svllm_qk_norm_rope_f32(float* q, float* k, const float* q_weight, const float* k_weight,
                           const void* positions, int pos_type, int64_t num_tokens,
                           int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                           int64_t q_row_stride, int64_t k_row_stride, float eps,
                           const float* inv_freq, svllm_stream stream);

/*
 * Neox-style rotary embedding alone, in place on q and k (Llama: no q/k norm). Same layout,
 * formula and inv_freq convention as svllm_qk_norm_rope_* without the norm.
 * Llama-3 scaling enters only through inv_freq (svllm_rope_inv_freq with a scaling struct).
 */
int svllm_rope_bf16(void* q, void* k, const void* positions, int pos_type, int64_t num_tokens,
                    int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                    int64_t q_row_stride, int64_t k_row_stride, const float* inv_freq,
                    svllm_stream stream);
int svllm_rope_f32(float* q, float* k, const void* positions, int pos_type, int64_t num_tokens,
                   int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                   int64_t q_row_stride, int64_t k_row_stride, const float* inv_freq,
                   svllm_stream stream);

/*
 * The two rotary ops fused with the paged-KV cache write that follows them in a decoder layer
 * (the reference's AGENTS.md names slot_mapping: "per token, the KV slot it writes:
 * block_id * block_size + offset"). Same in-place q/k results as svllm_qk_norm_rope_* /
 * svllm_rope_*, and in the same pass, for every token t with slot s = slot_mapping[t]:
 *   k_cache[s] = the rotated k[t]  ([num_kv_heads, head_dim]),  v_cache[s] = v[t].
 * k_cache, v_cache: [num_slots, num_kv_heads, head_dim] contiguous (a [num_blocks, block_size,
 * num_kv_heads, head_dim] cache with num_slots = num_blocks * block_size); v: [num_tokens,
 * num_kv_heads, head_dim] at row stride v_row_stride (a view of a fused qkv tensor works);
 * slot_mapping: [num_tokens] int64, 8-byte aligned. A negative slot skips the token (padding);
 * a slot >= num_slots writes nothing and raises SVLLM_DEVERR_BAD_INDEX.
 * New op: the next step of the path after RoPE (planned with the paged KV cache,
 * docs/ROADMAP.md:24-25).
 */
int svllm_qk_norm_rope_cache_bf16(void* q, void* k, const void* v, const void* q_weight,
                                  const void* k_weight, const void* positions, int pos_type,
                                  const int64_t* slot_mapping, void* k_cache, void* v_cache,
                                  int64_t num_slots, int64_t num_tokens, int64_t num_heads,
                                  int64_t num_kv_heads, int64_t head_dim, int64_t q_row_stride,
                                  int64_t k_row_stride, int64_t v_row_stride, float eps,
                                  const float* inv_freq, svllm_stream stream);
int svllm_qk_norm_rope_cache_f32(float* q, float* k, const float* v, const float* q_weight,
                                 const float* k_weight, const void* positions, int pos_type,
                                 const int64_t* slot_mapping, float* k_cache, float* v_cache,
                                 int64_t num_slots, int64_t num_tokens, int64_t num_heads,
                                 int64_t num_kv_heads, int64_t head_dim, int64_t q_row_stride,
                                 int64_t k_row_stride, int64_t v_row_stride, float eps,
                                 const float* inv_freq, svllm_stream stream);
int svllm_rope_cache_bf16(void* q, void* k, const void* v, const void* positions, int pos_type,
                          const int64_t* slot_mapping, void* k_cache, void* v_cache,
                          int64_t num_slots, int64_t num_tokens, int64_t num_heads,
                          int64_t num_kv_heads, int64_t head_dim, int64_t q_row_stride,
                          int64_t k_row_stride, int64_t v_row_stride, const float* inv_freq,
                          svllm_stream stream);
int svllm_rope_cache_f32(float* q, float* k, const float* v, const void* positions, int pos_type,
                         const int64_t* slot_mapping, float* k_cache, float* v_cache,
                         int64_t num_slots, int64_t num_tokens, int64_t num_heads,
                         int64_t num_kv_heads, int64_t head_dim, int64_t q_row_stride,
                         int64_t k_row_stride, int64_t v_row_stride, const float* inv_freq,
                         svllm_stream stream);

/*
 * Host helper: the rotary inverse-frequency table, head_dim/2 fp32 values written to the HOST
 * array inv_freq, by Hugging Face's fp32 formula: inv[i] = 1 / powf(theta, fp32(2i) / head_dim)
 * with every step an fp32 operation. With scaling != NULL the Llama-3 rule
 * (src/model/config.h:10-15) follows, also in fp32: wavelength w = 2*pi / inv;
 * w > orig/low_freq_factor -> inv/factor; w < orig/high_freq_factor -> inv; otherwise
 * (1 - s) * inv / factor + s * inv with s = (orig / w - low) / (high - low).
 * torch's fp32 pow and the C library's powf agree on almost every entry; the LibTorch op layer
 * builds the table with torch itself, so that it equals Hugging Face's bit for bit.
 */
int svllm_rope_inv_freq(double theta, int64_t head_dim, const svllm_llama3_scaling* scaling,
                        float* inv_freq);

/*
 * SiLU(gate) * up.  out = round(round(gate / (1 + exp(-gate))) * up).
 * gate, up, out: [num_rows, inter] with row strides (gate and up may be the two halves of one
 * [num_rows, 2 * inter] tensor). New op (docs/ROADMAP.md:40 "SiLU-and-mul").
 */
int svllm_silu_and_mul_bf16(void* out, const void* gate, const void* up, int64_t num_rows,
                            int64_t inter, int64_t out_row_stride, int64_t gate_row_stride,
                            int64_t up_row_stride, svllm_stream stream);
int svllm_silu_and_mul_f32(float* out, const float* gate, const float* up, int64_t num_rows,
                           int64_t inter, int64_t out_row_stride, int64_t gate_row_stride,
                           int64_t up_row_stride, svllm_stream stream);

/*
 * Token-embedding gather, a bit-exact row copy: out[t] = table[ids[t]].
 * ids: [num_tokens] of id_type; table: [vocab_size, hidden] (row stride table_row_stride);
 * out: [num_tokens, hidden] (row stride out_row_stride). An id outside [0, vocab_size) zeroes
 * its output row and raises SVLLM_DEVERR_BAD_INDEX in *err (or the library word); it never
 * faults. The table is model.embed_tokens.weight (tests/cpp/safetensors_test.cpp:161-162);
 * ids are int32 as the tokenizer returns them (src/tokenizer/tokenizer.h:22) or int64.
 */
int svllm_embedding_bf16(void* out, const void* ids, int id_type, const void* table,
                         int64_t num_tokens, int64_t vocab_size, int64_t hidden,
                         int64_t out_row_stride, int64_t table_row_stride, int* err,
                         svllm_stream stream);
int svllm_embedding_f32(float* out, const void* ids, int id_type, const float* table,
                        int64_t num_tokens, int64_t vocab_size, int64_t hidden,
                        int64_t out_row_stride, int64_t table_row_stride, int* err,
                        svllm_stream stream);

/*
 * Greedy sampling: out_ids[r] = argmax over logits[r, 0:vocab] (torch.argmax semantics: the
 * first index of the maximum, a NaN above every number). logits: [num_rows, vocab] at
 * row_stride elements, typically the tied-embedding LM head's output after the final norm
 * (src/model/config.h:28). out_ids: [num_rows] int64, device. Few rows are split over the CTAs
 * of a thread-block cluster and reduced through distributed shared memory.
 * New op (sampling on the GPU, docs/design-spec.md:28-29).
 */
int svllm_argmax_bf16(const void* logits, int64_t num_rows, int64_t vocab, int64_t row_stride,
                      int64_t* out_ids, svllm_stream stream);
int svllm_argmax_f32(const float* logits, int64_t num_rows, int64_t vocab, int64_t row_stride,
                     int64_t* out_ids, svllm_stream stream);

/*
 * Greedy sampling fused with the LM head: out_ids[r] = argmax over n of
 * bf16(sum_k hidden[r, k] * weight[n, k]), the logits never written to memory (tcgen05 GEMM,
 * fp32 accumulation, each logit rounded to bf16 as a bf16 matmul would store it, then
 * torch.argmax semantics). hidden: [num_rows, hidden_size] bf16 at hidden_stride elements;
 * weight: [vocab, hidden_size] bf16 at weight_stride elements (the tied embedding table,
 * src/model/config.h:28); both 16-byte aligned with strides of whole 16 bytes, else
 * SVLLM_ERR_UNSUPPORTED. logits: null, or a [num_rows, vocab] bf16 output at logits_stride
 * elements that also receives the logits. workspace: at least 8 * num_rows bytes, 8-byte
 * aligned, zero on entry and zero again when the call's work completes (so one zeroed buffer
 * serves every call on a stream; calls that overlap on the GPU must not share it).
 * New op (the LM head and sampling on the GPU, docs/design-spec.md:28-29).
 */
int svllm_lm_head_argmax_bf16(const void* hidden, int64_t num_rows, int64_t hidden_size,
                              int64_t hidden_stride, const void* weight, int64_t vocab,
                              int64_t weight_stride, int64_t* out_ids, void* logits,
                              int64_t logits_stride, void* workspace, int64_t workspace_bytes,
                              svllm_stream stream);

/*
 * Decode attention over a paged KV cache (one query token per request): for request b and query
 * head h, out[b, h] = softmax_j(scale * q[b, h] . k_j) v_j over the first seq_lens[b] cached
 * rows of KV head h / (num_heads / num_kv_heads), row j at slot block_tables[b][j / block_size]
 * * block_size + j % block_size of k_cache / v_cache [num_blocks, block_size, num_kv_heads,
 * head_dim]. q: [num_seqs, num_heads, head_dim] at q_token_stride elements per request (a view
 * of the qkv projection); out: [num_seqs, num_heads, head_dim] contiguous; block_tables:
 * [num_seqs, max_blocks] int32; seq_lens: [num_seqs] int32, each at most max_seq_len (which
 * sizes the context split). bf16, fp32 softmax and accumulation. head_dim 64 or 128, up to 8
 * query heads per KV head (a power of two), 16-byte aligned q and caches, else
 * SVLLM_ERR_UNSUPPORTED. A table entry outside the cache raises SVLLM_DEVERR_BAD_INDEX and reads
 * block 0. New op: the reference plans this kernel (docs/ROADMAP.md, decode attention).
 */
int svllm_paged_decode_attention_bf16(void* out, const void* q, int64_t q_token_stride,
                                      const void* k_cache, const void* v_cache,
                                      int64_t num_blocks, int64_t block_size,
                                      const int32_t* block_tables, int64_t max_blocks,
                                      const int32_t* seq_lens, int64_t num_seqs,
                                      int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                                      int64_t max_seq_len, float scale, svllm_stream stream);

/*
 * A linear layer at decode batch sizes: out[r, n] = bf16(sum_k x[r, k] * weight[n, k]) for
 * r < num_rows <= 16 (the weight streamed into tensor-core registers, fp32 accumulation, one
 * rounding to bf16). x: [num_rows, in_features] bf16 at x_stride elements; weight:
 * [out_features, in_features] bf16 at weight_stride elements (a checkpoint's projection, no
 * bias); out: [num_rows, out_features] bf16 at out_stride elements. More than 16 rows,
 * in_features not a multiple of 8, or x or weight not 16-byte aligned with strides of whole 16
 * bytes: SVLLM_ERR_UNSUPPORTED, and the caller's GEMM serves the call. out must not overlap x.
 * The weight is read before the previous kernel in the stream has finished (programmatic
 * dependent launch, when that kernel allows it, as this library's kernels do): it must not be
 * written by the kernel immediately before the call.
 * Replaces, for decode steps, at::linear in the model forward the reference plans (src/model,
 * docs/ROADMAP.md:24-25).
 */
int svllm_decode_linear_bf16(void* out, int64_t out_stride, const void* x, int64_t num_rows,
                             int64_t in_features, int64_t x_stride, const void* weight,
                             int64_t out_features, int64_t weight_stride, svllm_stream stream);

/*
 * svllm_lm_head_argmax_bf16 without a workspace argument, for callers that cannot allocate
 * device memory: a host program driving this C ABI through an FFI with no CUDA allocator of its
 * own, or one whose device memory is all owned by another allocator. It allocates nothing; the
 * per-row scratch is an array inside this library (32 KB per GPU that loads it, held until the
 * process exits), so num_rows is at most 4096 (SVLLM_ERR_TOO_LARGE beyond). The first call on a
 * device looks the array's address up (make that call before any stream capture). Every call
 * shares the array: each clears the rows it uses on its stream before the GEMM, and calls that
 * overlap on the GPU (other streams, other host threads) race on it and must not.
 * No counterpart in the reference: an addition of this library.
 */
int svllm_lm_head_argmax_static_bf16(const void* hidden, int64_t num_rows, int64_t hidden_size,
                                     int64_t hidden_stride, const void* weight, int64_t vocab,
                                     int64_t weight_stride, int64_t* out_ids, void* logits,
                                     int64_t logits_stride, svllm_stream stream);

/*
 * Reads (and with reset != 0 clears) the library's own error word on `device`. Synchronises
 * that device. For validation, not for the hot path.
 */
int svllm_read_device_error(int device, int reset, int* flags);

#ifdef __cplusplus
}
#endif

#endif /* SVLLM_KERNELS_H_ */

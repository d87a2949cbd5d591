/*
 * svllm_oracle.c - CPU restatement of small-vLLM's fused per-layer ops. TEST INFRASTRUCTURE.
 *
 * This file is the oracle: only the tests, the smoke check and bench.py's CPU-baseline leg load
 * it (as oracle/libsvllm_oracle.so, through oracle/oracle.py). Nothing in the product links or
 * calls it; the product's CUDA path fails loudly when its extension is missing.
 *
 * Every function restates the reference's algorithm (or, for the ops the reference lacks, the
 * Hugging Face formula its design commits to, docs/design-spec.md:105-106 "matches PyTorch",
 * "matches Hugging Face") in plain C with OpenMP over rows, one IEEE operation at a time
 * (compiled with -ffp-contract=off, so no multiply-add is fused behind our back):
 *
 *   rms_norm       src/ops/cpu/rms_norm.cpp:13-44 (sum of squares; 1 / sqrt(sum / H + eps);
 *                  normalised value rounded to bf16 before the weight multiply, :38-40).
 *                  The sum of squares is accumulated in double and rounded once to fp32: the
 *                  value every fp32-accumulating kernel approximates, whatever its order.
 *   add_rms_norm   residual' = round(x + residual), then rms_norm(residual') - Hugging Face's
 *                  decoder layer (residual add, then post_attention_layernorm).
 *   qk_norm_rope   Qwen3RMSNorm per head (src/model/config.h:29 qk_norm) then
 *                  apply_rotary_pos_emb with cos/sin rounded to the activation dtype.
 *   rope           apply_rotary_pos_emb alone (Llama, src/model/config.h:10-15 scaling enters
 *                  through inv_freq).
 *   silu_and_mul   round(round(g / (1 + expf(-g))) * u), torch's silu then mul.
 *   embedding      out[t] = table[ids[t]] byte for byte; bad ids give zero rows (counted).
 *   inv_freq       1 / powf(theta, fp32(2i) / D) with the Llama-3 rule in fp32, Hugging Face's
 *                  _compute_default_rope_parameters / _compute_llama3_parameters order.
 *
 * bf16 buffers are uint16_t bit patterns; rounding to bf16 is round-to-nearest-even.
 * Parity is pinned: rms_norm against the reference's own OpenMP kernel built from its sources
 * (oracle/_ref), the other ops against Hugging Face modules run on seeded inputs
 * (tests/golden/make_golden.py writes the fixtures, tests/test_oracle_golden.py checks them).
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <string.h>

#define EXPORT __attribute__((visibility("default")))

static inline float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

/* 1 / sqrt(sum / n + eps) in fp32 with the sum of squares taken in double. */
static inline float inv_rms_bf16(const uint16_t* v, int64_t n, float eps) {
  double ss = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    const double f = bf16_to_f32(v[i]);
    ss += f * f;
  }
  return 1.0f / sqrtf((float)ss / (float)n + eps);
}

static inline float inv_rms_f32(const float* v, int64_t n, float eps) {
  double ss = 0.0;
  for (int64_t i = 0; i < n; ++i) ss += (double)v[i] * (double)v[i];
  return 1.0f / sqrtf((float)ss / (float)n + eps);
}

/* ----------------------------------------------------------------------------------------- */

EXPORT void orc_rms_norm_bf16(uint16_t* out, const uint16_t* x, const uint16_t* w, int64_t rows,
                              int64_t hidden, float eps) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* xr = x + r * hidden;
    uint16_t* orow = out + r * hidden;
    const float inv = inv_rms_bf16(xr, hidden, eps);
    for (int64_t i = 0; i < hidden; ++i) {
      const float n = round_bf16(bf16_to_f32(xr[i]) * inv);
      orow[i] = f32_to_bf16(n * bf16_to_f32(w[i]));
    }
  }
}

EXPORT void orc_rms_norm_f32(float* out, const float* x, const float* w, int64_t rows,
                             int64_t hidden, float eps) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * hidden;
    float* orow = out + r * hidden;
    const float inv = inv_rms_f32(xr, hidden, eps);
    for (int64_t i = 0; i < hidden; ++i) orow[i] = (xr[i] * inv) * w[i];
  }
}

EXPORT void orc_add_rms_norm_bf16(uint16_t* x, uint16_t* residual, const uint16_t* w,
                                  int64_t rows, int64_t hidden, float eps) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    uint16_t* xr = x + r * hidden;
    uint16_t* rr = residual + r * hidden;
    for (int64_t i = 0; i < hidden; ++i) rr[i] = f32_to_bf16(bf16_to_f32(xr[i]) + bf16_to_f32(rr[i]));
    const float inv = inv_rms_bf16(rr, hidden, eps);
    for (int64_t i = 0; i < hidden; ++i) {
      const float n = round_bf16(bf16_to_f32(rr[i]) * inv);
      xr[i] = f32_to_bf16(n * bf16_to_f32(w[i]));
    }
  }
}

EXPORT void orc_add_rms_norm_f32(float* x, float* residual, const float* w, int64_t rows,
                                 int64_t hidden, float eps) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    float* xr = x + r * hidden;
    float* rr = residual + r * hidden;
    for (int64_t i = 0; i < hidden; ++i) rr[i] = xr[i] + rr[i];
    const float inv = inv_rms_f32(rr, hidden, eps);
    for (int64_t i = 0; i < hidden; ++i) xr[i] = (rr[i] * inv) * w[i];
  }
}

/* ----------------------------------------------------------------------------------------- */
/* Rotary embedding. One head of d elements, rotated in place with pairs (i, i + d/2).       */

static inline float position_at(const void* pos, int pos_i64, int64_t t) {
  return pos_i64 ? (float)((const int64_t*)pos)[t] : (float)((const int32_t*)pos)[t];
}

static void rope_head_bf16(uint16_t* h, int64_t d, const float* cb, const float* sb) {
  const int64_t half = d / 2;
  for (int64_t i = 0; i < half; ++i) {
    const float x1 = bf16_to_f32(h[i]);
    const float x2 = bf16_to_f32(h[i + half]);
    const float y1 = round_bf16(x1 * cb[i]) - round_bf16(x2 * sb[i]);
    const float y2 = round_bf16(x2 * cb[i]) + round_bf16(x1 * sb[i]);
    h[i] = f32_to_bf16(y1);
    h[i + half] = f32_to_bf16(y2);
  }
}

static void rope_head_f32(float* h, int64_t d, const float* c, const float* s) {
  const int64_t half = d / 2;
  for (int64_t i = 0; i < half; ++i) {
    const float x1 = h[i];
    const float x2 = h[i + half];
    h[i] = x1 * c[i] - x2 * s[i];
    h[i + half] = x2 * c[i] + x1 * s[i];
  }
}

static void norm_head_bf16(uint16_t* h, int64_t d, const uint16_t* w, float eps) {
  const float inv = inv_rms_bf16(h, d, eps);
  for (int64_t i = 0; i < d; ++i) {
    const float n = round_bf16(bf16_to_f32(h[i]) * inv);
    h[i] = f32_to_bf16(n * bf16_to_f32(w[i]));
  }
}

static void norm_head_f32(float* h, int64_t d, const float* w, float eps) {
  const float inv = inv_rms_f32(h, d, eps);
  for (int64_t i = 0; i < d; ++i) h[i] = (h[i] * inv) * w[i];
}

#define MAX_HALF 256

/* q [T, Hq, D] and k [T, Hk, D] contiguous; qw/kw NULL for rope alone. */
static void qk_rope_bf16(uint16_t* q, uint16_t* k, const uint16_t* qw, const uint16_t* kw,
                         const void* pos, int pos_i64, int64_t T, int64_t hq, int64_t hk,
                         int64_t d, float eps, const float* inv_freq) {
  const int64_t half = d / 2;
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < T; ++t) {
    float cb[MAX_HALF], sb[MAX_HALF];
    const float p = position_at(pos, pos_i64, t);
    for (int64_t i = 0; i < half; ++i) {
      const float a = p * inv_freq[i];
      cb[i] = round_bf16(cosf(a));
      sb[i] = round_bf16(sinf(a));
    }
    for (int64_t h = 0; h < hq; ++h) {
      uint16_t* x = q + (t * hq + h) * d;
      if (qw) norm_head_bf16(x, d, qw, eps);
      rope_head_bf16(x, d, cb, sb);
    }
    for (int64_t h = 0; h < hk; ++h) {
      uint16_t* x = k + (t * hk + h) * d;
      if (kw) norm_head_bf16(x, d, kw, eps);
      rope_head_bf16(x, d, cb, sb);
    }
  }
}

static void qk_rope_f32(float* q, float* k, const float* qw, const float* kw, const void* pos,
                        int pos_i64, int64_t T, int64_t hq, int64_t hk, int64_t d, float eps,
                        const float* inv_freq) {
  const int64_t half = d / 2;
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < T; ++t) {
    float c[MAX_HALF], s[MAX_HALF];
    const float p = position_at(pos, pos_i64, t);
    for (int64_t i = 0; i < half; ++i) {
      const float a = p * inv_freq[i];
      c[i] = cosf(a);
      s[i] = sinf(a);
    }
    for (int64_t h = 0; h < hq; ++h) {
      float* x = q + (t * hq + h) * d;
      if (qw) norm_head_f32(x, d, qw, eps);
      rope_head_f32(x, d, c, s);
    }
    for (int64_t h = 0; h < hk; ++h) {
      float* x = k + (t * hk + h) * d;
      if (kw) norm_head_f32(x, d, kw, eps);
      rope_head_f32(x, d, c, s);
    }
  }
}

EXPORT int orc_qk_norm_rope_bf16(uint16_t* q, uint16_t* k, const uint16_t* qw, const uint16_t* kw,
                                 const void* pos, int pos_i64, int64_t T, int64_t hq, int64_t hk,
                                 int64_t d, float eps, const float* inv_freq) {
  if (d <= 0 || d % 2 || d / 2 > MAX_HALF) return 1;
  qk_rope_bf16(q, k, qw, kw, pos, pos_i64, T, hq, hk, d, eps, inv_freq);
  return 0;
}

EXPORT int orc_qk_norm_rope_f32(float* q, float* k, const float* qw, const float* kw,
                                const void* pos, int pos_i64, int64_t T, int64_t hq, int64_t hk,
                                int64_t d, float eps, const float* inv_freq) {
  if (d <= 0 || d % 2 || d / 2 > MAX_HALF) return 1;
  qk_rope_f32(q, k, qw, kw, pos, pos_i64, T, hq, hk, d, eps, inv_freq);
  return 0;
}

EXPORT int orc_rope_bf16(uint16_t* q, uint16_t* k, const void* pos, int pos_i64, int64_t T,
                         int64_t hq, int64_t hk, int64_t d, const float* inv_freq) {
  if (d <= 0 || d % 2 || d / 2 > MAX_HALF) return 1;
  qk_rope_bf16(q, k, NULL, NULL, pos, pos_i64, T, hq, hk, d, 0.0f, inv_freq);
  return 0;
}

EXPORT int orc_rope_f32(float* q, float* k, const void* pos, int pos_i64, int64_t T, int64_t hq,
                        int64_t hk, int64_t d, const float* inv_freq) {
  if (d <= 0 || d % 2 || d / 2 > MAX_HALF) return 1;
  qk_rope_f32(q, k, NULL, NULL, pos, pos_i64, T, hq, hk, d, 0.0f, inv_freq);
  return 0;
}

/*
 * Hugging Face's inverse frequencies in fp32; factor <= 0 means no Llama-3 rule. torch evaluates
 * `scalar / tensor` as reciprocal(tensor) * scalar and `tensor / scalar` as a true division; the
 * steps below follow that, one fp32 operation each.
 */
EXPORT int orc_inv_freq(double theta, int64_t d, double factor, double low_ff, double high_ff,
                        int64_t orig_max, float* out) {
  if (d <= 0 || d % 2) return 1;
  const float base = (float)theta;
  for (int64_t i = 0; i < d / 2; ++i) {
    const float e = (float)(2 * i) / (float)d;
    out[i] = 1.0f / powf(base, e);
  }
  if (factor > 0.0) {
    const float f = (float)factor;
    const float lo = (float)low_ff;
    const float old_len = (float)orig_max;
    const float low_wavelen = (float)((double)orig_max / low_ff);
    const float high_wavelen = (float)((double)orig_max / high_ff);
    const float two_pi = (float)(2.0 * 3.14159265358979323846);
    const float span = (float)(high_ff - low_ff);
    for (int64_t i = 0; i < d / 2; ++i) {
      const float inv = out[i];
      const float wavelen = (1.0f / inv) * two_pi;
      const float inv_llama = wavelen > low_wavelen ? inv / f : inv;
      const float smooth = ((1.0f / wavelen) * old_len - lo) / span;
      const float smoothed = (1.0f - smooth) * inv_llama / f + smooth * inv_llama;
      const int medium = !(wavelen < high_wavelen) && !(wavelen > low_wavelen);
      out[i] = medium ? smoothed : inv_llama;
    }
  }
  return 0;
}

/* ----------------------------------------------------------------------------------------- */

EXPORT void orc_silu_and_mul_bf16(uint16_t* out, const uint16_t* gate, const uint16_t* up,
                                  int64_t rows, int64_t inter) {
  const int64_t n = rows * inter;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float g = bf16_to_f32(gate[i]);
    const float s = round_bf16(g / (1.0f + expf(-g)));
    out[i] = f32_to_bf16(s * bf16_to_f32(up[i]));
  }
}

EXPORT void orc_silu_and_mul_f32(float* out, const float* gate, const float* up, int64_t rows,
                                 int64_t inter) {
  const int64_t n = rows * inter;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float g = gate[i];
    out[i] = (g / (1.0f + expf(-g))) * up[i];
  }
}

/* Returns the number of ids outside [0, vocab); their rows are zero. */
EXPORT int64_t orc_embedding(void* out, const void* ids, int ids_i64, const void* table,
                             int64_t T, int64_t vocab, int64_t row_bytes) {
  int64_t bad = 0;
#pragma omp parallel for schedule(static) reduction(+ : bad)
  for (int64_t t = 0; t < T; ++t) {
    const int64_t id = ids_i64 ? ((const int64_t*)ids)[t] : (int64_t)((const int32_t*)ids)[t];
    char* dst = (char*)out + t * row_bytes;
    if (id < 0 || id >= vocab) {
      memset(dst, 0, (size_t)row_bytes);
      ++bad;
    } else {
      memcpy(dst, (const char*)table + id * row_bytes, (size_t)row_bytes);
    }
  }
  return bad;
}

/* Threads of the OpenMP loops above (the CPU baseline sets it to the cores it reports, whatever
   OMP_NUM_THREADS the launcher exported). Returns the count now in force. */
EXPORT int orc_set_num_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
}

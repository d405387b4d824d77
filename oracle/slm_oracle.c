/*
 * CPU oracle for the KV-cache hot path of small-lm-rs (rust/engine).
 *
 * TEST INFRASTRUCTURE ONLY: a plain-C restatement of the reference's CPU
 * arithmetic, used by tests/, the smoke check and the bench's CPU-baseline
 * leg as the checker. The product never links or calls it.
 *
 * Every function names the reference lines it restates. Operation order,
 * accumulation order, initial values and error checks follow those lines;
 * the Rust bounds-checked slice lookups become direct index arithmetic after
 * the same up-front validation.
 *
 * Build: gcc -O2 -std=c11 -ffp-contract=off -fno-fast-math -fopenmp (see
 * oracle/Makefile). -ffp-contract=off matters: Rust does not fuse `a*b - c*d`.
 */
#include "slm_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* linear.rs:14-23 — round-to-nearest-even to bf16, returned as f32.        */
/* ------------------------------------------------------------------------ */
float orc_round_to_bfloat16(float value) {
  if (!isfinite(value)) return value;
  uint32_t bits;
  memcpy(&bits, &value, 4);
  uint32_t lsb = (bits >> 16) & 1u;
  uint32_t rounded = bits + (0x7fffu + lsb); /* wrapping_add */
  rounded &= 0xffff0000u;
  float out;
  memcpy(&out, &rounded, 4);
  return out;
}

/* ------------------------------------------------------------------------ */
/* RoPE                                                                      */
/* ------------------------------------------------------------------------ */

/* rope.rs:21-43; inverse frequencies at :33-36:
 *   denominator = head_dimension as f32
 *   inv[pair]   = theta.powf(-(2.0 * pair as f32) / denominator)           */
int orc_rope_inverse_frequencies(int32_t head_dim, float theta, float* out) {
  if (head_dim <= 0 || head_dim % 2 != 0) return ORC_ERR_INVALID_CONFIGURATION;
  if (!isfinite(theta) || theta <= 0.0f) return ORC_ERR_INVALID_CONFIGURATION;
  float denominator = (float)head_dim;
  for (int32_t pair = 0; pair < head_dim / 2; ++pair) {
    float exponent = -(2.0f * (float)pair) / denominator;
    out[pair] = powf(theta, exponent);
  }
  return ORC_OK;
}

/* rope.rs:82-100 — interleaved (even, odd) pairs:
 *   angle = (position as f32) * inv;  (sin, cos) = angle.sin_cos()
 *   even' = even*cos - odd*sin;       odd' = even*sin + odd*cos            */
int orc_rope_apply_head(float* head, int32_t head_dim, const float* inv_freq,
                        int64_t position) {
  if (head_dim <= 0 || head_dim % 2 != 0) return ORC_ERR_INVALID_INPUT;
  float pos = (float)position;
  for (int32_t pair = 0; pair < head_dim / 2; ++pair) {
    float angle = pos * inv_freq[pair];
    float s = sinf(angle);
    float c = cosf(angle);
    float even = head[2 * pair];
    float odd = head[2 * pair + 1];
    float a = even * c;
    float b = odd * s;
    head[2 * pair] = a - b;
    float e = even * s;
    float f = odd * c;
    head[2 * pair + 1] = e + f;
  }
  return ORC_OK;
}

/* rope.rs:108-134 */
int orc_rope_apply_heads(float* values, int32_t num_heads, int32_t head_dim,
                         const float* inv_freq, int64_t position) {
  if (num_heads <= 0) return ORC_ERR_INVALID_INPUT;
  for (int32_t h = 0; h < num_heads; ++h) {
    int rc = orc_rope_apply_head(values + (int64_t)h * head_dim, head_dim,
                                 inv_freq, position);
    if (rc) return rc;
  }
  return ORC_OK;
}

/* attention.rs:422-482 — token t of the batch sits at absolute position
 * position_offset + t; query heads first, then key heads (V untouched). */
int orc_apply_rotary_with_offset(float* query, float* key, int64_t tokens,
                                 int32_t q_heads, int32_t kv_heads,
                                 int32_t head_dim, const float* inv_freq,
                                 int64_t position_offset) {
  int64_t qs = (int64_t)q_heads * head_dim;
  int64_t ks = (int64_t)kv_heads * head_dim;
  for (int64_t t = 0; t < tokens; ++t) {
    int64_t pos = position_offset + t;
    int rc = orc_rope_apply_heads(query + t * qs, q_heads, head_dim, inv_freq, pos);
    if (rc) return rc;
    rc = orc_rope_apply_heads(key + t * ks, kv_heads, head_dim, inv_freq, pos);
    if (rc) return rc;
  }
  return ORC_OK;
}

/* ------------------------------------------------------------------------ */
/* softmax.rs:12-45                                                          */
/* ------------------------------------------------------------------------ */
int orc_softmax_in_place(float* values, int64_t n) {
  if (n <= 0) return ORC_ERR_INVALID_INPUT;
  for (int64_t i = 0; i < n; ++i)
    if (!isfinite(values[i])) return ORC_ERR_INVALID_INPUT;
  float maximum = -INFINITY; /* fold(f32::NEG_INFINITY, f32::max) */
  for (int64_t i = 0; i < n; ++i) maximum = fmaxf(maximum, values[i]);
  float sum = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    values[i] = expf(values[i] - maximum);
    sum += values[i];
  }
  if (!isfinite(sum) || sum <= 0.0f) return ORC_ERR_INVALID_INPUT;
  for (int64_t i = 0; i < n; ++i) values[i] /= sum;
  return ORC_OK;
}

/* softmax.rs:53-59 */
int orc_softmax_rows(float* values, int64_t rows, int64_t columns) {
  if (rows <= 0 || columns <= 0) return ORC_ERR_INVALID_INPUT;
  for (int64_t r = 0; r < rows; ++r) {
    int rc = orc_softmax_in_place(values + r * columns, columns);
    if (rc) return rc;
  }
  return ORC_OK;
}

/* ------------------------------------------------------------------------ */
/* Dense KV cache — kv_cache.rs:66-412                                        */
/* ------------------------------------------------------------------------ */
struct orc_cache {
  int32_t num_layers;
  int32_t max_sequence_length;
  int32_t kv_heads;
  int32_t head_dim;
  int32_t quantize_bf16;
  int64_t* lengths; /* per layer */
  float* keys;      /* [layers][max_seq][kv_heads][d] */
  float* values;
};

/* kv_cache.rs:43-55, 101-116 */
orc_cache* orc_cache_allocate(int32_t num_layers, int32_t max_sequence_length,
                              int32_t kv_heads, int32_t head_dim,
                              int32_t quantize_bf16) {
  if (num_layers <= 0 || max_sequence_length <= 0 || kv_heads <= 0 || head_dim <= 0)
    return NULL;
  orc_cache* c = (orc_cache*)calloc(1, sizeof(orc_cache));
  if (!c) return NULL;
  c->num_layers = num_layers;
  c->max_sequence_length = max_sequence_length;
  c->kv_heads = kv_heads;
  c->head_dim = head_dim;
  c->quantize_bf16 = quantize_bf16;
  size_t per_layer = (size_t)max_sequence_length * kv_heads * head_dim;
  c->lengths = (int64_t*)calloc((size_t)num_layers, sizeof(int64_t));
  c->keys = (float*)calloc(per_layer * num_layers, sizeof(float));
  c->values = (float*)calloc(per_layer * num_layers, sizeof(float));
  if (!c->lengths || !c->keys || !c->values) {
    orc_cache_free(c);
    return NULL;
  }
  return c;
}

void orc_cache_free(orc_cache* c) {
  if (!c) return;
  free(c->lengths);
  free(c->keys);
  free(c->values);
  free(c);
}

static size_t layer_base(const orc_cache* c, int32_t layer) {
  return (size_t)layer * c->max_sequence_length * c->kv_heads * c->head_dim;
}

/* kv_cache.rs:182-230 — validate shape, reject non-finite (:192-197), check
 * capacity (:203-211), then copy at [len*W, (len+T)*W) and grow the length.
 * Validation completes before storage is mutated. */
int orc_cache_append_layer(orc_cache* c, int32_t layer, const float* keys,
                           const float* values, int64_t token_count) {
  if (token_count <= 0) return ORC_ERR_INVALID_INPUT; /* validate_matrix */
  int64_t width = (int64_t)c->kv_heads * c->head_dim;
  int64_t n = token_count * width;
  for (int64_t i = 0; i < n; ++i)
    if (!isfinite(keys[i])) return ORC_ERR_NON_FINITE;
  for (int64_t i = 0; i < n; ++i)
    if (!isfinite(values[i])) return ORC_ERR_NON_FINITE;
  if (layer < 0 || layer >= c->num_layers) return ORC_ERR_INVALID_INPUT;
  int64_t current = c->lengths[layer];
  int64_t new_length = current + token_count;
  if (new_length > c->max_sequence_length) return ORC_ERR_CAPACITY;
  float* kd = c->keys + layer_base(c, layer) + current * width;
  float* vd = c->values + layer_base(c, layer) + current * width;
  if (c->quantize_bf16) {
    for (int64_t i = 0; i < n; ++i) kd[i] = orc_round_to_bfloat16(keys[i]);
    for (int64_t i = 0; i < n; ++i) vd[i] = orc_round_to_bfloat16(values[i]);
  } else {
    memcpy(kd, keys, (size_t)n * sizeof(float));
    memcpy(vd, values, (size_t)n * sizeof(float));
  }
  c->lengths[layer] = new_length;
  return ORC_OK;
}

/* kv_cache.rs:157-170 */
int64_t orc_cache_layer_sequence_length(const orc_cache* c, int32_t layer) {
  if (layer < 0 || layer >= c->num_layers) return ORC_ERR_INVALID_INPUT;
  return c->lengths[layer];
}

/* kv_cache.rs:129-135 — minimum over layers */
int64_t orc_cache_sequence_length(const orc_cache* c) {
  int64_t m = c->lengths[0];
  for (int32_t l = 1; l < c->num_layers; ++l)
    if (c->lengths[l] < m) m = c->lengths[l];
  return m;
}

/* kv_cache.rs:139-141 */
int32_t orc_cache_is_empty(const orc_cache* c) {
  for (int32_t l = 0; l < c->num_layers; ++l)
    if (c->lengths[l] != 0) return 0;
  return 1;
}

/* kv_cache.rs:145-150 */
int32_t orc_cache_is_synchronized(const orc_cache* c) {
  int64_t e = orc_cache_sequence_length(c);
  for (int32_t l = 0; l < c->num_layers; ++l)
    if (c->lengths[l] != e) return 0;
  return 1;
}

/* kv_cache.rs:285-293 — capacity after the longest layer, saturating */
int64_t orc_cache_remaining_capacity(const orc_cache* c) {
  int64_t used = 0;
  for (int32_t l = 0; l < c->num_layers; ++l)
    if (c->lengths[l] > used) used = c->lengths[l];
  int64_t rem = (int64_t)c->max_sequence_length - used;
  return rem > 0 ? rem : 0;
}

/* kv_cache.rs:302-321 — transactional: fails unless every layer >= target */
int orc_cache_truncate_all(orc_cache* c, int64_t sequence_length) {
  for (int32_t l = 0; l < c->num_layers; ++l)
    if (c->lengths[l] < sequence_length) return ORC_ERR_INVALID_INPUT;
  for (int32_t l = 0; l < c->num_layers; ++l) c->lengths[l] = sequence_length;
  return ORC_OK;
}

/* kv_cache.rs:323-346 */
int orc_cache_truncate_layer(orc_cache* c, int32_t layer, int64_t sequence_length) {
  if (layer < 0 || layer >= c->num_layers) return ORC_ERR_INVALID_INPUT;
  if (sequence_length > c->lengths[layer] || sequence_length < 0)
    return ORC_ERR_INVALID_INPUT;
  c->lengths[layer] = sequence_length;
  return ORC_OK;
}

/* kv_cache.rs:296-300 */
void orc_cache_clear(orc_cache* c) {
  for (int32_t l = 0; l < c->num_layers; ++l) c->lengths[l] = 0;
}

/* kv_cache.rs:237-248, 348-364 */
static int layer_prefix(const orc_cache* c, int32_t layer, int keys, float* out) {
  if (layer < 0 || layer >= c->num_layers) return ORC_ERR_INVALID_INPUT;
  size_t n = (size_t)c->lengths[layer] * c->kv_heads * c->head_dim;
  const float* src = (keys ? c->keys : c->values) + layer_base(c, layer);
  memcpy(out, src, n * sizeof(float));
  return ORC_OK;
}
int orc_cache_layer_keys(const orc_cache* c, int32_t layer, float* out) {
  return layer_prefix(c, layer, 1, out);
}
int orc_cache_layer_values(const orc_cache* c, int32_t layer, float* out) {
  return layer_prefix(c, layer, 0, out);
}

/* kv_cache.rs:366-411 */
static const float* head_slice(const orc_cache* c, int32_t layer, int64_t pos,
                               int32_t kvh, int keys) {
  if (layer < 0 || layer >= c->num_layers) return NULL;
  if (pos < 0 || pos >= c->lengths[layer]) return NULL;
  if (kvh < 0 || kvh >= c->kv_heads) return NULL;
  int64_t width = (int64_t)c->kv_heads * c->head_dim;
  const float* base = (keys ? c->keys : c->values) + layer_base(c, layer);
  return base + pos * width + (int64_t)kvh * c->head_dim;
}
int orc_cache_key_head(const orc_cache* c, int32_t layer, int64_t position,
                       int32_t kv_head, float* out) {
  const float* p = head_slice(c, layer, position, kv_head, 1);
  if (!p) return ORC_ERR_INVALID_INPUT;
  memcpy(out, p, (size_t)c->head_dim * sizeof(float));
  return ORC_OK;
}
int orc_cache_value_head(const orc_cache* c, int32_t layer, int64_t position,
                         int32_t kv_head, float* out) {
  const float* p = head_slice(c, layer, position, kv_head, 0);
  if (!p) return ORC_ERR_INVALID_INPUT;
  memcpy(out, p, (size_t)c->head_dim * sizeof(float));
  return ORC_OK;
}

/* ------------------------------------------------------------------------ */
/* Cached decode attention — attention.rs:677-759                             */
/* ------------------------------------------------------------------------ */
int orc_attend_cached_query(const orc_cache* c, int32_t layer,
                            const float* query, int32_t q_heads, float* out) {
  if (layer < 0 || layer >= c->num_layers) return ORC_ERR_INVALID_INPUT;
  if (q_heads <= 0 || q_heads % c->kv_heads != 0) return ORC_ERR_INVALID_INPUT;
  int64_t L = c->lengths[layer];
  if (L == 0) return ORC_ERR_INVALID_INPUT; /* :690-695 */
  const int32_t d = c->head_dim;
  const int32_t group = q_heads / c->kv_heads;
  float* probs = (float*)malloc((size_t)q_heads * (size_t)L * sizeof(float));
  if (!probs) return ORC_ERR_INVALID_INPUT;
  const float scale = 1.0f / sqrtf((float)d); /* (d as f32).sqrt().recip() */
  /* scores: :706-730 — dot = fold(0, q.mul_add(k, sum)); score = dot*scale */
  for (int32_t h = 0; h < q_heads; ++h) {
    const float* q = query + (int64_t)h * d;
    int32_t kvh = h / group; /* :718 */
    for (int64_t s = 0; s < L; ++s) {
      const float* k = head_slice(c, layer, s, kvh, 1);
      float dot = 0.0f;
      for (int32_t i = 0; i < d; ++i) dot = fmaf(q[i], k[i], dot);
      probs[(int64_t)h * L + s] = dot * scale;
    }
  }
  int rc = orc_softmax_rows(probs, q_heads, L); /* :731 */
  if (rc) {
    free(probs);
    return rc;
  }
  /* values: :733-757 — out = fold_s value.mul_add(p, out), starting at 0 */
  for (int32_t h = 0; h < q_heads; ++h) {
    float* o = out + (int64_t)h * d;
    for (int32_t i = 0; i < d; ++i) o[i] = 0.0f;
    int32_t kvh = h / group; /* :749 */
    const float* prow = probs + (int64_t)h * L;
    for (int64_t s = 0; s < L; ++s) {
      const float* v = head_slice(c, layer, s, kvh, 0);
      float p = prow[s];
      for (int32_t i = 0; i < d; ++i) o[i] = fmaf(v[i], p, o[i]);
    }
  }
  free(probs);
  return ORC_OK;
}

/* attention.rs:794-816 — position = pre-append layer length; RoPE on Q and K
 * (:802), append (:803-808), attend (:810); on attention failure the layer is
 * truncated back to its original length (:814). */
int orc_forward_cached_attention(orc_cache* c, int32_t layer, float* query,
                                 float* key, const float* value,
                                 int32_t q_heads, const float* inv_freq,
                                 float* out) {
  if (layer < 0 || layer >= c->num_layers) return ORC_ERR_INVALID_INPUT;
  int64_t pos = c->lengths[layer];
  int rc = orc_apply_rotary_with_offset(query, key, 1, q_heads, c->kv_heads,
                                        c->head_dim, inv_freq, pos);
  if (rc) return rc;
  rc = orc_cache_append_layer(c, layer, key, value, 1);
  if (rc) return rc;
  rc = orc_attend_cached_query(c, layer, query, q_heads, out);
  if (rc) {
    orc_cache_truncate_layer(c, layer, pos);
    return rc;
  }
  return ORC_OK;
}

int orc_forward_cached_attention_batch(orc_cache** caches, int32_t n,
                                       int32_t layer, float* query, float* key,
                                       const float* value, int32_t q_heads,
                                       const float* inv_freq, float* out,
                                       int32_t threads) {
  if (n <= 0) return ORC_ERR_INVALID_INPUT;
  const int32_t kvh = caches[0]->kv_heads, d = caches[0]->head_dim;
  const int64_t qs = (int64_t)q_heads * d, ks = (int64_t)kvh * d;
  int first_error = ORC_OK;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1)
#endif
  for (int32_t i = 0; i < n; ++i) {
    int rc = orc_forward_cached_attention(caches[i], layer, query + i * qs,
                                          key + i * ks, value + i * ks, q_heads,
                                          inv_freq, out + i * qs);
    if (rc) {
#ifdef _OPENMP
#pragma omp critical
#endif
      if (first_error == ORC_OK) first_error = rc;
    }
  }
  (void)threads;
  return first_error;
}

/* ------------------------------------------------------------------------ */
/* Prefill causal attention — attention.rs:195-399                            */
/* ------------------------------------------------------------------------ */

/* attention.rs:195-245 */
int orc_scaled_causal_scores(const float* query, const float* key,
                             int64_t T, int32_t q_heads, int32_t kv_heads,
                             int32_t d, float* scores) {
  if (T <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads)
    return ORC_ERR_INVALID_INPUT;
  const int32_t group = q_heads / kv_heads;
  const float scale = 1.0f / sqrtf((float)d);
  int64_t count = (int64_t)q_heads * T * T;
  for (int64_t i = 0; i < count; ++i) scores[i] = -FLT_MAX; /* f32::MIN */
  for (int32_t h = 0; h < q_heads; ++h) {
    int32_t kvh = h / group; /* :121-132 */
    for (int64_t qp = 0; qp < T; ++qp) {
      const float* q = query + (qp * q_heads + h) * (int64_t)d;
      int64_t row = ((int64_t)h * T + qp) * T;
      for (int64_t sp = 0; sp <= qp; ++sp) {
        const float* k = key + (sp * kv_heads + kvh) * (int64_t)d;
        float dot = 0.0f;
        for (int32_t i = 0; i < d; ++i) dot = fmaf(q[i], k[i], dot);
        scores[row + sp] = dot * scale;
      }
    }
  }
  return ORC_OK;
}

/* attention.rs:256-269 */
int orc_causal_probabilities(const float* query, const float* key, int64_t T,
                             int32_t q_heads, int32_t kv_heads, int32_t d,
                             float* probabilities) {
  int rc = orc_scaled_causal_scores(query, key, T, q_heads, kv_heads, d, probabilities);
  if (rc) return rc;
  return orc_softmax_rows(probabilities, (int64_t)q_heads * T, T);
}

/* attention.rs:282-399 — out[t][h] = fold_s value.mul_add(p, out) */
int orc_attend_values(const float* probabilities, const float* value,
                      int64_t T, int32_t q_heads, int32_t kv_heads, int32_t d,
                      float* out) {
  if (T <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads)
    return ORC_ERR_INVALID_INPUT;
  int64_t count = (int64_t)q_heads * T * T;
  for (int64_t i = 0; i < count; ++i)
    if (!isfinite(probabilities[i]) || probabilities[i] < 0.0f)
      return ORC_ERR_INVALID_INPUT; /* :298-306 */
  const int32_t group = q_heads / kv_heads;
  for (int64_t qp = 0; qp < T; ++qp) {
    for (int32_t h = 0; h < q_heads; ++h) {
      int32_t kvh = h / group;
      const float* prow = probabilities + ((int64_t)h * T + qp) * T;
      float* o = out + (qp * q_heads + h) * (int64_t)d;
      for (int32_t i = 0; i < d; ++i) o[i] = 0.0f;
      for (int64_t sp = 0; sp < T; ++sp) {
        const float* v = value + (sp * kv_heads + kvh) * (int64_t)d;
        float p = prow[sp];
        for (int32_t i = 0; i < d; ++i) o[i] = fmaf(v[i], p, o[i]);
      }
    }
  }
  return ORC_OK;
}

/* ------------------------------------------------------------------------ */
/* Projections — linear.rs:44-152 (output elements are independent, so      */
/* spreading them over threads, as Rayon does, cannot change any value).     */
/* ------------------------------------------------------------------------ */
int orc_linear(const float* input, int64_t rows, int64_t in_features,
               const float* weight, int64_t out_features, float* out,
               int32_t threads) {
  if (rows <= 0 || in_features <= 0 || out_features <= 0) return ORC_ERR_INVALID_INPUT;
  float* ri = (float*)malloc((size_t)(rows * in_features) * sizeof(float));
  float* rw = (float*)malloc((size_t)(out_features * in_features) * sizeof(float));
  if (!ri || !rw) {
    free(ri);
    free(rw);
    return ORC_ERR_INVALID_INPUT;
  }
  for (int64_t i = 0; i < rows * in_features; ++i) ri[i] = orc_round_to_bfloat16(input[i]);
  for (int64_t i = 0; i < out_features * in_features; ++i)
    rw[i] = orc_round_to_bfloat16(weight[i]);
  int64_t total = rows * out_features;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
#endif
  for (int64_t flat = 0; flat < total; ++flat) {
    int64_t r = flat / out_features, o = flat % out_features;
    const float* x = ri + r * in_features;
    const float* w = rw + o * in_features;
    float sum = 0.0f;
    for (int64_t i = 0; i < in_features; ++i) sum = fmaf(x[i], w[i], sum);
    out[flat] = sum;
  }
  free(ri);
  free(rw);
  (void)threads;
  return ORC_OK;
}

int orc_linear_fp32(const float* input, int64_t rows, int64_t in_features,
                    const float* weight, int64_t out_features, float* out,
                    int32_t threads) {
  if (rows <= 0 || in_features <= 0 || out_features <= 0) return ORC_ERR_INVALID_INPUT;
  int64_t total = rows * out_features;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
#endif
  for (int64_t flat = 0; flat < total; ++flat) {
    int64_t r = flat / out_features, o = flat % out_features;
    const float* x = input + r * in_features;
    const float* w = weight + o * in_features;
    float sum = 0.0f;
    for (int64_t i = 0; i < in_features; ++i) sum = fmaf(x[i], w[i], sum);
    out[flat] = sum;
  }
  (void)threads;
  return ORC_OK;
}

int32_t orc_max_threads(void) {
#ifdef _OPENMP
  return (int32_t)omp_get_max_threads();
#else
  return 1;
#endif
}

/* ---- model-level functions -------------------------------------------- */

/* rmsnorm.rs:80-91 */
int orc_rmsnorm_rows(const float* input, int64_t rows, int64_t hidden,
                     const float* weight, float epsilon, float* out) {
  if (rows <= 0 || hidden <= 0) return ORC_ERR_INVALID_INPUT;
  const float width = (float)hidden;
  for (int64_t r = 0; r < rows; ++r) {
    const float* x = input + r * hidden;
    float square_sum = 0.0f;
    for (int64_t i = 0; i < hidden; ++i) square_sum = fmaf(x[i], x[i], square_sum);
    const float inverse_rms = 1.0f / sqrtf(square_sum / width + epsilon);
    for (int64_t i = 0; i < hidden; ++i) out[r * hidden + i] = x[i] * inverse_rms * weight[i];
  }
  return ORC_OK;
}

/* situ_glu.rs:131-138 */
static float orc_sigmoid(float value) {
  if (value >= 0.0f) return 1.0f / (1.0f + expf(-value));
  const float e = expf(value);
  return e / (1.0f + e);
}
/* situ_glu.rs:59-62 */
float orc_situ_gate_activation(float value, float beta_gate) {
  return beta_gate * tanhf(value / beta_gate) * orc_sigmoid(value);
}
/* situ_glu.rs:64-67 */
float orc_situ_up_activation(float value, float beta_up) {
  return beta_up * tanhf(value / beta_up);
}

/* situ_glu.rs:80-128 */
int orc_situ_glu(const float* input, int64_t rows, int64_t hidden,
                 int64_t intermediate, const float* gate_weight,
                 const float* up_weight, const float* down_weight,
                 float beta_gate, float beta_up, float* out, int32_t threads) {
  if (rows <= 0 || hidden <= 0 || intermediate <= 0) return ORC_ERR_INVALID_INPUT;
  const size_t n = (size_t)(rows * intermediate);
  float* gate = (float*)malloc(n * sizeof(float));
  float* up = (float*)malloc(n * sizeof(float));
  int rc = (gate && up) ? ORC_OK : ORC_ERR_INVALID_INPUT;
  if (rc == ORC_OK) rc = orc_linear(input, rows, hidden, gate_weight, intermediate, gate, threads);
  if (rc == ORC_OK) rc = orc_linear(input, rows, hidden, up_weight, intermediate, up, threads);
  if (rc == ORC_OK) {
    for (size_t i = 0; i < n; ++i)
      gate[i] = orc_situ_gate_activation(gate[i], beta_gate) * orc_situ_up_activation(up[i], beta_up);
    rc = orc_linear(gate, rows, intermediate, down_weight, hidden, out, threads);
  }
  free(gate);
  free(up);
  return rc;
}

/* embedding.rs:15-56 */
int orc_embedding_lookup(const uint32_t* token_ids, int64_t n, const float* table,
                         int64_t vocab, int64_t hidden, float* out) {
  if (n <= 0 || vocab <= 0 || hidden <= 0) return ORC_ERR_INVALID_INPUT;
  for (int64_t t = 0; t < n; ++t) {
    if ((int64_t)token_ids[t] >= vocab) return ORC_ERR_INVALID_INPUT;
    memcpy(out + t * hidden, table + (int64_t)token_ids[t] * hidden, (size_t)hidden * sizeof(float));
  }
  return ORC_OK;
}

/* greedy.rs: argmax_finite */
int orc_argmax_finite(const float* logits, int64_t n, uint32_t* out) {
  if (n <= 0) return ORC_ERR_INVALID_INPUT;
  for (int64_t i = 0; i < n; ++i)
    if (!isfinite(logits[i])) return ORC_ERR_INVALID_INPUT;
  int64_t best = 0;
  float best_value = logits[0];
  for (int64_t i = 1; i < n; ++i)
    if (logits[i] > best_value) {
      best = i;
      best_value = logits[i];
    }
  *out = (uint32_t)best;
  return ORC_OK;
}

int32_t orc_model_tensor_count(int32_t num_layers) { return 2 + 9 * num_layers; }

/* transformer.rs:183-204 (ffn_residual) and :296-311 (add_residual_in_place):
 * x += down(situ(norm(x))). */
static int orc_ffn_residual(const orc_model_config* cfg, const float* const* lt, float* x,
                            int64_t rows, float* scratch_norm, float* scratch_out,
                            int32_t threads) {
  const int64_t H = cfg->hidden_size;
  int rc = orc_rmsnorm_rows(x, rows, H, lt[5], cfg->rms_norm_epsilon, scratch_norm);
  if (rc == ORC_OK)
    rc = orc_situ_glu(scratch_norm, rows, H, cfg->intermediate_size, lt[6], lt[7], lt[8],
                      cfg->situ_beta_gate, cfg->situ_beta_up, scratch_out, threads);
  if (rc == ORC_OK)
    for (int64_t i = 0; i < rows * H; ++i) x[i] += scratch_out[i];
  return rc;
}

/* model.rs:206-227 (final norm) and :193-205 (tied fp32 vocabulary projection) */
static int orc_final_logits(const orc_model_config* cfg, const float* const* tensors,
                            const float* x, int64_t rows, float* scratch, float* logits,
                            int32_t threads) {
  const int64_t H = cfg->hidden_size;
  int rc = orc_rmsnorm_rows(x, rows, H, tensors[1 + 9 * cfg->num_layers], cfg->rms_norm_epsilon,
                            scratch);
  if (rc == ORC_OK) rc = orc_linear_fp32(scratch, rows, H, tensors[0], cfg->vocab_size, logits, threads);
  return rc;
}

int orc_model_prefill(const orc_model_config* cfg, const float* const* tensors,
                      orc_cache* cache, const uint32_t* token_ids, int64_t tokens,
                      float* logits, int32_t threads) {
  if (!cfg || !tensors || !cache || tokens <= 0) return ORC_ERR_INVALID_INPUT;
  if (!orc_cache_is_empty(cache)) return ORC_ERR_INVALID_INPUT;  /* model.rs:304-309 */
  const int64_t H = cfg->hidden_size, KV = (int64_t)cfg->num_key_value_heads * cfg->head_dimension;
  const int64_t I = cfg->intermediate_size, T = tokens;
  const int32_t hq = cfg->num_query_heads, hkv = cfg->num_key_value_heads, d = cfg->head_dimension;
  float inv_freq[256];
  if (d > 512) return ORC_ERR_INVALID_INPUT;
  int rc = orc_rope_inverse_frequencies(d, cfg->rope_theta, inv_freq);
  float* x = (float*)malloc((size_t)(T * H) * sizeof(float));
  float* xn = (float*)malloc((size_t)(T * H) * sizeof(float));
  float* q = (float*)malloc((size_t)(T * H) * sizeof(float));
  float* k = (float*)malloc((size_t)(T * KV) * sizeof(float));
  float* v = (float*)malloc((size_t)(T * KV) * sizeof(float));
  float* att = (float*)malloc((size_t)(T * H) * sizeof(float));
  float* o = (float*)malloc((size_t)(T * (H > I ? H : I)) * sizeof(float));
  float* probs = (float*)malloc((size_t)((int64_t)hq * T * T) * sizeof(float));
  if (!x || !xn || !q || !k || !v || !att || !o || !probs) rc = ORC_ERR_INVALID_INPUT;
  if (rc == ORC_OK) rc = orc_embedding_lookup(token_ids, T, tensors[0], cfg->vocab_size, H, x);
  for (int32_t l = 0; rc == ORC_OK && l < cfg->num_layers; ++l) {
    const float* const* lt = tensors + 1 + 9 * l;
    rc = orc_rmsnorm_rows(x, T, H, lt[0], cfg->rms_norm_epsilon, xn);
    if (rc == ORC_OK) rc = orc_linear(xn, T, H, lt[1], H, q, threads);
    if (rc == ORC_OK) rc = orc_linear(xn, T, H, lt[2], KV, k, threads);
    if (rc == ORC_OK) rc = orc_linear(xn, T, H, lt[3], KV, v, threads);
    if (rc == ORC_OK) rc = orc_apply_rotary_with_offset(q, k, T, hq, hkv, d, inv_freq, 0);
    if (rc == ORC_OK) rc = orc_causal_probabilities(q, k, T, hq, hkv, d, probs);
    if (rc == ORC_OK) rc = orc_attend_values(probs, v, T, hq, hkv, d, att);
    if (rc == ORC_OK) rc = orc_linear(att, T, H, lt[4], H, o, threads);
    if (rc == ORC_OK) rc = orc_cache_append_layer(cache, l, k, v, T);  /* attention.rs:863-868 */
    if (rc == ORC_OK)
      for (int64_t i = 0; i < T * H; ++i) x[i] += o[i];
    if (rc == ORC_OK) rc = orc_ffn_residual(cfg, lt, x, T, xn, o, threads);
  }
  if (rc == ORC_OK) rc = orc_final_logits(cfg, tensors, x, T, xn, logits, threads);
  if (rc != ORC_OK) orc_cache_clear(cache);
  free(x);
  free(xn);
  free(q);
  free(k);
  free(v);
  free(att);
  free(o);
  free(probs);
  return rc;
}

int orc_model_decode(const orc_model_config* cfg, const float* const* tensors,
                     orc_cache* cache, uint32_t token_id, float* logits, int32_t threads) {
  if (!cfg || !tensors || !cache) return ORC_ERR_INVALID_INPUT;
  /* model.rs:344-364 */
  if (!orc_cache_is_synchronized(cache) || orc_cache_sequence_length(cache) == 0 ||
      orc_cache_remaining_capacity(cache) == 0)
    return ORC_ERR_INVALID_INPUT;
  const int64_t previous = orc_cache_sequence_length(cache);
  const int64_t H = cfg->hidden_size, KV = (int64_t)cfg->num_key_value_heads * cfg->head_dimension;
  const int64_t I = cfg->intermediate_size;
  float inv_freq[256];
  if (cfg->head_dimension > 512) return ORC_ERR_INVALID_INPUT;
  int rc = orc_rope_inverse_frequencies(cfg->head_dimension, cfg->rope_theta, inv_freq);
  float* x = (float*)malloc((size_t)H * sizeof(float));
  float* xn = (float*)malloc((size_t)H * sizeof(float));
  float* q = (float*)malloc((size_t)H * sizeof(float));
  float* k = (float*)malloc((size_t)KV * sizeof(float));
  float* v = (float*)malloc((size_t)KV * sizeof(float));
  float* att = (float*)malloc((size_t)H * sizeof(float));
  float* o = (float*)malloc((size_t)(H > I ? H : I) * sizeof(float));
  if (!x || !xn || !q || !k || !v || !att || !o) rc = ORC_ERR_INVALID_INPUT;
  if (rc == ORC_OK) rc = orc_embedding_lookup(&token_id, 1, tensors[0], cfg->vocab_size, H, x);
  for (int32_t l = 0; rc == ORC_OK && l < cfg->num_layers; ++l) {
    const float* const* lt = tensors + 1 + 9 * l;
    rc = orc_rmsnorm_rows(x, 1, H, lt[0], cfg->rms_norm_epsilon, xn);
    if (rc == ORC_OK) rc = orc_linear(xn, 1, H, lt[1], H, q, threads);
    if (rc == ORC_OK) rc = orc_linear(xn, 1, H, lt[2], KV, k, threads);
    if (rc == ORC_OK) rc = orc_linear(xn, 1, H, lt[3], KV, v, threads);
    if (rc == ORC_OK)
      rc = orc_forward_cached_attention(cache, l, q, k, v, cfg->num_query_heads, inv_freq, att);
    if (rc == ORC_OK) rc = orc_linear(att, 1, H, lt[4], H, o, threads);
    if (rc == ORC_OK)
      for (int64_t i = 0; i < H; ++i) x[i] += o[i];
    if (rc == ORC_OK) rc = orc_ffn_residual(cfg, lt, x, 1, xn, o, threads);
  }
  if (rc == ORC_OK) rc = orc_final_logits(cfg, tensors, x, 1, xn, logits, threads);
  if (rc != ORC_OK) orc_cache_truncate_all(cache, previous);
  free(x);
  free(xn);
  free(q);
  free(k);
  free(v);
  free(att);
  free(o);
  return rc;
}

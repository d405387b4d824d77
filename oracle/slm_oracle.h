/*
 * CPU oracle for the KV-cache hot path of small-lm-rs (rust/engine).
 *
 * TEST INFRASTRUCTURE ONLY. This is a restatement, in plain C, of the
 * reference's CPU arithmetic (one function per reference function, each
 * citing the file:line it follows). It exists so that tests, the smoke check
 * and the bench's CPU-baseline leg can check the CUDA path against the
 * reference's numbers. Nothing in the product (the CUDA library, its C ABI
 * or its Python mirror) may call it.
 *
 * Numeric contract (what makes it bit-faithful to the Rust code):
 *   - Rust `f32::mul_add` is a correctly rounded fused multiply-add: `fmaf`.
 *   - Rust never contracts `a*b - c*d` into an FMA; this file is compiled
 *     with -ffp-contract=off and without -ffast-math for the same reason.
 *   - Rust `f32::{exp, sin, cos, powf, tanh, sqrt}` lower to the platform
 *     libm on Linux (glibc): `expf`, `sinf`, `cosf`, `powf`, `tanhf`, `sqrtf`.
 *
 * Status codes are the same integers as the CUDA library's C ABI.
 */
#ifndef SLM_ORACLE_H
#define SLM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  ORC_OK = 0,
  ORC_ERR_INVALID_CONFIGURATION = -1,
  ORC_ERR_INVALID_INPUT = -2,
  ORC_ERR_CAPACITY = -3,
  ORC_ERR_NON_FINITE = -4,
};

/* linear.rs:14-23 */
float orc_round_to_bfloat16(float value);

/* rope.rs:21-43 (inverse frequencies, :33-36) */
int orc_rope_inverse_frequencies(int32_t head_dim, float theta, float* out);
/* rope.rs:82-100 */
int orc_rope_apply_head(float* head, int32_t head_dim, const float* inv_freq,
                        int64_t position);
/* rope.rs:108-134 */
int orc_rope_apply_heads(float* values, int32_t num_heads, int32_t head_dim,
                         const float* inv_freq, int64_t position);
/* attention.rs:422-482: Q and K rows of T tokens at positions offset.. */
int orc_apply_rotary_with_offset(float* query, float* key, int64_t tokens,
                                 int32_t q_heads, int32_t kv_heads,
                                 int32_t head_dim, const float* inv_freq,
                                 int64_t position_offset);

/* softmax.rs:12-45 */
int orc_softmax_in_place(float* values, int64_t n);
/* softmax.rs:53-59 */
int orc_softmax_rows(float* values, int64_t rows, int64_t columns);

/* Dense per-request KV cache: kv_cache.rs:66-412. `quantize_bf16` stores
 * every appended value through orc_round_to_bfloat16 (bf16 KV storage has no
 * reference counterpart; the quantiser is the reference's own rounding). */
typedef struct orc_cache orc_cache;
orc_cache* orc_cache_allocate(int32_t num_layers, int32_t max_sequence_length,
                              int32_t kv_heads, int32_t head_dim,
                              int32_t quantize_bf16);
void orc_cache_free(orc_cache* cache);
int orc_cache_append_layer(orc_cache* cache, int32_t layer, const float* keys,
                           const float* values, int64_t token_count);
int64_t orc_cache_layer_sequence_length(const orc_cache* cache, int32_t layer);
int64_t orc_cache_sequence_length(const orc_cache* cache);
int32_t orc_cache_is_empty(const orc_cache* cache);
int32_t orc_cache_is_synchronized(const orc_cache* cache);
int64_t orc_cache_remaining_capacity(const orc_cache* cache);
int orc_cache_truncate_all(orc_cache* cache, int64_t sequence_length);
int orc_cache_truncate_layer(orc_cache* cache, int32_t layer,
                             int64_t sequence_length);
void orc_cache_clear(orc_cache* cache);
/* kv_cache.rs:237-248: copies the initialized prefix [len, kv_heads, d]. */
int orc_cache_layer_keys(const orc_cache* cache, int32_t layer, float* out);
int orc_cache_layer_values(const orc_cache* cache, int32_t layer, float* out);
/* kv_cache.rs:256-278 */
int orc_cache_key_head(const orc_cache* cache, int32_t layer, int64_t position,
                       int32_t kv_head, float* out);
int orc_cache_value_head(const orc_cache* cache, int32_t layer,
                         int64_t position, int32_t kv_head, float* out);

/* attention.rs:677-759: one rotated query [q_heads, d] against a layer. */
int orc_attend_cached_query(const orc_cache* cache, int32_t layer,
                            const float* query, int32_t q_heads, float* out);
/* attention.rs:794-810: RoPE(Q, K) at the layer length, append (K, V), then
 * attend. `query` and `key` are rotated in place. On an attention failure
 * the layer is truncated back (attention.rs:814). */
int orc_forward_cached_attention(orc_cache* cache, int32_t layer,
                                 float* query, float* key, const float* value,
                                 int32_t q_heads, const float* inv_freq,
                                 float* out);
/* The same step for n independent sequences of one layer; `threads` > 1
 * spreads whole sequences over OpenMP threads (each sequence is computed
 * exactly as above). q: [n, q_heads, d], k/v: [n, kv_heads, d]. */
int orc_forward_cached_attention_batch(orc_cache** caches, int32_t n,
                                       int32_t layer, float* query, float* key,
                                       const float* value, int32_t q_heads,
                                       const float* inv_freq, float* out,
                                       int32_t threads);

/* attention.rs:195-245: [q_heads, T, T], masked entries = f32::MIN. */
int orc_scaled_causal_scores(const float* query, const float* key,
                             int64_t tokens, int32_t q_heads, int32_t kv_heads,
                             int32_t head_dim, float* scores);
/* attention.rs:256-269 */
int orc_causal_probabilities(const float* query, const float* key,
                             int64_t tokens, int32_t q_heads, int32_t kv_heads,
                             int32_t head_dim, float* probabilities);
/* attention.rs:282-399: -> [T, q_heads, d] */
int orc_attend_values(const float* probabilities, const float* value,
                      int64_t tokens, int32_t q_heads, int32_t kv_heads,
                      int32_t head_dim, float* out);

/* linear.rs:44-107 (bf16 operands, fp32 fma accumulation) */
int orc_linear(const float* input, int64_t rows, int64_t in_features,
               const float* weight, int64_t out_features, float* out,
               int32_t threads);
/* linear.rs:119-152 */
int orc_linear_fp32(const float* input, int64_t rows, int64_t in_features,
                    const float* weight, int64_t out_features, float* out,
                    int32_t threads);

int32_t orc_max_threads(void);

/* rmsnorm.rs:80-91: per row, square sum by fma fold, inv = 1/sqrt(s/w + eps),
 * out = value * inv * scale (left to right). */
int orc_rmsnorm_rows(const float* input, int64_t rows, int64_t hidden,
                     const float* weight, float epsilon, float* out);
/* situ_glu.rs:59-70 and the sign-branched sigmoid of :131-138 */
float orc_situ_gate_activation(float value, float beta_gate);
float orc_situ_up_activation(float value, float beta_up);
/* situ_glu.rs:80-128: down(gate_act(gate(x)) * up_act(up(x))), bf16 linears */
int orc_situ_glu(const float* input, int64_t rows, int64_t hidden,
                 int64_t intermediate, const float* gate_weight,
                 const float* up_weight, const float* down_weight,
                 float beta_gate, float beta_up, float* out, int32_t threads);
/* embedding.rs:15-56 */
int orc_embedding_lookup(const uint32_t* token_ids, int64_t n,
                         const float* table, int64_t vocab, int64_t hidden,
                         float* out);
/* greedy.rs: argmax_finite (first maximum wins; empty or non-finite fails) */
int orc_argmax_finite(const float* logits, int64_t n, uint32_t* out);

/* The decoder-only model (model.rs, transformer.rs). `tensors` are fp32
 * arrays in the reference layout ([out, in] matrices), in this order:
 * token_embedding [vocab, hidden]; per layer: attention_norm [hidden],
 * q_proj [hidden, hidden], k_proj [kv, hidden], v_proj [kv, hidden],
 * o_proj [hidden, hidden], ffn_norm [hidden], gate_proj [inter, hidden],
 * up_proj [inter, hidden], down_proj [hidden, inter]; final_norm [hidden]
 * (kv = kv_heads * head_dim; names as weights.rs:347-375). */
typedef struct orc_model_config {
  int32_t vocab_size, hidden_size, intermediate_size, num_layers;
  int32_t num_query_heads, num_key_value_heads, head_dimension;
  float rms_norm_epsilon, rope_theta, situ_beta_gate, situ_beta_up;
} orc_model_config;
int32_t orc_model_tensor_count(int32_t num_layers);
/* model.rs:297-330 with transformer.rs:221-258 and attention.rs:835-870:
 * prompt prefill into an empty cache; logits [tokens, vocab]. The cache is
 * cleared on failure (model.rs:323-328). */
int orc_model_prefill(const orc_model_config* cfg, const float* const* tensors,
                      orc_cache* cache, const uint32_t* token_ids,
                      int64_t tokens, float* logits, int32_t threads);
/* model.rs:342-397 with transformer.rs:259-292 and attention.rs:772-825:
 * one cached token; logits [vocab]. Rolled back on failure (model.rs:390-396). */
int orc_model_decode(const orc_model_config* cfg, const float* const* tensors,
                     orc_cache* cache, uint32_t token_id, float* logits,
                     int32_t threads);

#ifdef __cplusplus
}
#endif

#endif /* SLM_ORACLE_H */

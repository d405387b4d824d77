/*
 * slmkv — B200 (sm_100a) KV-cache hot path for small-lm-rs, behind a C ABI.
 *
 * One context owns, on one GPU, a paged KV pool shared by many sequences:
 *   K pool, V pool : [layer][block][kv_head][slot 0..15][head_dim]  (f32 | bf16)
 *   block table    : [sequence slot][logical block] -> physical block id
 * A sequence is the paged counterpart of the reference's per-request dense
 * `KvCache` (rust/engine/src/kv_cache.rs:89-92): it keeps one logical length
 * per layer, exactly like `LayerKvCache::sequence_length`, and the token at
 * position p of layer l lives in slot p % 16 of physical block
 * block_table[seq][p / 16] of layer l.
 *
 * Conventions (the reference's, kv_cache.rs:172-230 and error.rs:14-121):
 *   - every call returns an slm_status; 0 is success and the negative codes
 *     below mirror EngineError::{InvalidConfiguration, InvalidInput};
 *   - validation completes before any host-visible state is mutated; a failed
 *     call leaves lengths, block tables and the pool as they were;
 *   - slm_last_error() returns the message of the last failure, formatted as
 *     the reference formats EngineError ("invalid input for KV cache: ...").
 * Threading: a context is used by one host thread at a time, and all calls on
 * one context are ordered on the stream they are given (use one stream per
 * context, or order the streams yourself).
 * Pointers named d_* are device pointers on the context's GPU; h_* are host.
 * No call falls back to the CPU: without a usable device every compute call
 * fails with SLM_ERR_NO_DEVICE.
 */
#ifndef SLMKV_H
#define SLMKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int slm_status;
enum {
  SLM_OK = 0,
  SLM_ERR_INVALID_CONFIGURATION = -1, /* EngineError::InvalidConfiguration */
  SLM_ERR_INVALID_INPUT = -2,         /* EngineError::InvalidInput (shape, index, state) */
  SLM_ERR_CAPACITY = -3,              /* InvalidInput: sequence would exceed its capacity */
  SLM_ERR_NON_FINITE = -4,            /* InvalidInput: appended K/V, or an attention
                                         score (softmax.rs:17-22), not finite */
  SLM_ERR_POOL_EXHAUSTED = -5,        /* no free physical block (paged pool only) */
  SLM_ERR_CUDA = -6,                  /* a CUDA runtime call failed */
  SLM_ERR_DEVICE_TIMEOUT = -7,        /* a kernel's bounded wait expired */
  SLM_ERR_NO_DEVICE = -8              /* context created without a device */
};

enum { SLM_KV_F32 = 0, SLM_KV_BF16 = 1 };

/* Model-side dimensions: KvCacheConfig (kv_cache.rs:8-18) plus what the
 * attention and RoPE need (config.rs: num_query_heads, rope_theta,
 * context_length), plus the paged pool size. */
typedef struct slm_config {
  int32_t num_layers;          /* KvCacheConfig::num_layers */
  int32_t num_query_heads;     /* ModelConfig::num_query_heads */
  int32_t num_key_value_heads; /* KvCacheConfig::num_key_value_heads */
  int32_t head_dimension;      /* KvCacheConfig::head_dimension (64 supported) */
  int32_t context_length;      /* ModelConfig::context_length (max positions) */
  float rope_theta;            /* ModelConfig::rope_theta */
  int32_t num_blocks;          /* physical 16-token blocks in the pool */
  int32_t max_sequences;       /* live sequence slots */
  int32_t kv_dtype;            /* SLM_KV_F32 (reference) or SLM_KV_BF16 */
} slm_config;

typedef struct slm_ctx slm_ctx;
typedef struct slm_batch slm_batch;
typedef void* slm_stream; /* a cudaStream_t; NULL = the legacy default stream */

/* ---- lifecycle ---------------------------------------------------------- */

/* Validates the config (kv_cache.rs:43-55, rope.rs:21-31, config.rs:91-198
 * head-divisibility) and allocates the pool, block table, RoPE table and
 * scratch on `device`. device = -1 creates a host-only context: bookkeeping
 * calls work, every compute call returns SLM_ERR_NO_DEVICE. */
slm_status slm_create(const slm_config* config, int32_t device, slm_ctx** out);
slm_status slm_destroy(slm_ctx* ctx);
/* Message of the last failed call ("" if none). Valid until the next call.
 * With ctx == NULL: the last failed call on this thread that has no context
 * (slm_create, slm_decode_attention_noalloc). */
const char* slm_last_error(const slm_ctx* ctx);
/* Bytes of device memory the context holds. */
slm_status slm_device_bytes(const slm_ctx* ctx, int64_t* bytes);
/* Number of kernels this context has launched since it was created. */
slm_status slm_launch_count(const slm_ctx* ctx, int64_t* launches);

/* ---- sequences: the reference's KvCache, one per request ------------------ */

/* KvCacheConfig::from_model + KvCache::allocate (kv_cache.rs:27-41, 101-116):
 * max_sequence_length in 1..=context_length. Blocks are taken lazily. */
slm_status slm_seq_create(slm_ctx* ctx, int32_t max_sequence_length, int32_t* seq_id);
/* Dropping a KvCache: releases its blocks (shared prefix blocks are kept
 * while other sequences or the prefix index hold them). */
slm_status slm_seq_free(slm_ctx* ctx, int32_t seq_id);
/* kv_cache.rs:157-170 */
slm_status slm_seq_layer_length(const slm_ctx* ctx, int32_t seq_id, int32_t layer,
                                int32_t* length);
/* kv_cache.rs:129-135 (minimum over layers) */
slm_status slm_seq_length(const slm_ctx* ctx, int32_t seq_id, int32_t* length);
/* kv_cache.rs:139-141 and 145-150 */
slm_status slm_seq_is_empty(const slm_ctx* ctx, int32_t seq_id, int32_t* is_empty);
slm_status slm_seq_is_synchronized(const slm_ctx* ctx, int32_t seq_id, int32_t* is_sync);
/* kv_cache.rs:285-293 (after the longest layer, saturating) */
slm_status slm_seq_remaining_capacity(const slm_ctx* ctx, int32_t seq_id, int32_t* remaining);
/* kv_cache.rs:302-321: transactional; fails unless every layer >= length. */
slm_status slm_seq_truncate_all(slm_ctx* ctx, int32_t seq_id, int32_t length);
/* truncate_all for n sequences at once (each transactional on its own);
 * stops at the first failure and returns it. */
slm_status slm_seqs_truncate_all(slm_ctx* ctx, int32_t n, const int32_t* h_seq_ids,
                                 const int32_t* h_lengths);
/* kv_cache.rs:323-346 */
slm_status slm_seq_truncate_layer(slm_ctx* ctx, int32_t seq_id, int32_t layer, int32_t length);
/* kv_cache.rs:296-300 */
slm_status slm_seq_clear(slm_ctx* ctx, int32_t seq_id);
/* Physical block ids of the sequence (paged layout; no reference
 * counterpart). Writes min(n_blocks, capacity) ids and the count. */
slm_status slm_seq_blocks(const slm_ctx* ctx, int32_t seq_id, int32_t* h_ids, int32_t capacity,
                          int32_t* n_blocks);

/* ---- single-sequence cache operations ------------------------------------- */

/* KvCache::append_layer (kv_cache.rs:182-230) with the K half of
 * ProjectedQkv::apply_rotary_with_offset (attention.rs:422-482) fused in:
 * keys/values are [token_count, kv_heads, head_dim] f32 on the device; when
 * `rotate_keys` is non-zero the keys are rotated at positions len..len+T-1
 * before they are stored (values are stored as given). Stream-ordered.
 * The finite check (kv_cache.rs:192-197) runs on the device: a non-finite
 * value makes the call fail with SLM_ERR_NON_FINITE and the layer keeps its
 * old length; the call synchronizes `stream` to report it. */
slm_status slm_append_layer(slm_ctx* ctx, int32_t seq_id, int32_t layer, const float* d_keys,
                            const float* d_values, int32_t token_count, int32_t rotate_keys,
                            slm_stream stream);
/* KvCache::layer_keys / layer_values (kv_cache.rs:237-248): gathers the
 * initialized prefix of one layer through the block table into dense
 * [len, kv_heads, head_dim] f32 device buffers (bf16 entries widen exactly).
 * Either output may be NULL. */
slm_status slm_gather_layer(slm_ctx* ctx, int32_t seq_id, int32_t layer, float* d_keys,
                            float* d_values, slm_stream stream);
/* GroupedQueryAttention::attend_cached_query (attention.rs:677-759) for one
 * sequence: query [q_heads, head_dim] already rotated, out [q_heads*head_dim].
 * Waits for `stream`: a score that is not finite (a non-finite query, or an
 * overflowing dot product) fails the call with SLM_ERR_NON_FINITE, as
 * softmax_rows fails the reference's call (attention.rs:731, softmax.rs:17-22). */
slm_status slm_attend_cached_query(slm_ctx* ctx, int32_t seq_id, int32_t layer,
                                   const float* d_query, float* d_out, slm_stream stream);

/* ---- batched steps: many sequences, one launch per layer ------------------ */

/* Opens a step for n sequences that each add token_counts[i] tokens to every
 * layer (1 for a decode step). Each sequence must be synchronized
 * (model.rs:345-350) and have room (kv_cache.rs:203-211); physical blocks for
 * the new positions are taken here (copy-on-write when a target block is
 * shared), and the step descriptor is uploaded once for all layers. Nothing
 * is mutated when it fails. One open batch per context. */
slm_status slm_batch_begin(slm_ctx* ctx, int32_t n, const int32_t* h_seq_ids,
                           const int32_t* h_token_counts, slm_stream stream, slm_batch** out);
/* Decode step of one layer for every sequence of the batch (all counts 1):
 * GroupedQueryAttention::forward_cached_token's cache part
 * (attention.rs:794-810): RoPE on Q and K at the pre-append position, append
 * K/V, then attention over the grown cache, in one kernel.
 * q: [n, q_heads, d], k/v: [n, kv_heads, d] (unrotated), out: [n, q_heads, d]. */
slm_status slm_batch_decode_layer(slm_batch* batch, int32_t layer, const float* d_query,
                                  const float* d_keys, const float* d_values, float* d_out);
/* One decode layer's device buffers, as slm_batch_decode_layer takes them. */
typedef struct slm_layer_io {
  const float* query;   /* [n, q_heads, d] */
  const float* keys;    /* [n, kv_heads, d], unrotated */
  const float* values;  /* [n, kv_heads, d] */
  float* out;           /* [n, q_heads, d] */
} slm_layer_io;
/* slm_batch_decode_layer for layers first_layer .. first_layer + n_layers - 1,
 * io[i] for layer first_layer + i, when the inputs of all of them are ready
 * (forward_cached_token's cache part, attention.rs:794-810, per layer). The
 * layers share the batch's plan, so with an f32 pool up to 8 of them run as
 * one launch: each warp of the grid takes its slice of the step's blocks in
 * every layer in turn, keeping its copies in flight across the layer
 * boundaries (bf16 pools: one launch per layer). Results equal the one-layer
 * calls'. Every layer is checked before anything is launched; a layer's
 * output may not overlap another layer's buffers. */
slm_status slm_batch_decode_layers(slm_batch* batch, int32_t first_layer, int32_t n_layers,
                                   const slm_layer_io* io);
/* slm_batch_decode_layers for a caller whose step inputs and outputs are in
 * host memory (an engine's host tensors, as forward_cached_token holds them,
 * attention.rs:772-779): h_query [n_layers][n][q_heads][d], h_keys and
 * h_values [n_layers][n][kv_heads][d] (unrotated), h_out
 * [n_layers][n][q_heads][d]. The inputs are copied into the context's own
 * device staging (allocated at the first call, grown when a call needs more),
 * the layers run as slm_batch_decode_layers, and the outputs are copied back
 * ahead of the step's statuses: h_out is complete when slm_batch_end or
 * slm_batch_wait returns for this batch, and the host buffers must stay valid
 * until then. Host buffers should be pinned (cudaHostAlloc, cudaHostRegister)
 * for the copies to overlap the GPU's work; up to 8 submitted steps keep
 * their own staging. */
slm_status slm_batch_decode_layers_host(slm_batch* batch, int32_t first_layer, int32_t n_layers,
                                        const float* h_query, const float* h_keys,
                                        const float* h_values, float* h_out);
/* Append-only form (prompt prefill, attention.rs:863-868): keys/values are the
 * batch's tokens concatenated in batch order, [sum(counts), kv_heads, d]. */
slm_status slm_batch_append_layer(slm_batch* batch, int32_t layer, const float* d_keys,
                                  const float* d_values, int32_t rotate_keys);
/* Causal attention of the batch's new tokens over each sequence's cache
 * (after slm_batch_append_layer for this layer): query token j of sequence i
 * sits at position base_i + j and sees positions 0..base_i+j. With base 0 this
 * is the prompt prefill of attention.rs:859-861 (causal_probabilities +
 * attend_values); with an attached prefix it extends the prefix.
 * q: [sum(counts), q_heads, d] (unrotated if rotate_query), out likewise. */
slm_status slm_batch_prefill_attention(slm_batch* batch, int32_t layer, const float* d_query,
                                       int32_t rotate_query, float* d_out);
/* The attention of slm_batch_prefill_attention (and, for a batch whose token
 * counts are all 1, the attention half of slm_batch_decode_layer, after
 * slm_batch_append_layer with rotate_keys) computed in the reference's own
 * operation order, bit for bit with its CPU path: scaled_causal_scores,
 * causal_probabilities and attend_values (attention.rs:195-399) for a prompt,
 * attend_cached_query (attention.rs:677-759) for a decoded token; each score
 * an in-order fma fold, softmax_in_place's sequential sum and glibc's expf
 * (softmax.rs:26-44), each output an in-order fma fold over the positions.
 * f32 pools only; rows of up to 57344 positions. Slower than the split-K
 * kernels (one warp per token row and query head, a sequential sum); the
 * model step uses it on its exact-order path. Same arguments as
 * slm_batch_prefill_attention. */
slm_status slm_batch_attention_exact(slm_batch* batch, int32_t layer, const float* d_query,
                                     int32_t rotate_query, float* d_out);
/* slm_batch_decode_layer in the reference's operation order, bit for bit
 * (f32 pools): forward_cached_token's cache part (attention.rs:794-810) --
 * RoPE on Q and K at the pre-append position, the append (a non-finite K/V
 * fails the sequence, kv_cache.rs:192-197), then attend_cached_query
 * (attention.rs:677-759) as slm_batch_attention_exact computes it -- in one
 * kernel per layer. Same arguments as slm_batch_decode_layer. */
slm_status slm_batch_decode_layer_exact(slm_batch* batch, int32_t layer, const float* d_query,
                                        const float* d_keys, const float* d_values, float* d_out);
/* Closes the step: waits for its stream, and reports per sequence (h_status
 * may be NULL) 0 or SLM_ERR_NON_FINITE. A sequence whose appends were not
 * finite, whose attention met a score that is not finite (softmax.rs:17-22,
 * in decode as attention.rs:731,814-815, in prefill as causal_probabilities),
 * or whose layers did not all advance by its count, is rolled back to its
 * length at slm_batch_begin (model.rs:390-396). Returns the first failure.
 * The pool never holds a non-finite value: a failed append stores zeros. */
slm_status slm_batch_end(slm_batch* batch, int32_t* h_status);
/* Abandons the step: every sequence goes back to its begin length. */
slm_status slm_batch_rollback(slm_batch* batch);
/* Pipelined steps (no reference counterpart: the reference runs one request
 * at a time, worker.rs:87-98). slm_batch_submit closes the step without
 * waiting for the GPU: the per-sequence status is copied back on the batch's
 * stream and the next step may begin at once, planned on the advanced
 * lengths. At most 8 submitted batches may be pending. slm_batch_wait waits
 * for a submitted batch and reports like slm_batch_end; batches resolve in
 * submission order (waiting for a later one resolves the earlier ones, whose
 * own wait then returns at once), and every submitted batch must be waited
 * for. A sequence that fails is rolled back to its length at that batch's
 * begin, and every later batch holding it reports the same failure and rolls
 * it back to the same length. slm_batch_end is submit + wait. */
slm_status slm_batch_submit(slm_batch* batch);
slm_status slm_batch_wait(slm_batch* batch, int32_t* h_status);

/* ---- prefix cache (no reference counterpart; README.md:247 lists it as
 *      future work). Full 16-token blocks are indexed by their token chain. -- */

/* Attaches to an EMPTY sequence the longest chain of indexed full blocks that
 * matches tokens[0..n_tokens); every layer's length becomes 16 * matched
 * blocks. The blocks are shared (reference-counted) and never written again:
 * a later write into one copies it first. */
slm_status slm_prefix_attach(slm_ctx* ctx, int32_t seq_id, const uint32_t* h_tokens,
                             int32_t n_tokens, int32_t* reused_tokens);
/* Indexes the full blocks of a synchronized sequence that hold
 * tokens[0..n_tokens) (n_tokens <= its length). Returns how many blocks are
 * now indexed for that chain. */
slm_status slm_prefix_publish(slm_ctx* ctx, int32_t seq_id, const uint32_t* h_tokens,
                              int32_t n_tokens, int32_t* indexed_blocks);
/* Number of blocks held by the index, and blocks free in the pool. */
slm_status slm_pool_stats(const slm_ctx* ctx, int32_t* free_blocks, int32_t* indexed_blocks);
/* Shuffles the free list with a seeded permutation, so that sequences get
 * scattered physical blocks. Pool must be unused. */
slm_status slm_pool_shuffle(slm_ctx* ctx, uint64_t seed);
/* The configuration a context was created with (KvCacheConfig::from_model's
 * inputs, kv_cache.rs:27-41). */
slm_status slm_ctx_config(const slm_ctx* ctx, slm_config* out);

/* ---- continuous batching (no reference counterpart: the reference serves
 *      one request at a time behind a Mutex, rust/server/src/worker.rs:87-98).
 * A scheduler owns the pool of one context: requests are admitted in arrival
 * order while fewer than max_running are running and the pool holds their
 * prompt; every step it plans one decode token for each running request whose
 * prompt is cached, and prompt chunks for the others within max_prefill_tokens
 * (a prompt may take several steps). The caller runs the step's KV work: a
 * decode batch (slm_batch_begin with counts 1, slm_batch_decode_layer per
 * layer) and a prefill batch (slm_batch_begin with the chunk counts,
 * slm_batch_append_layer and slm_batch_prefill_attention per layer), then
 * commits the statuses. The first output token comes with the end of the
 * prompt (GenerationService: prefill logits pick it); each decode step adds
 * one; a request is finished after max_new_tokens and its sequence is freed.
 * When the pool cannot hold a step, the most recently admitted requests are
 * preempted: their sequences are freed and they go back to the front of the
 * queue, to prefill again what they had cached (recomputation). Sequence
 * capacity per request: prompt_len + max_new_tokens <= context_length. */
typedef struct slm_sched slm_sched;
typedef struct {
  int32_t max_running;         /* requests stepped together (>= 1) */
  int32_t max_prefill_tokens;  /* prompt tokens planned per step (>= 1) */
} slm_sched_config;
slm_status slm_sched_create(slm_ctx* ctx, const slm_sched_config* config, slm_sched** out);
slm_status slm_sched_destroy(slm_sched* sched);
slm_status slm_sched_submit(slm_sched* sched, int64_t request_id, int32_t prompt_len,
                            int32_t max_new_tokens);
/* Plans the next step into caller arrays of capacity max_running: the decode
 * sequences, and the prefill sequences with their token counts. A step with
 * nothing to do returns 0 and 0. */
slm_status slm_sched_plan(slm_sched* sched, int32_t* n_decode, int32_t* decode_seq,
                          int32_t* n_prefill, int32_t* prefill_seq, int32_t* prefill_count);
/* The requests behind the last plan, in plan order: their ids and the cache
 * position each entry starts at (a decode entry feeds the token at that
 * position; a prefill entry feeds positions pos .. pos + count - 1, its
 * prompt, or after a preemption its prompt and generated tokens again). Any
 * array may be NULL. */
slm_status slm_sched_plan_requests(const slm_sched* sched, int64_t* decode_request,
                                   int32_t* decode_pos, int64_t* prefill_request,
                                   int32_t* prefill_pos);
/* Commits the last plan: the per-sequence statuses its batches reported (in
 * plan order; NULL when that part was empty). Requests whose sequence failed
 * are finished with that status. Fills the requests finished by this step
 * (arrays of capacity max_running; their output token counts in h_generated,
 * NULL to skip). */
slm_status slm_sched_commit(slm_sched* sched, const int32_t* decode_status,
                            const int32_t* prefill_status, int32_t* n_finished,
                            int64_t* finished_id, int32_t* finished_status, int32_t* h_generated);
/* Queue sizes and counters: waiting, running, preemptions so far, output
 * tokens so far. */
slm_status slm_sched_counts(const slm_sched* sched, int32_t* waiting, int32_t* running,
                            int64_t* preemptions, int64_t* generated_tokens);

/* ---- allocation-free decode attention ------------------------------------
 * No counterpart in the reference. For callers that cannot allocate device
 * memory: engines that hand out all device memory from one arena of their
 * own, and plugins loaded into hosts that forbid new device allocations
 * after start-up. It computes GroupedQueryAttention::attend_cached_query
 * (attention.rs:677-759) for n sequences of a paged KV cache the caller owns,
 * with the library's decode kernel, and allocates nothing: the plan, split-K
 * partials, merge counters and error word live in one 2 MiB file-scope device
 * array that every GPU loading this library holds until the process exits.
 *   d_key_pool, d_value_pool  [num_blocks][kv_heads][16][64] f32, one layer
 *   h_block_table             host [n][max_blocks_per_sequence] physical blocks
 *   h_lengths                 host [n], each in 1..=16*max_blocks_per_sequence
 *   d_query                   [n][q_heads][64], already rotated
 *   d_out                     [n][q_heads][64]
 * Limits (SLM_ERR_INVALID_INPUT beyond them): n * kv_heads <= 4096 and
 * sum(ceil(len/16)) * kv_heads <= 131072 blocks; q_heads / kv_heads in
 * {1, 2, 4, 8}; num_blocks * kv_heads <= INT32_MAX. Runs on the calling
 * thread's current device and returns after the result is in d_out (it
 * synchronizes `stream`). The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress); make that first call before any
 * stream capture. All calls share the array and clear what must start at
 * zero; calls that overlap on the GPU (other streams or threads) race on it.
 * A score that is not finite fails the call with SLM_ERR_NON_FINITE
 * (softmax.rs:17-22). Errors: slm_last_error(NULL). */
slm_status slm_decode_attention_noalloc(const float* d_key_pool, const float* d_value_pool,
                                        int32_t num_blocks, int32_t num_query_heads,
                                        int32_t num_key_value_heads, const int32_t* h_block_table,
                                        int32_t max_blocks_per_sequence, const int32_t* h_lengths,
                                        int32_t n, const float* d_query, float* d_out,
                                        slm_stream stream);

/* ---- full-model steps (SmallLMModel, model.rs) ------------------------------
 * The decoder-only model around the KV path: token embedding, per layer
 * RMSNorm -> q/k/v projections -> the batch's cache step -> output projection
 * + residual -> RMSNorm -> SiTU-GLU -> residual, then the final RMSNorm and
 * the tied fp32 vocabulary projection. Projections take bf16-rounded
 * operands with fp32 accumulation (linear.rs:44-107); the vocabulary
 * projection is fp32 (linear.rs:119-152). */
typedef struct slm_model slm_model;
typedef struct slm_model_config {
  int32_t vocab_size;        /* ModelConfig::vocab_size */
  int32_t hidden_size;       /* ModelConfig::hidden_size = num_query_heads * head_dimension */
  int32_t intermediate_size; /* ModelConfig::intermediate_size */
  float rms_norm_epsilon;    /* ModelConfig::rms_norm_epsilon */
  float situ_beta_gate;      /* ModelConfig::situ_beta_gate */
  float situ_beta_up;        /* ModelConfig::situ_beta_up */
} slm_model_config;
/* Layers, heads, head dimension and RoPE come from the context's config.
 * `h_tensors` are host fp32 arrays in the reference layout ([out, in]
 * matrices), 2 + 9 * num_layers of them in the order of weights.rs:347-375:
 * token_embedding [vocab, hidden]; per layer attention_norm [hidden],
 * q_proj [hidden, hidden], k_proj [kv, hidden], v_proj [kv, hidden],
 * o_proj [hidden, hidden], ffn_norm [hidden], gate_proj [inter, hidden],
 * up_proj [inter, hidden], down_proj [hidden, inter]; final_norm [hidden]
 * (kv = num_key_value_heads * head_dimension). Projection matrices are stored
 * on the device rounded to bf16 (the rounding linear.rs applies to them at
 * every call); the embedding and the norms stay fp32. */
slm_status slm_model_create(slm_ctx* ctx, const slm_model_config* config,
                            const float* const* h_tensors, int32_t n_tensors, slm_model** out);
slm_status slm_model_destroy(slm_model* model);
/* Steps of up to `max_rows` token rows (0..1024; default 1024, or 0 when the
 * model's rows do not fit the kernels' shared memory) compute every projection
 * output as linear.rs:98-103 does: one fp32 fma fold over the input features in
 * order, so f32-KV logits match the CPU engine to ~1e-6. Larger steps, and
 * every step when 0, use tensor-core GEMMs: another accumulation order, within
 * the reference's GPU-vs-CPU logit thresholds (parity/runner.rs:33-43) and
 * faster on wide models. Not an engine method: a B200 execution choice. */
slm_status slm_model_set_exact_rows(slm_model* model, int32_t max_rows);
/* One cached decode step (model.rs:342-397) for every sequence of an open
 * batch whose token counts are all 1: d_token_ids [n] (device int32) are
 * embedded and run through every layer (the batch's decode step per layer);
 * d_logits [n, vocab] (device, may be NULL) and d_next_token [n] (device,
 * the first maximal logit, greedy.rs; may be NULL). A token id outside the
 * vocabulary or non-finite logits make the batch's end report
 * SLM_ERR_INVALID_INPUT and roll the step back (model.rs:390-396). */
slm_status slm_model_decode(slm_model* model, slm_batch* batch, const int32_t* d_token_ids,
                            float* d_logits, int32_t* d_next_token);
/* Prompt prefill (model.rs:297-330) for every sequence of an open batch:
 * d_token_ids [sum(counts)] (device int32, the batch's tokens in batch order;
 * token j of sequence i is at position base_i + j). Only each sequence's last
 * position is projected to the vocabulary: d_logits [n, vocab] (may be NULL)
 * and d_next_token [n] (may be NULL). */
slm_status slm_model_prefill(slm_model* model, slm_batch* batch, const int32_t* d_token_ids,
                             float* d_logits, int32_t* d_next_token);
/* ModelWeights::load (weights.rs:117-190) into a device model: a SafeTensors
 * file whose tensors are exactly the expected set for this config and the
 * context's layers and heads (names and shapes of weights.rs:344-378), every
 * one F32 (little-endian); `expected_parameter_count` (0: not checked) must
 * equal their total (ModelConfig::expected_parameter_count). A malformed file
 * or any mismatch fails with SLM_ERR_INVALID_INPUT ("invalid weights: ..."). */
slm_status slm_model_load_safetensors(slm_ctx* ctx, const slm_model_config* config, const char* path,
                                      int64_t expected_parameter_count, slm_model** out);
/* The same checks without a device (layers, KV heads and head dimension
 * given); reports the parameter count. Errors: slm_last_error(NULL). */
slm_status slm_safetensors_check(const slm_model_config* config, int32_t num_layers,
                                 int32_t num_key_value_heads, int32_t head_dimension, const char* path,
                                 int64_t expected_parameter_count, int64_t* parameter_count);

#ifdef __cplusplus
}
#endif

#endif /* SLMKV_H */

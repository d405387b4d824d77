//! Raw bindings to libslmkv (`include/slmkv.h`), the B200 (sm_100a)
//! KV-cache path of small-lm-rs: one declaration per C function, in the
//! header's order, with the header's argument names. Pointers named `d_*`
//! are device pointers on the context's GPU, `h_*` host pointers; every
//! function returns an `slm_status` (0 or one of the `SLM_ERR_*` codes,
//! which mirror `EngineError`, error.rs:14-121). The safe API is the
//! `slmkv` crate.
//!
//! small-lm-rs forbids `unsafe` in its workspace (rust/engine/src/lib.rs:12,
//! Cargo.toml:27-29); this crate is where the FFI's unsafety lives.
#![allow(unsafe_code)]
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_void};

pub const SLM_OK: i32 = 0;
pub const SLM_ERR_INVALID_CONFIGURATION: i32 = -1;
pub const SLM_ERR_INVALID_INPUT: i32 = -2;
pub const SLM_ERR_CAPACITY: i32 = -3;
pub const SLM_ERR_NON_FINITE: i32 = -4;
pub const SLM_ERR_POOL_EXHAUSTED: i32 = -5;
pub const SLM_ERR_CUDA: i32 = -6;
pub const SLM_ERR_DEVICE_TIMEOUT: i32 = -7;
pub const SLM_ERR_NO_DEVICE: i32 = -8;

pub const SLM_KV_F32: i32 = 0;
pub const SLM_KV_BF16: i32 = 1;

/// `slm_config`: KvCacheConfig (kv_cache.rs:8-18) plus the attention and
/// RoPE dimensions and the paged pool's size.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq)]
pub struct SlmConfig {
    pub num_layers: i32,
    pub num_query_heads: i32,
    pub num_key_value_heads: i32,
    pub head_dimension: i32,
    pub context_length: i32,
    pub rope_theta: f32,
    pub num_blocks: i32,
    pub max_sequences: i32,
    pub kv_dtype: i32,
}

/// `slm_layer_io`: one decode layer's device buffers (`slm_batch_decode_layers`).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct SlmLayerIo {
    pub query: *const f32,
    pub keys: *const f32,
    pub values: *const f32,
    pub out: *mut f32,
}

/// `slm_sched_config`.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct SlmSchedConfig {
    pub max_running: i32,
    pub max_prefill_tokens: i32,
}

/// `slm_model_config`: the ModelConfig fields the model step needs.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq)]
pub struct SlmModelConfig {
    pub vocab_size: i32,
    pub hidden_size: i32,
    pub intermediate_size: i32,
    pub rms_norm_epsilon: f32,
    pub situ_beta_gate: f32,
    pub situ_beta_up: f32,
}

/// Opaque handles.
#[repr(C)]
pub struct SlmCtx {
    _private: [u8; 0],
}
#[repr(C)]
pub struct SlmBatch {
    _private: [u8; 0],
}
#[repr(C)]
pub struct SlmSched {
    _private: [u8; 0],
}
#[repr(C)]
pub struct SlmModel {
    _private: [u8; 0],
}

extern "C" {
    pub fn slm_create(config: *const SlmConfig, device: i32, out: *mut *mut SlmCtx) -> i32;
    pub fn slm_destroy(ctx: *mut SlmCtx) -> i32;
    pub fn slm_last_error(ctx: *const SlmCtx) -> *const c_char;
    pub fn slm_device_bytes(ctx: *const SlmCtx, bytes: *mut i64) -> i32;
    pub fn slm_launch_count(ctx: *const SlmCtx, launches: *mut i64) -> i32;
    pub fn slm_seq_create(ctx: *mut SlmCtx, max_sequence_length: i32, seq_id: *mut i32) -> i32;
    pub fn slm_seq_free(ctx: *mut SlmCtx, seq_id: i32) -> i32;
    pub fn slm_seq_layer_length(ctx: *const SlmCtx, seq_id: i32, layer: i32, length: *mut i32) -> i32;
    pub fn slm_seq_length(ctx: *const SlmCtx, seq_id: i32, length: *mut i32) -> i32;
    pub fn slm_seq_is_empty(ctx: *const SlmCtx, seq_id: i32, is_empty: *mut i32) -> i32;
    pub fn slm_seq_is_synchronized(ctx: *const SlmCtx, seq_id: i32, is_sync: *mut i32) -> i32;
    pub fn slm_seq_remaining_capacity(ctx: *const SlmCtx, seq_id: i32, remaining: *mut i32) -> i32;
    pub fn slm_seq_truncate_all(ctx: *mut SlmCtx, seq_id: i32, length: i32) -> i32;
    pub fn slm_seqs_truncate_all(ctx: *mut SlmCtx, n: i32, h_seq_ids: *const i32, h_lengths: *const i32) -> i32;
    pub fn slm_seq_truncate_layer(ctx: *mut SlmCtx, seq_id: i32, layer: i32, length: i32) -> i32;
    pub fn slm_seq_clear(ctx: *mut SlmCtx, seq_id: i32) -> i32;
    pub fn slm_seq_blocks(ctx: *const SlmCtx, seq_id: i32, h_ids: *mut i32, capacity: i32, n_blocks: *mut i32) -> i32;
    pub fn slm_append_layer(ctx: *mut SlmCtx, seq_id: i32, layer: i32, d_keys: *const f32, d_values: *const f32, token_count: i32, rotate_keys: i32, stream: *mut c_void) -> i32;
    pub fn slm_gather_layer(ctx: *mut SlmCtx, seq_id: i32, layer: i32, d_keys: *mut f32, d_values: *mut f32, stream: *mut c_void) -> i32;
    pub fn slm_attend_cached_query(ctx: *mut SlmCtx, seq_id: i32, layer: i32, d_query: *const f32, d_out: *mut f32, stream: *mut c_void) -> i32;
    pub fn slm_batch_begin(ctx: *mut SlmCtx, n: i32, h_seq_ids: *const i32, h_token_counts: *const i32, stream: *mut c_void, out: *mut *mut SlmBatch) -> i32;
    pub fn slm_batch_decode_layer(batch: *mut SlmBatch, layer: i32, d_query: *const f32, d_keys: *const f32, d_values: *const f32, d_out: *mut f32) -> i32;
    pub fn slm_batch_decode_layers(batch: *mut SlmBatch, first_layer: i32, n_layers: i32, io: *const SlmLayerIo) -> i32;
    pub fn slm_batch_decode_layers_host(batch: *mut SlmBatch, first_layer: i32, n_layers: i32, h_query: *const f32, h_keys: *const f32, h_values: *const f32, h_out: *mut f32) -> i32;
    pub fn slm_batch_append_layer(batch: *mut SlmBatch, layer: i32, d_keys: *const f32, d_values: *const f32, rotate_keys: i32) -> i32;
    pub fn slm_batch_prefill_attention(batch: *mut SlmBatch, layer: i32, d_query: *const f32, rotate_query: i32, d_out: *mut f32) -> i32;
    pub fn slm_batch_attention_exact(batch: *mut SlmBatch, layer: i32, d_query: *const f32, rotate_query: i32, d_out: *mut f32) -> i32;
    pub fn slm_batch_decode_layer_exact(batch: *mut SlmBatch, layer: i32, d_query: *const f32, d_keys: *const f32, d_values: *const f32, d_out: *mut f32) -> i32;
    pub fn slm_batch_end(batch: *mut SlmBatch, h_status: *mut i32) -> i32;
    pub fn slm_batch_rollback(batch: *mut SlmBatch) -> i32;
    pub fn slm_batch_submit(batch: *mut SlmBatch) -> i32;
    pub fn slm_batch_wait(batch: *mut SlmBatch, h_status: *mut i32) -> i32;
    pub fn slm_prefix_attach(ctx: *mut SlmCtx, seq_id: i32, h_tokens: *const u32, n_tokens: i32, reused_tokens: *mut i32) -> i32;
    pub fn slm_prefix_publish(ctx: *mut SlmCtx, seq_id: i32, h_tokens: *const u32, n_tokens: i32, indexed_blocks: *mut i32) -> i32;
    pub fn slm_pool_stats(ctx: *const SlmCtx, free_blocks: *mut i32, indexed_blocks: *mut i32) -> i32;
    pub fn slm_pool_shuffle(ctx: *mut SlmCtx, seed: u64) -> i32;
    pub fn slm_ctx_config(ctx: *const SlmCtx, out: *mut SlmConfig) -> i32;
    pub fn slm_sched_create(ctx: *mut SlmCtx, config: *const SlmSchedConfig, out: *mut *mut SlmSched) -> i32;
    pub fn slm_sched_destroy(sched: *mut SlmSched) -> i32;
    pub fn slm_sched_submit(sched: *mut SlmSched, request_id: i64, prompt_len: i32, max_new_tokens: i32) -> i32;
    pub fn slm_sched_plan(sched: *mut SlmSched, n_decode: *mut i32, decode_seq: *mut i32, n_prefill: *mut i32, prefill_seq: *mut i32, prefill_count: *mut i32) -> i32;
    pub fn slm_sched_plan_requests(sched: *const SlmSched, decode_request: *mut i64, decode_pos: *mut i32, prefill_request: *mut i64, prefill_pos: *mut i32) -> i32;
    pub fn slm_sched_commit(sched: *mut SlmSched, decode_status: *const i32, prefill_status: *const i32, n_finished: *mut i32, finished_id: *mut i64, finished_status: *mut i32, h_generated: *mut i32) -> i32;
    pub fn slm_sched_counts(sched: *const SlmSched, waiting: *mut i32, running: *mut i32, preemptions: *mut i64, generated_tokens: *mut i64) -> i32;
    pub fn slm_decode_attention_noalloc(d_key_pool: *const f32, d_value_pool: *const f32, num_blocks: i32, num_query_heads: i32, num_key_value_heads: i32, h_block_table: *const i32, max_blocks_per_sequence: i32, h_lengths: *const i32, n: i32, d_query: *const f32, d_out: *mut f32, stream: *mut c_void) -> i32;
    pub fn slm_model_create(ctx: *mut SlmCtx, config: *const SlmModelConfig, h_tensors: *const *const f32, n_tensors: i32, out: *mut *mut SlmModel) -> i32;
    pub fn slm_model_destroy(model: *mut SlmModel) -> i32;
    pub fn slm_model_set_exact_rows(model: *mut SlmModel, max_rows: i32) -> i32;
    pub fn slm_model_decode(model: *mut SlmModel, batch: *mut SlmBatch, d_token_ids: *const i32, d_logits: *mut f32, d_next_token: *mut i32) -> i32;
    pub fn slm_model_prefill(model: *mut SlmModel, batch: *mut SlmBatch, d_token_ids: *const i32, d_logits: *mut f32, d_next_token: *mut i32) -> i32;
    pub fn slm_model_load_safetensors(ctx: *mut SlmCtx, config: *const SlmModelConfig, path: *const c_char, expected_parameter_count: i64, out: *mut *mut SlmModel) -> i32;
    pub fn slm_safetensors_check(config: *const SlmModelConfig, num_layers: i32, num_key_value_heads: i32, head_dimension: i32, path: *const c_char, expected_parameter_count: i64, parameter_count: *mut i64) -> i32;
}

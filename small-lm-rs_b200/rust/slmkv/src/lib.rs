//! Safe API over libslmkv, the B200 KV-cache path of small-lm-rs.
//!
//! The types mirror the reference engine's (rust/engine/src): a [`Context`]
//! owns one GPU's paged KV pool; a [`KvCache`] is one request's cache in it,
//! with `KvCache`'s methods (kv_cache.rs:101-412) and errors; a [`Batch`] is
//! one model step for many requests (model.rs:342-397: every sequence must be
//! synchronized and have room, and a failed sequence is rolled back to its
//! length at the step's start); a [`Model`] runs SmallLMModel's cached
//! decode and prefill (model.rs:297-397) for a whole batch; a [`Scheduler`]
//! plans continuous-batching steps.
//!
//! Device memory is not managed here: tensors are passed as [`DevicePtr`]s
//! the caller owns (from its CUDA runtime or allocator), f32, row-major
//! `[rows, heads, 64]`, 16-byte aligned. Creating a `DevicePtr` is the one
//! unsafe step: the caller vouches that the address is valid device memory
//! of the context's GPU for as long as the call runs on its stream.
#![allow(unsafe_code)]

use std::ffi::{CStr, CString};
use std::fmt;
use std::os::raw::c_void;
use std::path::Path;

use slmkv_sys as sys;

/// The library's errors, grouped as the reference's `EngineError`
/// (error.rs:14-121) groups them; `code` is the `SLM_ERR_*` status.
#[derive(Clone, Debug, PartialEq, Eq)]
pub enum Error {
    /// `EngineError::InvalidConfiguration`.
    InvalidConfiguration { message: String },
    /// `EngineError::InvalidInput`: shape, index, state, capacity,
    /// non-finite values or scores, or an exhausted pool.
    InvalidInput { code: i32, message: String },
    /// A CUDA failure, an expired device wait, or no device.
    Device { code: i32, message: String },
}

impl fmt::Display for Error {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        match self {
            Error::InvalidConfiguration { message } => write!(f, "{message}"),
            Error::InvalidInput { message, .. } => write!(f, "{message}"),
            Error::Device { code, message } => write!(f, "device error {code}: {message}"),
        }
    }
}

impl std::error::Error for Error {}

pub type Result<T> = std::result::Result<T, Error>;

fn error_from(code: i32, message: String) -> Error {
    match code {
        sys::SLM_ERR_INVALID_CONFIGURATION => Error::InvalidConfiguration { message },
        sys::SLM_ERR_INVALID_INPUT
        | sys::SLM_ERR_CAPACITY
        | sys::SLM_ERR_NON_FINITE
        | sys::SLM_ERR_POOL_EXHAUSTED => Error::InvalidInput { code, message },
        _ => Error::Device { code, message },
    }
}

fn last_error(ctx: *const sys::SlmCtx) -> String {
    // SAFETY: slm_last_error returns a NUL-terminated string owned by the
    // library, valid until the next call on the same context (or thread).
    unsafe {
        let p = sys::slm_last_error(ctx);
        if p.is_null() {
            String::new()
        } else {
            CStr::from_ptr(p).to_string_lossy().into_owned()
        }
    }
}

fn check(ctx: *const sys::SlmCtx, rc: i32) -> Result<()> {
    if rc == sys::SLM_OK {
        Ok(())
    } else {
        Err(error_from(rc, last_error(ctx)))
    }
}

/// A device address of `T` elements on the context's GPU.
#[derive(Clone, Copy, Debug)]
pub struct DevicePtr<T> {
    ptr: *mut T,
}

impl<T> DevicePtr<T> {
    /// # Safety
    /// `ptr` must be device memory of the context's GPU, large enough for
    /// every call it is passed to, and stay valid until that call's work on
    /// its stream is done.
    pub unsafe fn new(ptr: *mut T) -> Self {
        DevicePtr { ptr }
    }
    /// No buffer (for the optional outputs).
    pub fn null() -> Self {
        DevicePtr { ptr: std::ptr::null_mut() }
    }
    fn c(&self) -> *const T {
        self.ptr as *const T
    }
    fn m(&self) -> *mut T {
        self.ptr
    }
}

/// A CUDA stream handle (`cudaStream_t`); the default is the legacy stream.
#[derive(Clone, Copy, Debug)]
pub struct Stream(pub *mut c_void);

impl Default for Stream {
    fn default() -> Self {
        Stream(std::ptr::null_mut())
    }
}

/// KV element type of the pool.
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum KvType {
    /// The reference's fp32 cache.
    F32,
    /// bf16 entries, rounded as linear.rs:14-23 rounds.
    Bf16,
}

/// `slm_config`: KvCacheConfig (kv_cache.rs:8-18) plus heads, RoPE and the
/// pool's size.
#[derive(Clone, Copy, Debug, PartialEq)]
pub struct Config {
    pub num_layers: i32,
    pub num_query_heads: i32,
    pub num_key_value_heads: i32,
    pub head_dimension: i32,
    pub context_length: i32,
    pub rope_theta: f32,
    pub num_blocks: i32,
    pub max_sequences: i32,
    pub kv_type: KvType,
}

impl Config {
    fn raw(&self) -> sys::SlmConfig {
        sys::SlmConfig {
            num_layers: self.num_layers,
            num_query_heads: self.num_query_heads,
            num_key_value_heads: self.num_key_value_heads,
            head_dimension: self.head_dimension,
            context_length: self.context_length,
            rope_theta: self.rope_theta,
            num_blocks: self.num_blocks,
            max_sequences: self.max_sequences,
            kv_dtype: match self.kv_type {
                KvType::F32 => sys::SLM_KV_F32,
                KvType::Bf16 => sys::SLM_KV_BF16,
            },
        }
    }
}

/// One GPU's paged KV pool, block tables, RoPE table and scratch. Used by
/// one host thread at a time (it may move between threads).
pub struct Context {
    raw: *mut sys::SlmCtx,
}

// SAFETY: the library keeps no thread-local state for a context; it only
// requires that one thread uses it at a time. The raw pointer field keeps
// `Context` !Sync, so a `&Context` never crosses threads.
unsafe impl Send for Context {}

impl Context {
    /// Validates the configuration (kv_cache.rs:43-55, rope.rs:21-31) and
    /// allocates the pool on `device` (-1: bookkeeping only, no device).
    pub fn new(config: &Config, device: i32) -> Result<Self> {
        let raw_cfg = config.raw();
        let mut raw = std::ptr::null_mut();
        // SAFETY: pointers to a live config and to the out handle.
        let rc = unsafe { sys::slm_create(&raw_cfg, device, &mut raw) };
        check(std::ptr::null(), rc)?;
        Ok(Context { raw })
    }

    /// Allocates a request's cache: KvCacheConfig::from_model +
    /// KvCache::allocate (kv_cache.rs:27-41,101-116). Blocks are taken lazily.
    pub fn allocate_kv_cache(&self, max_sequence_length: i32) -> Result<KvCache<'_>> {
        let mut id = 0;
        // SAFETY: a live context and an out pointer.
        check(self.raw, unsafe { sys::slm_seq_create(self.raw, max_sequence_length, &mut id) })?;
        Ok(KvCache { ctx: self, id })
    }

    /// Opens a step in which each cache adds `token_counts[i]` tokens to every
    /// layer (1 for a decode step); see `slm_batch_begin`.
    pub fn begin<'c>(&'c self, caches: &[&KvCache<'c>], token_counts: &[i32],
                     stream: Stream) -> Result<Batch<'c>> {
        if caches.len() != token_counts.len() {
            return Err(Error::InvalidInput {
                code: sys::SLM_ERR_INVALID_INPUT,
                message: "invalid input for batch: one token count per cache".into(),
            });
        }
        let ids: Vec<i32> = caches.iter().map(|c| c.id).collect();
        let mut raw = std::ptr::null_mut();
        // SAFETY: arrays of caches.len() elements, live for the call.
        let rc = unsafe {
            sys::slm_batch_begin(self.raw, ids.len() as i32, ids.as_ptr(), token_counts.as_ptr(),
                                 stream.0, &mut raw)
        };
        check(self.raw, rc)?;
        Ok(Batch { ctx: self, raw, n: ids.len(), open: true })
    }

    /// Free blocks and blocks held by the prefix index.
    pub fn pool_stats(&self) -> Result<(i32, i32)> {
        let (mut free, mut indexed) = (0, 0);
        // SAFETY: out pointers.
        check(self.raw, unsafe { sys::slm_pool_stats(self.raw, &mut free, &mut indexed) })?;
        Ok((free, indexed))
    }

    /// Kernels launched since creation.
    pub fn launch_count(&self) -> Result<i64> {
        let mut n = 0;
        // SAFETY: out pointer.
        check(self.raw, unsafe { sys::slm_launch_count(self.raw, &mut n) })?;
        Ok(n)
    }

    pub fn raw(&self) -> *mut sys::SlmCtx {
        self.raw
    }
}

impl Drop for Context {
    fn drop(&mut self) {
        // SAFETY: the handle came from slm_create and is destroyed once.
        unsafe {
            sys::slm_destroy(self.raw);
        }
    }
}

/// One request's KV cache in a context's pool: the reference's `KvCache`
/// (kv_cache.rs:89-412) with one length per layer.
pub struct KvCache<'c> {
    ctx: &'c Context,
    id: i32,
}

impl<'c> KvCache<'c> {
    fn q(&self, f: impl FnOnce(*mut sys::SlmCtx, i32, *mut i32) -> i32) -> Result<i32> {
        let mut v = 0;
        check(self.ctx.raw, f(self.ctx.raw, self.id, &mut v))?;
        Ok(v)
    }

    /// kv_cache.rs:157-170
    pub fn layer_sequence_length(&self, layer: i32) -> Result<i32> {
        // SAFETY: out pointer.
        self.q(|c, id, out| unsafe { sys::slm_seq_layer_length(c, id, layer, out) })
    }
    /// kv_cache.rs:129-135 (the shortest layer)
    pub fn sequence_length(&self) -> Result<i32> {
        self.q(|c, id, out| unsafe { sys::slm_seq_length(c, id, out) })
    }
    /// kv_cache.rs:139-141
    pub fn is_empty(&self) -> Result<bool> {
        Ok(self.q(|c, id, out| unsafe { sys::slm_seq_is_empty(c, id, out) })? != 0)
    }
    /// kv_cache.rs:145-150
    pub fn is_synchronized(&self) -> Result<bool> {
        Ok(self.q(|c, id, out| unsafe { sys::slm_seq_is_synchronized(c, id, out) })? != 0)
    }
    /// kv_cache.rs:285-293
    pub fn remaining_capacity(&self) -> Result<i32> {
        self.q(|c, id, out| unsafe { sys::slm_seq_remaining_capacity(c, id, out) })
    }
    /// kv_cache.rs:302-321
    pub fn truncate_all(&self, length: i32) -> Result<()> {
        // SAFETY: plain values.
        check(self.ctx.raw, unsafe { sys::slm_seq_truncate_all(self.ctx.raw, self.id, length) })
    }
    /// kv_cache.rs:323-346
    pub fn truncate_layer(&self, layer: i32, length: i32) -> Result<()> {
        check(self.ctx.raw,
              unsafe { sys::slm_seq_truncate_layer(self.ctx.raw, self.id, layer, length) })
    }
    /// kv_cache.rs:296-300
    pub fn clear(&self) -> Result<()> {
        check(self.ctx.raw, unsafe { sys::slm_seq_clear(self.ctx.raw, self.id) })
    }

    /// KvCache::append_layer (kv_cache.rs:182-230) with RoPE on the keys at
    /// the layer's current positions when `rotate_keys`: keys/values are
    /// `[token_count, kv_heads, 64]`. A non-finite value fails the call and
    /// leaves the layer as it was.
    pub fn append_layer(&self, layer: i32, keys: DevicePtr<f32>, values: DevicePtr<f32>,
                        token_count: i32, rotate_keys: bool, stream: Stream) -> Result<()> {
        // SAFETY: the DevicePtr contract covers the device buffers.
        let rc = unsafe {
            sys::slm_append_layer(self.ctx.raw, self.id, layer, keys.c(), values.c(), token_count,
                                  rotate_keys as i32, stream.0)
        };
        check(self.ctx.raw, rc)
    }

    /// KvCache::layer_keys / layer_values (kv_cache.rs:237-248): the layer's
    /// initialized prefix into dense `[len, kv_heads, 64]` buffers (either
    /// may be null).
    pub fn gather_layer(&self, layer: i32, keys: DevicePtr<f32>, values: DevicePtr<f32>,
                        stream: Stream) -> Result<()> {
        let rc = unsafe {
            sys::slm_gather_layer(self.ctx.raw, self.id, layer, keys.m(), values.m(), stream.0)
        };
        check(self.ctx.raw, rc)
    }

    /// GroupedQueryAttention::attend_cached_query (attention.rs:677-759):
    /// query `[q_heads, 64]`, already rotated; out `[q_heads * 64]`.
    pub fn attend_cached_query(&self, layer: i32, query: DevicePtr<f32>, out: DevicePtr<f32>,
                               stream: Stream) -> Result<()> {
        let rc = unsafe {
            sys::slm_attend_cached_query(self.ctx.raw, self.id, layer, query.c(), out.m(),
                                         stream.0)
        };
        check(self.ctx.raw, rc)
    }

    /// Physical block ids (paged layout).
    pub fn blocks(&self) -> Result<Vec<i32>> {
        let mut n = 0;
        check(self.ctx.raw, unsafe {
            sys::slm_seq_blocks(self.ctx.raw, self.id, std::ptr::null_mut(), 0, &mut n)
        })?;
        let mut ids = vec![0i32; n as usize];
        check(self.ctx.raw, unsafe {
            sys::slm_seq_blocks(self.ctx.raw, self.id, ids.as_mut_ptr(), n, &mut n)
        })?;
        Ok(ids)
    }

    /// Attaches the longest indexed chain of full blocks matching `tokens`
    /// to this empty cache; returns the tokens reused.
    pub fn attach_prefix(&self, tokens: &[u32]) -> Result<i32> {
        let mut reused = 0;
        check(self.ctx.raw, unsafe {
            sys::slm_prefix_attach(self.ctx.raw, self.id, tokens.as_ptr(), tokens.len() as i32,
                                   &mut reused)
        })?;
        Ok(reused)
    }

    /// Indexes this cache's full blocks holding `tokens`; returns the blocks
    /// now indexed for that chain.
    pub fn publish_prefix(&self, tokens: &[u32]) -> Result<i32> {
        let mut indexed = 0;
        check(self.ctx.raw, unsafe {
            sys::slm_prefix_publish(self.ctx.raw, self.id, tokens.as_ptr(), tokens.len() as i32,
                                    &mut indexed)
        })?;
        Ok(indexed)
    }

    /// The sequence id the C API uses for this cache.
    pub fn id(&self) -> i32 {
        self.id
    }
}

impl Drop for KvCache<'_> {
    fn drop(&mut self) {
        // SAFETY: the id came from slm_seq_create on this context.
        unsafe {
            sys::slm_seq_free(self.ctx.raw, self.id);
        }
    }
}

/// One step for many caches; dropped while open, it is rolled back.
pub struct Batch<'c> {
    ctx: &'c Context,
    raw: *mut sys::SlmBatch,
    n: usize,
    open: bool,
}

impl<'c> Batch<'c> {
    fn open_raw(&self) -> Result<*mut sys::SlmBatch> {
        if self.open {
            Ok(self.raw)
        } else {
            Err(Error::InvalidInput {
                code: sys::SLM_ERR_INVALID_INPUT,
                message: "invalid input for batch: the batch is not open".into(),
            })
        }
    }

    /// forward_cached_token's cache part (attention.rs:794-810) for every
    /// sequence: RoPE on Q and K at the pre-append position, append, attend.
    /// q `[n, q_heads, 64]`, k/v `[n, kv_heads, 64]`, out `[n, q_heads, 64]`.
    pub fn decode_layer(&mut self, layer: i32, q: DevicePtr<f32>, k: DevicePtr<f32>,
                        v: DevicePtr<f32>, out: DevicePtr<f32>) -> Result<()> {
        let b = self.open_raw()?;
        check(self.ctx.raw,
              unsafe { sys::slm_batch_decode_layer(b, layer, q.c(), k.c(), v.c(), out.m()) })
    }

    /// `decode_layer` for layers `first_layer ..` in order, one
    /// `(q, k, v, out)` per layer, when all of their inputs are ready: up to
    /// eight layers run as one launch. A layer's output may not overlap
    /// another layer's buffers.
    pub fn decode_layers(&mut self, first_layer: i32,
                         layers: &[(DevicePtr<f32>, DevicePtr<f32>, DevicePtr<f32>, DevicePtr<f32>)])
                         -> Result<()> {
        let b = self.open_raw()?;
        let io: Vec<sys::SlmLayerIo> = layers
            .iter()
            .map(|(q, k, v, out)| sys::SlmLayerIo { query: q.c(), keys: k.c(), values: v.c(), out: out.m() })
            .collect();
        check(self.ctx.raw, unsafe {
            sys::slm_batch_decode_layers(b, first_layer, io.len() as i32, io.as_ptr())
        })
    }

    /// `decode_layers` with the step's inputs and outputs in host memory
    /// (`[n_layers][n][heads][64]` each; pinned for the copies to overlap):
    /// `out` is complete once this batch's `end` / `wait` has returned.
    pub fn decode_layers_host(&mut self, first_layer: i32, n_layers: i32, q: &[f32], k: &[f32],
                              v: &[f32], out: &mut [f32]) -> Result<()> {
        let b = self.open_raw()?;
        let mut cfg = sys::SlmConfig::default();
        check(self.ctx.raw, unsafe { sys::slm_ctx_config(self.ctx.raw, &mut cfg) })?;
        let (hq, hkv) = (cfg.num_query_heads as usize, cfg.num_key_value_heads as usize);
        let per = self.n * 64 * n_layers.max(0) as usize;
        if q.len() < per * hq || k.len() < per * hkv || v.len() < per * hkv || out.len() < per * hq {
            return Err(Error::InvalidInput {
                code: sys::SLM_ERR_INVALID_INPUT,
                message: "invalid input for batch: host buffers shorter than the layers need".into(),
            });
        }
        check(self.ctx.raw, unsafe {
            sys::slm_batch_decode_layers_host(b, first_layer, n_layers, q.as_ptr(), k.as_ptr(),
                                              v.as_ptr(), out.as_mut_ptr())
        })
    }

    /// `decode_layer` in the reference's operation order, bit for bit with
    /// its CPU path (f32 pools).
    pub fn decode_layer_exact(&mut self, layer: i32, q: DevicePtr<f32>, k: DevicePtr<f32>,
                              v: DevicePtr<f32>, out: DevicePtr<f32>) -> Result<()> {
        let b = self.open_raw()?;
        check(self.ctx.raw, unsafe {
            sys::slm_batch_decode_layer_exact(b, layer, q.c(), k.c(), v.c(), out.m())
        })
    }

    /// Appends the batch's tokens of one layer (prompt prefill).
    pub fn append_layer(&mut self, layer: i32, k: DevicePtr<f32>, v: DevicePtr<f32>,
                        rotate_keys: bool) -> Result<()> {
        let b = self.open_raw()?;
        check(self.ctx.raw,
              unsafe { sys::slm_batch_append_layer(b, layer, k.c(), v.c(), rotate_keys as i32) })
    }

    /// Causal attention of the batch's new tokens over each cache
    /// (attention.rs:835-870).
    pub fn prefill_attention(&mut self, layer: i32, q: DevicePtr<f32>, rotate_query: bool,
                             out: DevicePtr<f32>) -> Result<()> {
        let b = self.open_raw()?;
        check(self.ctx.raw, unsafe {
            sys::slm_batch_prefill_attention(b, layer, q.c(), rotate_query as i32, out.m())
        })
    }

    /// The same attention in the reference's operation order, bit for bit
    /// with its CPU path (f32 pools).
    pub fn attention_exact(&mut self, layer: i32, q: DevicePtr<f32>, rotate_query: bool,
                           out: DevicePtr<f32>) -> Result<()> {
        let b = self.open_raw()?;
        check(self.ctx.raw, unsafe {
            sys::slm_batch_attention_exact(b, layer, q.c(), rotate_query as i32, out.m())
        })
    }

    /// Closes the step: per cache `Ok(())` or the error that rolled it back
    /// to its length at the step's start (model.rs:390-396).
    pub fn end(mut self) -> Result<Vec<Result<()>>> {
        let b = self.open_raw()?;
        let mut status = vec![0i32; self.n];
        self.open = false;
        let rc = unsafe { sys::slm_batch_end(b, status.as_mut_ptr()) };
        if rc != sys::SLM_OK && status.iter().all(|&s| s == sys::SLM_OK) {
            return Err(error_from(rc, last_error(self.ctx.raw)));
        }
        let msg = last_error(self.ctx.raw);
        Ok(status.into_iter()
            .map(|s| if s == sys::SLM_OK { Ok(()) } else { Err(error_from(s, msg.clone())) })
            .collect())
    }

    /// Abandons the step: every cache back to its length at the start.
    pub fn rollback(mut self) -> Result<()> {
        let b = self.open_raw()?;
        self.open = false;
        check(self.ctx.raw, unsafe { sys::slm_batch_rollback(b) })
    }

    pub fn raw(&self) -> *mut sys::SlmBatch {
        self.raw
    }
}

impl Drop for Batch<'_> {
    fn drop(&mut self) {
        if self.open {
            // SAFETY: an open batch of this context.
            unsafe {
                sys::slm_batch_rollback(self.raw);
            }
        }
    }
}

/// `slm_model_config`: the ModelConfig fields the model step needs.
#[derive(Clone, Copy, Debug, PartialEq)]
pub struct ModelConfig {
    pub vocab_size: i32,
    pub hidden_size: i32,
    pub intermediate_size: i32,
    pub rms_norm_epsilon: f32,
    pub situ_beta_gate: f32,
    pub situ_beta_up: f32,
}

impl ModelConfig {
    fn raw(&self) -> sys::SlmModelConfig {
        sys::SlmModelConfig {
            vocab_size: self.vocab_size,
            hidden_size: self.hidden_size,
            intermediate_size: self.intermediate_size,
            rms_norm_epsilon: self.rms_norm_epsilon,
            situ_beta_gate: self.situ_beta_gate,
            situ_beta_up: self.situ_beta_up,
        }
    }
}

/// SmallLMModel's steps on the GPU (model.rs:297-397) for whole batches.
pub struct Model<'c> {
    ctx: &'c Context,
    raw: *mut sys::SlmModel,
}

impl<'c> Model<'c> {
    /// Weights as host fp32 arrays in the reference layout and order
    /// (weights.rs:347-375): embedding, per layer the nine tensors, final norm.
    pub fn new(ctx: &'c Context, config: &ModelConfig, tensors: &[&[f32]]) -> Result<Self> {
        let ptrs: Vec<*const f32> = tensors.iter().map(|t| t.as_ptr()).collect();
        let raw_cfg = config.raw();
        let mut raw = std::ptr::null_mut();
        check(ctx.raw, unsafe {
            sys::slm_model_create(ctx.raw, &raw_cfg, ptrs.as_ptr(), ptrs.len() as i32, &mut raw)
        })?;
        Ok(Model { ctx, raw })
    }

    /// ModelWeights::load (weights.rs:117-190) from a SafeTensors file.
    pub fn load_safetensors(ctx: &'c Context, config: &ModelConfig, path: &Path,
                            expected_parameter_count: i64) -> Result<Self> {
        let c_path = CString::new(path.to_string_lossy().as_bytes()).map_err(|_| {
            Error::InvalidInput { code: sys::SLM_ERR_INVALID_INPUT,
                                  message: "invalid weights: path holds a NUL byte".into() }
        })?;
        let raw_cfg = config.raw();
        let mut raw = std::ptr::null_mut();
        check(ctx.raw, unsafe {
            sys::slm_model_load_safetensors(ctx.raw, &raw_cfg, c_path.as_ptr(),
                                            expected_parameter_count, &mut raw)
        })?;
        Ok(Model { ctx, raw })
    }

    /// Steps of up to `max_rows` token rows project in linear.rs's order.
    pub fn set_exact_rows(&mut self, max_rows: i32) -> Result<()> {
        check(self.ctx.raw, unsafe { sys::slm_model_set_exact_rows(self.raw, max_rows) })
    }

    /// SmallLMModel::forward_cached_token (model.rs:342-397) for every
    /// sequence of `batch` (token counts 1): token ids `[n]` (device i32),
    /// logits `[n, vocab]` and greedy next tokens `[n]` (either may be null).
    pub fn decode(&self, batch: &mut Batch<'c>, token_ids: DevicePtr<i32>,
                  logits: DevicePtr<f32>, next_tokens: DevicePtr<i32>) -> Result<()> {
        let b = batch.open_raw()?;
        check(self.ctx.raw, unsafe {
            sys::slm_model_decode(self.raw, b, token_ids.c(), logits.m(), next_tokens.m())
        })
    }

    /// SmallLMModel::forward_prefill_with_cache (model.rs:297-330): the
    /// batch's tokens in batch order; logits of each sequence's last row.
    pub fn prefill(&self, batch: &mut Batch<'c>, token_ids: DevicePtr<i32>,
                   logits: DevicePtr<f32>, next_tokens: DevicePtr<i32>) -> Result<()> {
        let b = batch.open_raw()?;
        check(self.ctx.raw, unsafe {
            sys::slm_model_prefill(self.raw, b, token_ids.c(), logits.m(), next_tokens.m())
        })
    }
}

impl Drop for Model<'_> {
    fn drop(&mut self) {
        unsafe {
            sys::slm_model_destroy(self.raw);
        }
    }
}

/// Continuous batching over a context's pool (slm_sched_*): the server's
/// replacement for one request at a time (rust/server/src/worker.rs:87-98).
pub struct Scheduler<'c> {
    ctx: &'c Context,
    raw: *mut sys::SlmSched,
    cap: usize,
}

/// The sequences of one planned step.
#[derive(Clone, Debug, Default, PartialEq, Eq)]
pub struct Plan {
    pub decode_seq: Vec<i32>,
    pub prefill_seq: Vec<i32>,
    pub prefill_count: Vec<i32>,
}

impl<'c> Scheduler<'c> {
    pub fn new(ctx: &'c Context, max_running: i32, max_prefill_tokens: i32) -> Result<Self> {
        let cfg = sys::SlmSchedConfig { max_running, max_prefill_tokens };
        let mut raw = std::ptr::null_mut();
        check(ctx.raw, unsafe { sys::slm_sched_create(ctx.raw, &cfg, &mut raw) })?;
        Ok(Scheduler { ctx, raw, cap: max_running.max(1) as usize })
    }

    pub fn submit(&mut self, request_id: i64, prompt_len: i32, max_new_tokens: i32) -> Result<()> {
        check(self.ctx.raw,
              unsafe { sys::slm_sched_submit(self.raw, request_id, prompt_len, max_new_tokens) })
    }

    pub fn plan(&mut self) -> Result<Plan> {
        let (mut nd, mut np) = (0, 0);
        let mut p = Plan {
            decode_seq: vec![0; self.cap],
            prefill_seq: vec![0; self.cap],
            prefill_count: vec![0; self.cap],
        };
        check(self.ctx.raw, unsafe {
            sys::slm_sched_plan(self.raw, &mut nd, p.decode_seq.as_mut_ptr(), &mut np,
                                p.prefill_seq.as_mut_ptr(), p.prefill_count.as_mut_ptr())
        })?;
        p.decode_seq.truncate(nd as usize);
        p.prefill_seq.truncate(np as usize);
        p.prefill_count.truncate(np as usize);
        Ok(p)
    }

    /// Commits the last plan with its batches' statuses; returns the
    /// requests it finished as (id, status, output tokens).
    pub fn commit(&mut self, decode_status: &[i32], prefill_status: &[i32])
                  -> Result<Vec<(i64, i32, i32)>> {
        let mut nf = 0;
        let mut ids = vec![0i64; self.cap];
        let mut st = vec![0i32; self.cap];
        let mut gen = vec![0i32; self.cap];
        let opt = |s: &[i32]| if s.is_empty() { std::ptr::null() } else { s.as_ptr() };
        check(self.ctx.raw, unsafe {
            sys::slm_sched_commit(self.raw, opt(decode_status), opt(prefill_status), &mut nf,
                                  ids.as_mut_ptr(), st.as_mut_ptr(), gen.as_mut_ptr())
        })?;
        Ok((0..nf as usize).map(|i| (ids[i], st[i], gen[i])).collect())
    }
}

impl Drop for Scheduler<'_> {
    fn drop(&mut self) {
        unsafe {
            sys::slm_sched_destroy(self.raw);
        }
    }
}

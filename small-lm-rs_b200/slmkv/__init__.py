"""Python mirror of small-lm-rs's KV-cache API over the B200 library.

``libslmkv.so`` (built from ``../csrc``) holds the CUDA kernels and the host
engine; this module binds its C ABI (``include/slmkv.h``) with ctypes and
mirrors the reference's Rust surface:

- ``KvCache`` follows ``rust/engine/src/kv_cache.rs`` (``allocate``,
  ``append_layer``, ``layer_sequence_length``, ``sequence_length``,
  ``is_empty``, ``is_synchronized``, ``remaining_capacity``, ``truncate_all``,
  ``truncate_layer``, ``clear``, ``layer_keys``, ``layer_values``,
  ``key_head``, ``value_head``), one instance per request as in the reference,
  but backed by blocks of a shared paged pool on the GPU;
- ``attend_cached_query`` follows ``attention.rs:677-759`` and
  ``Batch.decode_layer`` the cache part of ``forward_cached_token``
  (``attention.rs:794-810``) for many sequences in one launch;
- errors are raised as ``InvalidConfiguration`` / ``InvalidInput``
  (``error.rs:14-60``) carrying the library's message.

Tensors are torch CUDA float32 tensors; calls run on torch's current stream.
There is no CPU fallback: without the library or a device, calls raise.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path
from typing import Sequence

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libslmkv.so"
CSRC = HERE.parent / "csrc"

OK = 0
ERR_INVALID_CONFIGURATION = -1
ERR_INVALID_INPUT = -2
ERR_CAPACITY = -3
ERR_NON_FINITE = -4
ERR_POOL_EXHAUSTED = -5
ERR_CUDA = -6
ERR_DEVICE_TIMEOUT = -7
ERR_NO_DEVICE = -8

KV_F32 = 0
KV_BF16 = 1

BLOCK_TOKENS = 16


class EngineError(RuntimeError):
    """Base of the errors raised by the library (error.rs:14-121)."""

    def __init__(self, code: int, message: str):
        super().__init__(message or f"slmkv status {code}")
        self.code = code


class InvalidConfiguration(EngineError):
    """EngineError::InvalidConfiguration."""


class InvalidInput(EngineError):
    """EngineError::InvalidInput (shape, index, capacity, non-finite, pool)."""


class DeviceError(EngineError):
    """A CUDA failure, an expired device wait, or no device."""


def _error_class(code: int):
    if code == ERR_INVALID_CONFIGURATION:
        return InvalidConfiguration
    if code in (ERR_INVALID_INPUT, ERR_CAPACITY, ERR_NON_FINITE, ERR_POOL_EXHAUSTED):
        return InvalidInput
    return DeviceError


class SlmConfig(C.Structure):
    _fields_ = [
        ("num_layers", C.c_int32),
        ("num_query_heads", C.c_int32),
        ("num_key_value_heads", C.c_int32),
        ("head_dimension", C.c_int32),
        ("context_length", C.c_int32),
        ("rope_theta", C.c_float),
        ("num_blocks", C.c_int32),
        ("max_sequences", C.c_int32),
        ("kv_dtype", C.c_int32),
    ]


class LayerIo(C.Structure):
    """slm_layer_io: one decode layer's device buffers."""
    _fields_ = [("query", C.c_void_p), ("keys", C.c_void_p), ("values", C.c_void_p),
                ("out", C.c_void_p)]


def layer_io_array(layers):
    """A ctypes array of LayerIo for slm_batch_decode_layers from (query,
    keys, values, out) tuples of device addresses (ints), built once for a
    loop that reuses its buffers."""
    arr = (LayerIo * len(layers))()
    for i, (q, k, v, o) in enumerate(layers):
        arr[i] = LayerIo(q, k, v, o)
    return arr


class SchedConfig(C.Structure):
    _fields_ = [("max_running", C.c_int32), ("max_prefill_tokens", C.c_int32)]


class ModelConfig(C.Structure):
    """slm_model_config: the model-only fields of ModelConfig (config.rs);
    layers, heads, head dimension and RoPE come from the pool."""
    _fields_ = [("vocab_size", C.c_int32), ("hidden_size", C.c_int32),
                ("intermediate_size", C.c_int32), ("rms_norm_epsilon", C.c_float),
                ("situ_beta_gate", C.c_float), ("situ_beta_up", C.c_float)]


# Every symbol include/slmkv.h declares, with its ctypes signature.
_i32, _i64, _u64, _vp = C.c_int32, C.c_int64, C.c_uint64, C.c_void_p
_pi32 = C.POINTER(C.c_int32)
_pu32 = C.POINTER(C.c_uint32)
SIGNATURES = {
    "slm_create": (C.c_int, [C.POINTER(SlmConfig), _i32, C.POINTER(_vp)]),
    "slm_destroy": (C.c_int, [_vp]),
    "slm_last_error": (C.c_char_p, [_vp]),
    "slm_device_bytes": (C.c_int, [_vp, C.POINTER(_i64)]),
    "slm_launch_count": (C.c_int, [_vp, C.POINTER(_i64)]),
    "slm_seq_create": (C.c_int, [_vp, _i32, _pi32]),
    "slm_seq_free": (C.c_int, [_vp, _i32]),
    "slm_seq_layer_length": (C.c_int, [_vp, _i32, _i32, _pi32]),
    "slm_seq_length": (C.c_int, [_vp, _i32, _pi32]),
    "slm_seq_is_empty": (C.c_int, [_vp, _i32, _pi32]),
    "slm_seq_is_synchronized": (C.c_int, [_vp, _i32, _pi32]),
    "slm_seq_remaining_capacity": (C.c_int, [_vp, _i32, _pi32]),
    "slm_seq_truncate_all": (C.c_int, [_vp, _i32, _i32]),
    "slm_seqs_truncate_all": (C.c_int, [_vp, _i32, _pi32, _pi32]),
    "slm_seq_truncate_layer": (C.c_int, [_vp, _i32, _i32, _i32]),
    "slm_seq_clear": (C.c_int, [_vp, _i32]),
    "slm_seq_blocks": (C.c_int, [_vp, _i32, _pi32, _i32, _pi32]),
    "slm_append_layer": (C.c_int, [_vp, _i32, _i32, _vp, _vp, _i32, _i32, _vp]),
    "slm_gather_layer": (C.c_int, [_vp, _i32, _i32, _vp, _vp, _vp]),
    "slm_attend_cached_query": (C.c_int, [_vp, _i32, _i32, _vp, _vp, _vp]),
    "slm_batch_begin": (C.c_int, [_vp, _i32, _pi32, _pi32, _vp, C.POINTER(_vp)]),
    "slm_batch_decode_layer": (C.c_int, [_vp, _i32, _vp, _vp, _vp, _vp]),
    "slm_batch_decode_layers": (C.c_int, [_vp, _i32, _i32, _vp]),
    "slm_batch_decode_layers_host": (C.c_int, [_vp, _i32, _i32, _vp, _vp, _vp, _vp]),
    "slm_batch_append_layer": (C.c_int, [_vp, _i32, _vp, _vp, _i32]),
    "slm_batch_prefill_attention": (C.c_int, [_vp, _i32, _vp, _i32, _vp]),
    "slm_batch_attention_exact": (C.c_int, [_vp, _i32, _vp, _i32, _vp]),
    "slm_batch_decode_layer_exact": (C.c_int, [_vp, _i32, _vp, _vp, _vp, _vp]),
    "slm_batch_end": (C.c_int, [_vp, _pi32]),
    "slm_batch_rollback": (C.c_int, [_vp]),
    "slm_batch_submit": (C.c_int, [_vp]),
    "slm_batch_wait": (C.c_int, [_vp, _pi32]),
    "slm_prefix_attach": (C.c_int, [_vp, _i32, _pu32, _i32, _pi32]),
    "slm_prefix_publish": (C.c_int, [_vp, _i32, _pu32, _i32, _pi32]),
    "slm_pool_stats": (C.c_int, [_vp, _pi32, _pi32]),
    "slm_pool_shuffle": (C.c_int, [_vp, _u64]),
    "slm_ctx_config": (C.c_int, [_vp, C.POINTER(SlmConfig)]),
    "slm_sched_create": (C.c_int, [_vp, C.POINTER(SchedConfig), C.POINTER(_vp)]),
    "slm_sched_destroy": (C.c_int, [_vp]),
    "slm_sched_submit": (C.c_int, [_vp, _i64, _i32, _i32]),
    "slm_sched_plan": (C.c_int, [_vp, _pi32, _pi32, _pi32, _pi32, _pi32]),
    "slm_sched_commit": (C.c_int, [_vp, _pi32, _pi32, _pi32, C.POINTER(_i64), _pi32, _pi32]),
    "slm_sched_counts": (C.c_int, [_vp, _pi32, _pi32, C.POINTER(_i64), C.POINTER(_i64)]),
    "slm_sched_plan_requests": (C.c_int, [_vp, C.POINTER(_i64), _pi32, C.POINTER(_i64), _pi32]),
    "slm_decode_attention_noalloc": (
        C.c_int, [_vp, _vp, _i32, _i32, _i32, _pi32, _i32, _pi32, _i32, _vp, _vp, _vp]),
    "slm_model_create": (C.c_int, [_vp, C.POINTER(ModelConfig), C.POINTER(_vp), _i32,
                                   C.POINTER(_vp)]),
    "slm_model_destroy": (C.c_int, [_vp]),
    "slm_model_set_exact_rows": (C.c_int, [_vp, _i32]),
    "slm_model_decode": (C.c_int, [_vp, _vp, _vp, _vp, _vp]),
    "slm_model_prefill": (C.c_int, [_vp, _vp, _vp, _vp, _vp]),
    "slm_model_load_safetensors": (C.c_int, [_vp, C.POINTER(ModelConfig), C.c_char_p, _i64,
                                             C.POINTER(_vp)]),
    "slm_safetensors_check": (C.c_int, [C.POINTER(ModelConfig), _i32, _i32, _i32, C.c_char_p,
                                        _i64, C.POINTER(_i64)]),
}

_lib = None


def build() -> None:
    """Compile libslmkv.so for sm_100a with the committed Makefile."""
    import subprocess

    subprocess.run(["make", "-s", "-C", str(CSRC)], check=True)


def lib() -> C.CDLL:
    """Load the in-tree library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `make -C {CSRC}` "
                "(there is no CPU fallback)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _i32_array(values: Sequence[int]):
    arr = (C.c_int32 * max(1, len(values)))(*[int(v) for v in values])
    return arr


def _u32_array(values: Sequence[int]):
    return (C.c_uint32 * max(1, len(values)))(*[int(v) for v in values])


def _stream_ptr(stream=None):
    import torch

    if stream is None and not torch.cuda.is_available():
        return C.c_void_p(0)  # host-only pools: the library rejects compute calls
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _ptr(t) -> C.c_void_p:
    if t is None:
        return C.c_void_p(0)
    import torch

    if not isinstance(t, torch.Tensor):
        raise TypeError("expected a torch tensor")
    if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
        raise InvalidInput(ERR_INVALID_INPUT,
                           "invalid input for slmkv: tensors must be contiguous CUDA float32")
    return C.c_void_p(t.data_ptr())


class KvPool:
    """One GPU's paged KV pool (an ``slm_ctx``): the storage that every
    ``KvCache`` of this device lives in."""

    def __init__(self, *, num_layers: int, num_query_heads: int, num_key_value_heads: int,
                 head_dimension: int = 64, context_length: int, rope_theta: float = 10000.0,
                 num_blocks: int, max_sequences: int, kv_dtype: int = KV_F32,
                 device: int | None = 0):
        self.config = SlmConfig(num_layers, num_query_heads, num_key_value_heads,
                                head_dimension, context_length, rope_theta, num_blocks,
                                max_sequences, kv_dtype)
        self.device = -1 if device is None else int(device)
        h = C.c_void_p()
        rc = lib().slm_create(C.byref(self.config), self.device, C.byref(h))
        if rc != OK:
            msg = (lib().slm_last_error(None) or b"").decode()
            raise _error_class(rc)(rc, msg)
        self._h = h
        self._batch = None

    @classmethod
    def from_model_config(cls, cfg: dict, *, num_blocks: int, max_sequences: int,
                          kv_dtype: int = KV_F32, device: int | None = 0) -> "KvPool":
        """Builds a pool from a reference model config dict (configs/model.json)."""
        return cls(num_layers=cfg["num_layers"], num_query_heads=cfg["num_query_heads"],
                   num_key_value_heads=cfg["num_key_value_heads"],
                   head_dimension=cfg["head_dimension"], context_length=cfg["context_length"],
                   rope_theta=cfg["rope_theta"], num_blocks=num_blocks,
                   max_sequences=max_sequences, kv_dtype=kv_dtype, device=device)

    # -- plumbing -----------------------------------------------------------
    @property
    def handle(self) -> C.c_void_p:
        if self._h is None:
            raise InvalidInput(ERR_INVALID_INPUT, "invalid input for slmkv: pool is closed")
        return self._h

    def check(self, rc: int) -> None:
        if rc != OK:
            msg = (lib().slm_last_error(self._h) or b"").decode()
            raise _error_class(rc)(rc, msg)

    def close(self) -> None:
        if getattr(self, "_h", None) is not None:
            lib().slm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def num_layers(self) -> int:
        return self.config.num_layers

    @property
    def kv_heads(self) -> int:
        return self.config.num_key_value_heads

    @property
    def q_heads(self) -> int:
        return self.config.num_query_heads

    @property
    def head_dim(self) -> int:
        return self.config.head_dimension

    def device_bytes(self) -> int:
        v = C.c_int64()
        self.check(lib().slm_device_bytes(self.handle, C.byref(v)))
        return v.value

    def launch_count(self) -> int:
        """Kernels this pool has launched (counted by the library)."""
        v = C.c_int64()
        self.check(lib().slm_launch_count(self.handle, C.byref(v)))
        return v.value

    def stats(self) -> tuple[int, int]:
        """(free blocks, blocks held by the prefix index)."""
        f, i = C.c_int32(), C.c_int32()
        self.check(lib().slm_pool_stats(self.handle, C.byref(f), C.byref(i)))
        return f.value, i.value

    def shuffle(self, seed: int) -> None:
        self.check(lib().slm_pool_shuffle(self.handle, C.c_uint64(seed)))

    # -- sequences ------------------------------------------------------------
    def allocate_kv_cache(self, max_sequence_length: int) -> "KvCache":
        """SmallLMModel::allocate_kv_cache (model.rs:64-67)."""
        return KvCache(self, max_sequence_length)

    def begin(self, caches: Sequence["KvCache"], token_counts: Sequence[int] | int = 1,
              stream=None) -> "Batch":
        return Batch(self, caches, token_counts, stream)

    def step_plan(self, caches: Sequence["KvCache"],
                  token_counts: Sequence[int] | int = 1) -> "StepPlan":
        return StepPlan(self, caches, token_counts)

    def truncate_many(self, caches: Sequence["KvCache"], lengths: Sequence[int]) -> None:
        """truncate_all (kv_cache.rs:302-321) for many caches in one call."""
        ids = _i32_array([c.seq_id for c in caches])
        lens = _i32_array(lengths)
        self.check(lib().slm_seqs_truncate_all(self.handle, len(caches), ids, lens))


class KvCache:
    """kv_cache.rs:89-412 — one request's cache, as blocks of a ``KvPool``."""

    def __init__(self, pool: KvPool, max_sequence_length: int):
        self.pool = pool
        sid = C.c_int32()
        pool.check(lib().slm_seq_create(pool.handle, int(max_sequence_length), C.byref(sid)))
        self.seq_id = sid.value
        self.max_sequence_length = int(max_sequence_length)

    def free(self) -> None:
        if self.seq_id is not None and self.pool._h is not None:
            self.pool.check(lib().slm_seq_free(self.pool.handle, self.seq_id))
        self.seq_id = None

    def _q(self, fn, *args) -> int:
        out = C.c_int32()
        self.pool.check(fn(self.pool.handle, self.seq_id, *args, C.byref(out)))
        return out.value

    def layer_sequence_length(self, layer: int) -> int:
        return self._q(lib().slm_seq_layer_length, int(layer))

    def sequence_length(self) -> int:
        return self._q(lib().slm_seq_length)

    def is_empty(self) -> bool:
        return bool(self._q(lib().slm_seq_is_empty))

    def is_synchronized(self) -> bool:
        return bool(self._q(lib().slm_seq_is_synchronized))

    def remaining_capacity(self) -> int:
        return self._q(lib().slm_seq_remaining_capacity)

    def truncate_all(self, sequence_length: int) -> None:
        self.pool.check(lib().slm_seq_truncate_all(self.pool.handle, self.seq_id,
                                                   int(sequence_length)))

    def truncate_layer(self, layer: int, sequence_length: int) -> None:
        self.pool.check(lib().slm_seq_truncate_layer(self.pool.handle, self.seq_id, int(layer),
                                                     int(sequence_length)))

    def clear(self) -> None:
        self.pool.check(lib().slm_seq_clear(self.pool.handle, self.seq_id))

    def blocks(self) -> list[int]:
        n = C.c_int32()
        cap = self.max_sequence_length // BLOCK_TOKENS + 2
        buf = (C.c_int32 * cap)()
        self.pool.check(lib().slm_seq_blocks(self.pool.handle, self.seq_id, buf, cap,
                                             C.byref(n)))
        return list(buf[: n.value])

    def append_layer(self, layer: int, keys, values, token_count: int, *,
                     rotate_keys: bool = False, stream=None) -> None:
        """kv_cache.rs:182-230 (keys/values [T, kv_heads, d] on the device);
        with ``rotate_keys`` the keys get RoPE at their absolute positions
        first (attention.rs:422-482)."""
        p = self.pool
        if keys.numel() != token_count * p.kv_heads * p.head_dim or \
                values.numel() != token_count * p.kv_heads * p.head_dim:
            raise InvalidInput(ERR_INVALID_INPUT,
                               "invalid input for KV-cache keys: shape does not match "
                               "[token_count, kv_heads * head_dim]")
        p.check(lib().slm_append_layer(p.handle, self.seq_id, int(layer), _ptr(keys),
                                       _ptr(values), int(token_count), int(bool(rotate_keys)),
                                       _stream_ptr(stream)))

    def _gather(self, layer: int, which: str, stream=None):
        import torch

        p = self.pool
        n = self.layer_sequence_length(layer)
        out = torch.empty((n, p.kv_heads, p.head_dim), dtype=torch.float32,
                          device=f"cuda:{p.device}")
        if n:
            k = out if which == "k" else None
            v = out if which == "v" else None
            p.check(lib().slm_gather_layer(p.handle, self.seq_id, int(layer), _ptr(k), _ptr(v),
                                           _stream_ptr(stream)))
        return out

    def layer_keys(self, layer: int, stream=None):
        """kv_cache.rs:237-239 -> [len, kv_heads, d] (device)."""
        return self._gather(layer, "k", stream)

    def layer_values(self, layer: int, stream=None):
        """kv_cache.rs:246-248 -> [len, kv_heads, d] (device)."""
        return self._gather(layer, "v", stream)

    def key_head(self, layer: int, position: int, kv_head: int):
        """kv_cache.rs:256-263"""
        self._check_head(layer, position, kv_head)
        return self.layer_keys(layer)[position, kv_head]

    def value_head(self, layer: int, position: int, kv_head: int):
        """kv_cache.rs:271-278"""
        self._check_head(layer, position, kv_head)
        return self.layer_values(layer)[position, kv_head]

    def _check_head(self, layer, position, kv_head):
        n = self.layer_sequence_length(layer)
        if not 0 <= position < n:
            raise InvalidInput(ERR_INVALID_INPUT,
                               f"invalid input for KV cache: token position {position} is "
                               f"outside 0..{n}")
        if not 0 <= kv_head < self.pool.kv_heads:
            raise InvalidInput(ERR_INVALID_INPUT,
                               f"invalid input for KV cache: key/value head {kv_head} is "
                               f"outside 0..{self.pool.kv_heads}")

    def attend_cached_query(self, layer: int, query, out=None, stream=None):
        """attention.rs:677-759: rotated query [q_heads, d] -> [q_heads * d]."""
        import torch

        p = self.pool
        if out is None:
            out = torch.empty(p.q_heads * p.head_dim, dtype=torch.float32,
                              device=f"cuda:{p.device}")
        p.check(lib().slm_attend_cached_query(p.handle, self.seq_id, int(layer), _ptr(query),
                                              _ptr(out), _stream_ptr(stream)))
        return out

    def attach_prefix(self, tokens: Sequence[int]) -> int:
        """Attaches the longest indexed chain of full blocks matching
        ``tokens`` to this (empty) cache; returns the reused token count."""
        n = C.c_int32()
        self.pool.check(lib().slm_prefix_attach(self.pool.handle, self.seq_id,
                                                _u32_array(tokens), len(tokens), C.byref(n)))
        return n.value

    def publish_prefix(self, tokens: Sequence[int]) -> int:
        """Indexes this cache's full blocks holding ``tokens``; returns how
        many blocks of the chain are indexed."""
        n = C.c_int32()
        self.pool.check(lib().slm_prefix_publish(self.pool.handle, self.seq_id,
                                                 _u32_array(tokens), len(tokens), C.byref(n)))
        return n.value


class _Fast:
    """ctypes entry points bound once, for the per-step calls."""

    def __init__(self):
        self._bound = False

    def bind(self):
        L = lib()
        self.begin = L.slm_batch_begin
        self.decode = L.slm_batch_decode_layer
        self.decode_many = L.slm_batch_decode_layers
        self.decode_host = L.slm_batch_decode_layers_host
        self.end = L.slm_batch_end
        self.submit = L.slm_batch_submit
        self.wait = L.slm_batch_wait
        self.truncate = L.slm_seqs_truncate_all
        self._bound = True

    def __getattr__(self, name):
        if name.startswith("_"):
            raise AttributeError(name)
        self.bind()
        return object.__getattribute__(self, name)


_fast = _Fast()


class Batch:
    """One step over many caches (``slm_batch_*``). Use as a context manager:
    leaving the block normally ends (commits) it, an exception rolls it back."""

    def __init__(self, pool: KvPool, caches: Sequence[KvCache],
                 token_counts: Sequence[int] | int = 1, stream=None, *, _arrays=None,
                 _stream=None):
        self.pool = pool
        self.caches = caches if _arrays is not None else list(caches)
        n = len(self.caches)
        if _arrays is not None:
            self._ids, self._counts, self._status, self.token_counts = _arrays
        else:
            if isinstance(token_counts, int):
                token_counts = [token_counts] * n
            self.token_counts = [int(t) for t in token_counts]
            self._ids = _i32_array([c.seq_id for c in self.caches])
            self._counts = _i32_array(self.token_counts)
            self._status = (C.c_int32 * max(1, n))()
        h = C.c_void_p()
        sp = _stream if _stream is not None else _stream_ptr(stream)
        rc = _fast.begin(pool.handle, n, self._ids, self._counts, sp, C.byref(h))
        if rc:
            pool.check(rc)
        self._h = h
        self.statuses: list[int] | None = None

    @classmethod
    def for_sequences(cls, pool: KvPool, n: int, seq_ids, counts, stream=None) -> "Batch":
        """A step over n sequence ids (ctypes int32 arrays of ids and token
        counts, e.g. a Scheduler plan's), without KvCache objects."""
        b = cls.__new__(cls)
        b.pool = pool
        b.caches = [None] * n
        b._ids, b._counts = seq_ids, counts
        b._status = (C.c_int32 * max(1, n))()
        b.token_counts = None
        h = C.c_void_p()
        rc = _fast.begin(pool.handle, n, seq_ids, counts, _stream_ptr(stream), C.byref(h))
        if rc:
            pool.check(rc)
        b._h = h
        b.statuses = None
        return b

    def decode_layer(self, layer: int, query, keys, values, out) -> None:
        self.pool.check(lib().slm_batch_decode_layer(self._h, int(layer), _ptr(query),
                                                     _ptr(keys), _ptr(values), _ptr(out)))

    def decode_layer_ptr(self, layer: int, query: int, keys: int, values: int, out: int) -> None:
        """decode_layer with raw device addresses (for callers that checked
        their tensors once, e.g. a serving loop's persistent buffers)."""
        rc = _fast.decode(self._h, layer, query, keys, values, out)
        if rc:
            self.pool.check(rc)

    def decode_layers(self, first_layer: int, layers) -> None:
        """slm_batch_decode_layers: decode_layer for layers first_layer, ...
        with one (query, keys, values, out) tuple of tensors per layer, all
        inputs ready; up to eight layers run as one launch."""
        arr = layer_io_array([tuple(_ptr(t).value for t in io) for io in layers])
        self.decode_layers_array(first_layer, len(layers), arr)

    def decode_layers_array(self, first_layer: int, n_layers: int, arr) -> None:
        """decode_layers with a prebuilt layer_io_array of device addresses."""
        rc = _fast.decode_many(self._h, first_layer, n_layers, arr)
        if rc:
            self.pool.check(rc)

    def decode_layers_host(self, first_layer: int, n_layers: int, query, keys, values, out) -> None:
        """slm_batch_decode_layers_host: the step's inputs and outputs in host
        memory (contiguous CPU float32 tensors, pinned for the copies to
        overlap; query/out [n_layers, n, q_heads, 64], keys/values [n_layers,
        n, kv_heads, 64]). `out` is complete once this batch's end() / wait()
        has returned; the tensors must live until then."""
        ptrs = []
        for t in (query, keys, values, out):
            if t.is_cuda or not t.is_contiguous() or str(t.dtype) != "torch.float32":
                raise InvalidInput(ERR_INVALID_INPUT, "invalid input for slmkv: host buffers must "
                                   "be contiguous CPU float32 tensors")
            ptrs.append(C.c_void_p(t.data_ptr()))
        self.decode_layers_host_ptr(first_layer, n_layers, *ptrs)

    def decode_layers_host_ptr(self, first_layer: int, n_layers: int, query, keys, values,
                               out) -> None:
        """decode_layers_host with raw host addresses."""
        rc = _fast.decode_host(self._h, first_layer, n_layers, query, keys, values, out)
        if rc:
            self.pool.check(rc)

    def append_layer(self, layer: int, keys, values, rotate_keys: bool = True) -> None:
        self.pool.check(lib().slm_batch_append_layer(self._h, int(layer), _ptr(keys),
                                                     _ptr(values), int(bool(rotate_keys))))

    def prefill_attention(self, layer: int, query, out, rotate_query: bool = True) -> None:
        self.pool.check(lib().slm_batch_prefill_attention(self._h, int(layer), _ptr(query),
                                                          int(bool(rotate_query)), _ptr(out)))

    def decode_layer_exact(self, layer: int, query, keys, values, out) -> None:
        """slm_batch_decode_layer_exact: decode_layer in the reference's
        operation order (attention.rs:794-810, 677-759), bit for bit; f32 pools."""
        self.pool.check(lib().slm_batch_decode_layer_exact(self._h, int(layer), _ptr(query),
                                                           _ptr(keys), _ptr(values), _ptr(out)))

    def attention_exact(self, layer: int, query, out, rotate_query: bool = True) -> None:
        """slm_batch_attention_exact: the batch's attention in the reference's
        operation order (attention.rs:195-399, 677-759), bit for bit; f32 pools."""
        self.pool.check(lib().slm_batch_attention_exact(self._h, int(layer), _ptr(query),
                                                        int(bool(rotate_query)), _ptr(out)))

    def end(self, raise_on_error: bool = True) -> list[int]:
        if self._h is None:
            return self.statuses or []
        rc = _fast.end(self._h, self._status)
        self._h = None
        self.statuses = list(self._status[: len(self.caches)])
        if rc != OK and raise_on_error:
            self.pool.check(rc)
        return self.statuses

    def submit(self) -> "Batch":
        """Closes the step without waiting for the GPU (``slm_batch_submit``):
        the next step may begin at once; ``wait()`` collects the statuses."""
        if self._h is None:
            raise EngineError("the batch is not open")
        rc = _fast.submit(self._h)
        if rc:
            # refused (too many pending): the step is still open; a CUDA
            # failure has rolled it back and closed it
            if rc != ERR_INVALID_INPUT:
                self._h = None
            self.pool.check(rc)
        self._submitted, self._h = self._h, None
        return self

    def wait(self, raise_on_error: bool = True) -> list[int]:
        """Statuses of a submitted step (``slm_batch_wait``); failed sequences
        were rolled back, and with them every later step that holds them."""
        h = getattr(self, "_submitted", None)
        if h is None:
            return self.statuses or []
        status = self._status
        rc = _fast.wait(h, status)
        self._submitted = None
        self.statuses = list(status[: len(self.caches)])
        if rc != OK and raise_on_error:
            self.pool.check(rc)
        return self.statuses

    def rollback(self) -> None:
        if self._h is not None:
            rc = lib().slm_batch_rollback(self._h)
            self._h = None
            self.pool.check(rc)

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb):
        if exc_type is None:
            self.end()
        else:
            self.rollback()


class StepPlan:
    """A fixed set of caches stepped repeatedly (a running batch): the id,
    count and status arrays handed to the library are built once."""

    def __init__(self, pool: KvPool, caches: Sequence[KvCache],
                 token_counts: Sequence[int] | int = 1):
        self.pool = pool
        self.caches = list(caches)
        n = len(self.caches)
        if isinstance(token_counts, int):
            token_counts = [token_counts] * n
        self.token_counts = [int(t) for t in token_counts]
        self._ids = _i32_array([c.seq_id for c in self.caches])
        self._counts = _i32_array(self.token_counts)
        self._status = (C.c_int32 * max(1, n))()
        self._stream = None  # the stream of the first begin(), reused after

    def begin(self, stream=None) -> Batch:
        """Opens the step on `stream` (default: torch's current stream at the
        plan's first step, remembered for the following steps)."""
        if stream is not None:
            sp = _stream_ptr(stream)
        else:
            if self._stream is None:
                self._stream = _stream_ptr(None)
            sp = self._stream
        return Batch(self.pool, self.caches, _stream=sp,
                     _arrays=(self._ids, self._counts, self._status, self.token_counts))

    def lengths(self, lengths: Sequence[int]):
        """A reusable length array for truncate_all."""
        return _i32_array(lengths)

    def truncate_all(self, lengths) -> None:
        """truncate_all (kv_cache.rs:302-321) for every cache of the plan;
        `lengths` is a sequence or an array from `lengths()`."""
        arr = lengths if isinstance(lengths, C.Array) else _i32_array(lengths)
        rc = _fast.truncate(self.pool.handle, len(self.caches), self._ids, arr)
        if rc:
            self.pool.check(rc)


def decode_attention_noalloc(key_pool, value_pool, block_table, lengths, query, out=None,
                             stream=None):
    """slm_decode_attention_noalloc: attend_cached_query (attention.rs:677-759)
    for n sequences of a caller-owned paged f32 cache, without any device
    allocation by the library (for engines that own all device memory as one
    arena, and plugins in hosts that forbid new device allocations).

    key_pool/value_pool: CUDA [num_blocks, kv_heads, 16, 64]; block_table:
    host int32 [n, max_blocks]; lengths: host int32 [n]; query: CUDA
    [n, q_heads, 64], rotated. Returns out [n, q_heads, 64]."""
    import numpy as np
    import torch

    def bad(msg):
        return InvalidInput(ERR_INVALID_INPUT,
                            f"invalid input for slm_decode_attention_noalloc: {msg}")

    table = np.ascontiguousarray(block_table, dtype=np.int32)
    lens = np.ascontiguousarray(lengths, dtype=np.int32)
    if key_pool.dim() != 4 or tuple(key_pool.shape[2:]) != (BLOCK_TOKENS, 64):
        raise bad("key pool must be [num_blocks, kv_heads, 16, 64]")
    if tuple(value_pool.shape) != tuple(key_pool.shape):
        raise bad("value pool must have the key pool's shape")
    if query.dim() != 3 or int(query.shape[2]) != 64:
        raise bad("query must be [n, q_heads, 64]")
    nb, hkv = int(key_pool.shape[0]), int(key_pool.shape[1])
    n, hq = int(query.shape[0]), int(query.shape[1])
    if table.ndim != 2 or table.shape[0] != n or lens.shape != (n,):
        raise bad(f"block table must be [{n}, max_blocks] and lengths [{n}]")
    if out is None:
        out = torch.empty_like(query)
    if tuple(out.shape) != tuple(query.shape):
        raise bad("out must have the query's shape")
    dev = torch.cuda.current_device()
    for name, t in (("key pool", key_pool), ("value pool", value_pool), ("query", query),
                    ("out", out)):
        if not t.is_cuda or t.device.index != dev or t.dtype != torch.float32 \
                or not t.is_contiguous():
            raise bad(f"{name} must be a contiguous f32 tensor on the current device")
    rc = lib().slm_decode_attention_noalloc(
        _ptr(key_pool), _ptr(value_pool), nb, hq, hkv,
        table.ctypes.data_as(_pi32), int(table.shape[1]), lens.ctypes.data_as(_pi32), n,
        _ptr(query), _ptr(out), _stream_ptr(stream))
    if rc != OK:
        msg = (lib().slm_last_error(None) or b"").decode()
        raise _error_class(rc)(rc, msg)
    return out


def _ptr_i32(t) -> C.c_void_p:
    """Device pointer of a contiguous CUDA int32 tensor (None -> NULL)."""
    if t is None:
        return C.c_void_p(0)
    import torch

    if not isinstance(t, torch.Tensor) or t.dtype != torch.int32 or not t.is_cuda \
            or not t.is_contiguous():
        raise InvalidInput(ERR_INVALID_INPUT,
                           "invalid input for slmkv: token ids must be a contiguous CUDA int32 tensor")
    return C.c_void_p(t.data_ptr())


class Model:
    """SmallLMModel (model.rs) on one pool's device: its cached decode step
    and prompt prefill run through an open ``Batch`` of that pool.

    ``tensors``: fp32 host arrays in the reference layout and order
    (``MODEL_TENSOR_ORDER``): token_embedding; per layer attention_norm, q, k,
    v, o, ffn_norm, gate, up, down; final_norm."""

    def __init__(self, pool: KvPool, *, vocab_size: int, intermediate_size: int,
                 tensors=None, rms_norm_epsilon: float = 1e-5, situ_beta_gate: float = 4.0,
                 situ_beta_up: float = 25.0, _handle=None):
        import numpy as np

        self.pool = pool
        self.vocab_size = vocab_size
        if _handle is not None:
            self._h = _handle
            return
        cfg = ModelConfig(vocab_size, pool.q_heads * pool.head_dim, intermediate_size,
                          rms_norm_epsilon, situ_beta_gate, situ_beta_up)
        keep = [np.ascontiguousarray(np.asarray(t, dtype=np.float32)) for t in tensors]
        arr = (_vp * len(keep))(*[C.c_void_p(a.ctypes.data) for a in keep])
        h = _vp()
        pool.check(lib().slm_model_create(pool.handle, C.byref(cfg), arr, len(keep), C.byref(h)))
        self._h = h

    @classmethod
    def from_safetensors(cls, pool: KvPool, path, *, vocab_size: int, intermediate_size: int,
                         expected_parameter_count: int = 0, rms_norm_epsilon: float = 1e-5,
                         situ_beta_gate: float = 4.0, situ_beta_up: float = 25.0) -> "Model":
        """ModelWeights::load (weights.rs:117-190) straight into the device model."""
        cfg = ModelConfig(vocab_size, pool.q_heads * pool.head_dim, intermediate_size,
                          rms_norm_epsilon, situ_beta_gate, situ_beta_up)
        h = _vp()
        pool.check(lib().slm_model_load_safetensors(pool.handle, C.byref(cfg),
                                                    str(path).encode(), expected_parameter_count,
                                                    C.byref(h)))
        return cls(pool, vocab_size=vocab_size, intermediate_size=intermediate_size, _handle=h)

    def set_exact_rows(self, max_rows: int) -> None:
        """Steps of up to ``max_rows`` token rows (0..1024) project in the
        reference's accumulation order (linear.rs:98-103); larger steps, or
        all when 0, on tensor-core GEMMs."""
        self.pool.check(lib().slm_model_set_exact_rows(self._h, int(max_rows)))

    def decode(self, batch: "Batch", token_ids, logits=None, next_tokens=None) -> None:
        """model.rs:342-397 for every sequence of ``batch`` (counts 1):
        token_ids [n] CUDA int32; logits [n, vocab] CUDA float32 and
        next_tokens [n] CUDA int32 are optional outputs."""
        self.pool.check(lib().slm_model_decode(self._h, batch._h, _ptr_i32(token_ids),
                                               _ptr(logits), _ptr_i32(next_tokens)))

    def prefill(self, batch: "Batch", token_ids, logits=None, next_tokens=None) -> None:
        """model.rs:297-330 for every sequence of ``batch``: token_ids
        [sum(counts)] in batch order; logits / next token of each sequence's
        last position ([n, vocab], [n])."""
        self.pool.check(lib().slm_model_prefill(self._h, batch._h, _ptr_i32(token_ids),
                                                _ptr(logits), _ptr_i32(next_tokens)))

    def close(self) -> None:
        if getattr(self, "_h", None) is not None:
            lib().slm_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def check_safetensors(path, *, vocab_size: int, hidden_size: int, intermediate_size: int,
                      num_layers: int, num_key_value_heads: int, head_dimension: int = 64,
                      expected_parameter_count: int = 0) -> int:
    """The checks of ModelWeights::load (weights.rs:117-190) without a device;
    returns the parameter count, raises InvalidInput with the reason."""
    cfg = ModelConfig(vocab_size, hidden_size, intermediate_size, 1e-5, 4.0, 25.0)
    n = _i64()
    rc = lib().slm_safetensors_check(C.byref(cfg), num_layers, num_key_value_heads,
                                     head_dimension, str(path).encode(), expected_parameter_count,
                                     C.byref(n))
    if rc != OK:
        raise _error_class(rc)(rc, (lib().slm_last_error(None) or b"").decode())
    return int(n.value)


MODEL_TENSOR_ORDER = ("attention_norm", "q_proj", "k_proj", "v_proj", "o_proj", "ffn_norm",
                      "gate_proj", "up_proj", "down_proj")


def model_tensor_shapes(*, vocab_size: int, hidden_size: int, intermediate_size: int,
                        num_layers: int, kv_width: int):
    """Names and shapes in the order the model takes them (weights.rs:347-375)."""
    out = [("token_embedding.weight", (vocab_size, hidden_size))]
    for layer in range(num_layers):
        shapes = {"attention_norm": (hidden_size,), "q_proj": (hidden_size, hidden_size),
                  "k_proj": (kv_width, hidden_size), "v_proj": (kv_width, hidden_size),
                  "o_proj": (hidden_size, hidden_size), "ffn_norm": (hidden_size,),
                  "gate_proj": (intermediate_size, hidden_size),
                  "up_proj": (intermediate_size, hidden_size),
                  "down_proj": (hidden_size, intermediate_size)}
        out += [(f"layers.{layer}.{n}.weight", shapes[n]) for n in MODEL_TENSOR_ORDER]
    out.append(("final_norm.weight", (hidden_size,)))
    return out


class Scheduler:
    """Continuous batching over one pool (``slm_sched_*``): requests are
    admitted in arrival order, every step plans a decode token for each
    request whose prompt is cached and prompt chunks for the others, and the
    caller runs the step's KV batches and commits their statuses. The pool
    belongs to the scheduler while it runs."""

    def __init__(self, pool: KvPool, *, max_running: int, max_prefill_tokens: int):
        self.pool = pool
        h = C.c_void_p()
        cfg = SchedConfig(int(max_running), int(max_prefill_tokens))
        pool.check(lib().slm_sched_create(pool.handle, C.byref(cfg), C.byref(h)))
        self._h = h
        self.max_running = min(int(max_running), pool.config.max_sequences)
        n = max(1, self.max_running)
        self._dseq, self._pseq, self._pcnt = (C.c_int32 * n)(), (C.c_int32 * n)(), (C.c_int32 * n)()
        self._fid, self._fst, self._fgen = (C.c_int64 * n)(), (C.c_int32 * n)(), (C.c_int32 * n)()
        self._dreq, self._preq = (C.c_int64 * n)(), (C.c_int64 * n)()
        self._dpos, self._ppos = (C.c_int32 * n)(), (C.c_int32 * n)()
        self._nd, self._np, self._nf = C.c_int32(), C.c_int32(), C.c_int32()

    def close(self) -> None:
        if self._h is not None:
            lib().slm_sched_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def submit(self, request_id: int, prompt_len: int, max_new_tokens: int) -> None:
        self.pool.check(lib().slm_sched_submit(self._h, int(request_id), int(prompt_len),
                                               int(max_new_tokens)))

    def plan(self):
        """(decode_seq, prefill_seq, prefill_count) of the next step: ctypes
        int32 arrays valid until the next plan, and their lengths."""
        self.pool.check(lib().slm_sched_plan(self._h, C.byref(self._nd), self._dseq,
                                             C.byref(self._np), self._pseq, self._pcnt))
        return self._nd.value, self._np.value

    def decode_seqs(self) -> list[int]:
        return list(self._dseq[: self._nd.value])

    def prefill_seqs(self) -> list[tuple[int, int]]:
        return list(zip(self._pseq[: self._np.value], self._pcnt[: self._np.value]))

    def plan_requests(self):
        """The requests behind the last plan: (decode [(request, pos)],
        prefill [(request, pos)]); a decode entry feeds the token at `pos`, a
        prefill entry positions pos .. pos + count - 1."""
        self.pool.check(lib().slm_sched_plan_requests(self._h, self._dreq, self._dpos,
                                                      self._preq, self._ppos))
        nd, np_ = self._nd.value, self._np.value
        return (list(zip(self._dreq[:nd], self._dpos[:nd])),
                list(zip(self._preq[:np_], self._ppos[:np_])))

    def plan_request_arrays(self):
        """plan_requests as numpy views (valid until the next plan): decode
        request ids and positions, prefill request ids and first positions."""
        import numpy as np

        self.pool.check(lib().slm_sched_plan_requests(self._h, self._dreq, self._dpos,
                                                      self._preq, self._ppos))
        nd, np_ = self._nd.value, self._np.value
        return (np.ctypeslib.as_array(self._dreq)[:nd], np.ctypeslib.as_array(self._dpos)[:nd],
                np.ctypeslib.as_array(self._preq)[:np_], np.ctypeslib.as_array(self._ppos)[:np_])

    def commit(self, decode_status=None, prefill_status=None) -> list[tuple[int, int, int]]:
        """Commits the last plan; returns the finished requests as
        (request_id, status, output tokens)."""
        def arr(x, n):
            if n == 0:
                return None
            if x is None:
                return (C.c_int32 * n)()
            return x if isinstance(x, C.Array) else _i32_array(list(x))
        rc = lib().slm_sched_commit(self._h, arr(decode_status, self._nd.value),
                                    arr(prefill_status, self._np.value), C.byref(self._nf),
                                    self._fid, self._fst, self._fgen)
        self.pool.check(rc)
        n = self._nf.value
        return list(zip(self._fid[:n], self._fst[:n], self._fgen[:n]))

    def counts(self) -> dict:
        w, r = C.c_int32(), C.c_int32()
        pre, gen = C.c_int64(), C.c_int64()
        self.pool.check(lib().slm_sched_counts(self._h, C.byref(w), C.byref(r), C.byref(pre),
                                               C.byref(gen)))
        return {"waiting": w.value, "running": r.value, "preemptions": pre.value,
                "generated_tokens": gen.value}

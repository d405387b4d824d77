"""ctypes wrapper around the CPU oracle (``liboracle.so``).

TEST INFRASTRUCTURE ONLY: a restatement of small-lm-rs's CPU arithmetic
(``rust/engine/src/{kv_cache,rope,softmax,attention,linear}.rs``), used by the
tests, the smoke check and the bench's CPU-baseline leg as the checker. The
CUDA library and its Python mirror never import this module. The model-level
functions follow ``rmsnorm.rs``, ``situ_glu.rs``, ``embedding.rs``,
``greedy.rs``, ``transformer.rs`` and ``model.rs``.

Each method names the reference lines that the C function restates; see
``slm_oracle.c`` for the line-by-line restatement.
"""

from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

OK = 0
ERR_INVALID_CONFIGURATION = -1
ERR_INVALID_INPUT = -2
ERR_CAPACITY = -3
ERR_NON_FINITE = -4

_f32p = C.POINTER(C.c_float)
_lib = None


def build() -> None:
    """Compile liboracle.so with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        i32, i64, vp = C.c_int32, C.c_int64, C.c_void_p
        sig = {
            "orc_round_to_bfloat16": (C.c_float, [C.c_float]),
            "orc_rope_inverse_frequencies": (C.c_int, [i32, C.c_float, _f32p]),
            "orc_rope_apply_head": (C.c_int, [_f32p, i32, _f32p, i64]),
            "orc_rope_apply_heads": (C.c_int, [_f32p, i32, i32, _f32p, i64]),
            "orc_apply_rotary_with_offset": (
                C.c_int, [_f32p, _f32p, i64, i32, i32, i32, _f32p, i64]),
            "orc_softmax_in_place": (C.c_int, [_f32p, i64]),
            "orc_softmax_rows": (C.c_int, [_f32p, i64, i64]),
            "orc_cache_allocate": (vp, [i32, i32, i32, i32, i32]),
            "orc_cache_free": (None, [vp]),
            "orc_cache_append_layer": (C.c_int, [vp, i32, _f32p, _f32p, i64]),
            "orc_cache_layer_sequence_length": (i64, [vp, i32]),
            "orc_cache_sequence_length": (i64, [vp]),
            "orc_cache_is_empty": (i32, [vp]),
            "orc_cache_is_synchronized": (i32, [vp]),
            "orc_cache_remaining_capacity": (i64, [vp]),
            "orc_cache_truncate_all": (C.c_int, [vp, i64]),
            "orc_cache_truncate_layer": (C.c_int, [vp, i32, i64]),
            "orc_cache_clear": (None, [vp]),
            "orc_cache_layer_keys": (C.c_int, [vp, i32, _f32p]),
            "orc_cache_layer_values": (C.c_int, [vp, i32, _f32p]),
            "orc_cache_key_head": (C.c_int, [vp, i32, i64, i32, _f32p]),
            "orc_cache_value_head": (C.c_int, [vp, i32, i64, i32, _f32p]),
            "orc_attend_cached_query": (C.c_int, [vp, i32, _f32p, i32, _f32p]),
            "orc_forward_cached_attention": (
                C.c_int, [vp, i32, _f32p, _f32p, _f32p, i32, _f32p, _f32p]),
            "orc_forward_cached_attention_batch": (
                C.c_int, [C.POINTER(vp), i32, i32, _f32p, _f32p, _f32p, i32, _f32p,
                          _f32p, i32]),
            "orc_scaled_causal_scores": (C.c_int, [_f32p, _f32p, i64, i32, i32, i32, _f32p]),
            "orc_causal_probabilities": (C.c_int, [_f32p, _f32p, i64, i32, i32, i32, _f32p]),
            "orc_attend_values": (C.c_int, [_f32p, _f32p, i64, i32, i32, i32, _f32p]),
            "orc_linear": (C.c_int, [_f32p, i64, i64, _f32p, i64, _f32p, i32]),
            "orc_linear_fp32": (C.c_int, [_f32p, i64, i64, _f32p, i64, _f32p, i32]),
            "orc_max_threads": (i32, []),
            "orc_rmsnorm_rows": (C.c_int, [_f32p, i64, i64, _f32p, C.c_float, _f32p]),
            "orc_situ_gate_activation": (C.c_float, [C.c_float, C.c_float]),
            "orc_situ_up_activation": (C.c_float, [C.c_float, C.c_float]),
            "orc_situ_glu": (C.c_int, [_f32p, i64, i64, i64, _f32p, _f32p, _f32p, C.c_float,
                                       C.c_float, _f32p, i32]),
            "orc_embedding_lookup": (C.c_int, [C.POINTER(C.c_uint32), i64, _f32p, i64, i64,
                                               _f32p]),
            "orc_argmax_finite": (C.c_int, [_f32p, i64, C.POINTER(C.c_uint32)]),
            "orc_model_tensor_count": (i32, [i32]),
            "orc_model_prefill": (C.c_int, [vp, C.POINTER(_f32p), vp, C.POINTER(C.c_uint32),
                                            i64, _f32p, i32]),
            "orc_model_decode": (C.c_int, [vp, C.POINTER(_f32p), vp, C.c_uint32, _f32p, i32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(_f32p)


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


class OracleError(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what}: oracle status {code}")
        self.code = code


def _check(rc: int, what: str) -> None:
    if rc != OK:
        raise OracleError(rc, what)


# --- scalar helpers ---------------------------------------------------------

def round_to_bfloat16(x: float) -> float:
    """linear.rs:14-23"""
    return float(lib().orc_round_to_bfloat16(float(x)))


def round_to_bfloat16_array(a: np.ndarray) -> np.ndarray:
    """Vectorised restatement of linear.rs:14-23 (same bit arithmetic)."""
    a = f32(a)
    bits = a.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32).view(np.float32)
    return np.where(np.isfinite(a), rounded, a).astype(np.float32)


def rope_inverse_frequencies(head_dim: int, theta: float) -> np.ndarray:
    """rope.rs:33-36"""
    out = np.zeros(head_dim // 2 if head_dim > 0 else 1, np.float32)
    _check(lib().orc_rope_inverse_frequencies(head_dim, theta, _p(out)), "inv_freq")
    return out


def rope_apply_head(head, inv_freq: np.ndarray, position: int) -> np.ndarray:
    """rope.rs:82-100 (returns a rotated copy)."""
    h = f32(head).copy()
    _check(lib().orc_rope_apply_head(_p(h), h.size, _p(f32(inv_freq)), position), "rope")
    return h


def rope_apply_heads(values, num_heads: int, head_dim: int, inv_freq, position: int):
    """rope.rs:108-134"""
    v = f32(values).copy()
    if v.size != num_heads * head_dim:
        raise OracleError(ERR_INVALID_INPUT, "rope heads shape")
    _check(lib().orc_rope_apply_heads(_p(v), num_heads, head_dim, _p(f32(inv_freq)),
                                      position), "rope heads")
    return v


def apply_rotary_with_offset(query, key, q_heads, kv_heads, head_dim, inv_freq, offset):
    """attention.rs:422-482 on [T, H, d] copies of query and key."""
    q = f32(query).copy()
    k = f32(key).copy()
    T = q.size // (q_heads * head_dim)
    _check(lib().orc_apply_rotary_with_offset(_p(q), _p(k), T, q_heads, kv_heads, head_dim,
                                              _p(f32(inv_freq)), offset), "rotary")
    return q, k


def softmax(values) -> np.ndarray:
    """softmax.rs:12-45"""
    v = f32(values).copy()
    _check(lib().orc_softmax_in_place(_p(v), v.size), "softmax")
    return v


def softmax_rows(values, rows: int, columns: int) -> np.ndarray:
    """softmax.rs:53-59"""
    v = f32(values).copy()
    if v.size != rows * columns:
        raise OracleError(ERR_INVALID_INPUT, "softmax shape")
    _check(lib().orc_softmax_rows(_p(v), rows, columns), "softmax rows")
    return v


def causal_scores(query, key, q_heads, kv_heads, head_dim):
    """attention.rs:195-245 -> [q_heads, T, T]"""
    q, k = f32(query), f32(key)
    T = q.size // (q_heads * head_dim)
    out = np.zeros(q_heads * T * T, np.float32)
    _check(lib().orc_scaled_causal_scores(_p(q), _p(k), T, q_heads, kv_heads, head_dim,
                                          _p(out)), "scores")
    return out


def causal_probabilities(query, key, q_heads, kv_heads, head_dim):
    """attention.rs:256-269"""
    q, k = f32(query), f32(key)
    T = q.size // (q_heads * head_dim)
    out = np.zeros(q_heads * T * T, np.float32)
    _check(lib().orc_causal_probabilities(_p(q), _p(k), T, q_heads, kv_heads, head_dim,
                                          _p(out)), "probabilities")
    return out


def attend_values(probabilities, value, q_heads, kv_heads, head_dim):
    """attention.rs:282-399 -> [T, q_heads, d]"""
    p, v = f32(probabilities), f32(value)
    T = v.size // (kv_heads * head_dim)
    out = np.zeros(T * q_heads * head_dim, np.float32)
    _check(lib().orc_attend_values(_p(p), _p(v), T, q_heads, kv_heads, head_dim, _p(out)),
           "attend values")
    return out


def prefill_attention(query_rot, key_rot, value, q_heads, kv_heads, head_dim):
    """attention.rs:860-861: causal_probabilities then attend_values."""
    probs = causal_probabilities(query_rot, key_rot, q_heads, kv_heads, head_dim)
    return attend_values(probs, value, q_heads, kv_heads, head_dim)


def linear(x, rows, in_features, weight, out_features, threads=1):
    """linear.rs:44-107"""
    out = np.zeros(rows * out_features, np.float32)
    _check(lib().orc_linear(_p(f32(x)), rows, in_features, _p(f32(weight)), out_features,
                            _p(out), threads), "linear")
    return out


def linear_fp32(x, rows, in_features, weight, out_features, threads=1):
    """linear.rs:119-152"""
    out = np.zeros(rows * out_features, np.float32)
    _check(lib().orc_linear_fp32(_p(f32(x)), rows, in_features, _p(f32(weight)),
                                 out_features, _p(out), threads), "linear_fp32")
    return out


def max_threads() -> int:
    return int(lib().orc_max_threads())


class DenseCache:
    """kv_cache.rs:89-412: dense [layers][max_seq][kv_heads][d] fp32 cache.

    ``quantize_bf16`` stores appended values through round_to_bfloat16
    (linear.rs:14-23); the reference itself only stores fp32.
    """

    def __init__(self, num_layers, max_sequence_length, kv_heads, head_dim,
                 quantize_bf16=False):
        self.num_layers, self.kv_heads, self.head_dim = num_layers, kv_heads, head_dim
        self.max_sequence_length = max_sequence_length
        self._h = lib().orc_cache_allocate(num_layers, max_sequence_length, kv_heads,
                                           head_dim, int(bool(quantize_bf16)))
        if not self._h:
            raise OracleError(ERR_INVALID_CONFIGURATION, "allocate")

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib().orc_cache_free(h)
            self._h = None

    @property
    def handle(self):
        return self._h

    def append_layer(self, layer, keys, values, token_count):
        _check(lib().orc_cache_append_layer(self._h, layer, _p(f32(keys)), _p(f32(values)),
                                            token_count), "append_layer")

    def layer_sequence_length(self, layer):
        n = lib().orc_cache_layer_sequence_length(self._h, layer)
        _check(0 if n >= 0 else int(n), "layer_sequence_length")
        return int(n)

    def sequence_length(self):
        return int(lib().orc_cache_sequence_length(self._h))

    def is_empty(self):
        return bool(lib().orc_cache_is_empty(self._h))

    def is_synchronized(self):
        return bool(lib().orc_cache_is_synchronized(self._h))

    def remaining_capacity(self):
        return int(lib().orc_cache_remaining_capacity(self._h))

    def truncate_all(self, n):
        _check(lib().orc_cache_truncate_all(self._h, n), "truncate_all")

    def truncate_layer(self, layer, n):
        _check(lib().orc_cache_truncate_layer(self._h, layer, n), "truncate_layer")

    def clear(self):
        lib().orc_cache_clear(self._h)

    def layer_keys(self, layer):
        n = self.layer_sequence_length(layer)
        out = np.zeros((n, self.kv_heads, self.head_dim), np.float32)
        _check(lib().orc_cache_layer_keys(self._h, layer, _p(out)), "layer_keys")
        return out

    def layer_values(self, layer):
        n = self.layer_sequence_length(layer)
        out = np.zeros((n, self.kv_heads, self.head_dim), np.float32)
        _check(lib().orc_cache_layer_values(self._h, layer, _p(out)), "layer_values")
        return out

    def key_head(self, layer, position, kv_head):
        out = np.zeros(self.head_dim, np.float32)
        _check(lib().orc_cache_key_head(self._h, layer, position, kv_head, _p(out)),
               "key_head")
        return out

    def value_head(self, layer, position, kv_head):
        out = np.zeros(self.head_dim, np.float32)
        _check(lib().orc_cache_value_head(self._h, layer, position, kv_head, _p(out)),
               "value_head")
        return out

    def attend_cached_query(self, layer, query, q_heads):
        """attention.rs:677-759"""
        out = np.zeros(q_heads * self.head_dim, np.float32)
        _check(lib().orc_attend_cached_query(self._h, layer, _p(f32(query)), q_heads,
                                             _p(out)), "attend_cached_query")
        return out

    def forward_cached_attention(self, layer, query, key, value, q_heads, inv_freq):
        """attention.rs:794-816; returns (out, rotated_query, rotated_key)."""
        q, k = f32(query).copy(), f32(key).copy()
        out = np.zeros(q_heads * self.head_dim, np.float32)
        _check(lib().orc_forward_cached_attention(self._h, layer, _p(q), _p(k),
                                                  _p(f32(value)), q_heads,
                                                  _p(f32(inv_freq)), _p(out)),
               "forward_cached_attention")
        return out, q, k


def forward_cached_attention_batch(caches, layer, query, key, value, q_heads, inv_freq,
                                   threads=1):
    """One decode layer for n independent sequences (each exactly as
    attention.rs:794-816), sequences spread over ``threads`` OpenMP threads."""
    n = len(caches)
    arr = (C.c_void_p * n)(*[c.handle for c in caches])
    q, k = f32(query).copy(), f32(key).copy()
    d = caches[0].head_dim
    out = np.zeros(n * q_heads * d, np.float32)
    _check(lib().orc_forward_cached_attention_batch(arr, n, layer, _p(q), _p(k),
                                                    _p(f32(value)), q_heads,
                                                    _p(f32(inv_freq)), _p(out), threads),
           "forward_cached_attention_batch")
    return out


# --- model level ------------------------------------------------------------

def rmsnorm_rows(x, rows: int, hidden: int, weight, epsilon: float) -> np.ndarray:
    """rmsnorm.rs:80-91"""
    out = np.zeros(rows * hidden, np.float32)
    _check(lib().orc_rmsnorm_rows(_p(f32(x)), rows, hidden, _p(f32(weight)), epsilon, _p(out)),
           "rmsnorm")
    return out


def situ_gate_activation(v: float, beta_gate: float) -> float:
    """situ_glu.rs:59-62 with the sigmoid of :131-138"""
    return float(lib().orc_situ_gate_activation(float(v), float(beta_gate)))


def situ_up_activation(v: float, beta_up: float) -> float:
    """situ_glu.rs:64-67"""
    return float(lib().orc_situ_up_activation(float(v), float(beta_up)))


def situ_glu(x, rows, hidden, intermediate, gate_w, up_w, down_w, beta_gate, beta_up,
             threads=1) -> np.ndarray:
    """situ_glu.rs:80-128"""
    out = np.zeros(rows * hidden, np.float32)
    _check(lib().orc_situ_glu(_p(f32(x)), rows, hidden, intermediate, _p(f32(gate_w)),
                              _p(f32(up_w)), _p(f32(down_w)), beta_gate, beta_up, _p(out),
                              threads), "situ_glu")
    return out


def embedding_lookup(token_ids, table, vocab: int, hidden: int) -> np.ndarray:
    """embedding.rs:15-56"""
    ids = np.ascontiguousarray(np.asarray(token_ids, dtype=np.uint32))
    out = np.zeros(ids.size * hidden, np.float32)
    _check(lib().orc_embedding_lookup(ids.ctypes.data_as(C.POINTER(C.c_uint32)), ids.size,
                                      _p(f32(table)), vocab, hidden, _p(out)), "embedding")
    return out


def argmax_finite(logits) -> int:
    """greedy.rs argmax_finite: the first maximum; empty or non-finite fails."""
    a = f32(logits)
    out = C.c_uint32(0)
    _check(lib().orc_argmax_finite(_p(a), a.size, C.byref(out)), "argmax")
    return int(out.value)


class _ModelConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("vocab_size", "hidden_size", "intermediate_size",
                                         "num_layers", "num_query_heads",
                                         "num_key_value_heads", "head_dimension")] + \
               [(n, C.c_float) for n in ("rms_norm_epsilon", "rope_theta", "situ_beta_gate",
                                         "situ_beta_up")]


class Model:
    """The decoder-only model (model.rs) over fp32 tensors in the reference
    layout, in the order of ``orc_model_tensor_count``: token_embedding; per
    layer attention_norm, q, k, v, o, ffn_norm, gate, up, down; final_norm."""

    def __init__(self, cfg: dict, tensors):
        self.cfg = dict(cfg)
        n = lib().orc_model_tensor_count(cfg["num_layers"])
        if len(tensors) != n:
            raise OracleError(ERR_INVALID_INPUT, f"model wants {n} tensors")
        self._keep = [f32(t) for t in tensors]
        self._arr = (_f32p * n)(*[_p(t) for t in self._keep])
        self._c = _ModelConfig(**{k: cfg[k] for k, _ in _ModelConfig._fields_})

    def new_cache(self, max_sequence_length: int, quantize_bf16=False) -> DenseCache:
        c = self.cfg
        return DenseCache(c["num_layers"], max_sequence_length, c["num_key_value_heads"],
                          c["head_dimension"], quantize_bf16)

    def prefill(self, cache: DenseCache, token_ids, threads=1) -> np.ndarray:
        """model.rs:297-330: logits [T, vocab]"""
        ids = np.ascontiguousarray(np.asarray(token_ids, dtype=np.uint32))
        out = np.zeros(ids.size * self.cfg["vocab_size"], np.float32)
        _check(lib().orc_model_prefill(C.byref(self._c), self._arr, cache.handle,
                                       ids.ctypes.data_as(C.POINTER(C.c_uint32)), ids.size,
                                       _p(out), threads), "model_prefill")
        return out.reshape(ids.size, self.cfg["vocab_size"])

    def decode(self, cache: DenseCache, token_id: int, threads=1) -> np.ndarray:
        """model.rs:342-397: logits [vocab]"""
        out = np.zeros(self.cfg["vocab_size"], np.float32)
        _check(lib().orc_model_decode(C.byref(self._c), self._arr, cache.handle,
                                      int(token_id), _p(out), threads), "model_decode")
        return out

"""Helpers shared by the GPU parity tests: seeded inputs, and building the
same cache contents in the CUDA pool and in the CPU oracle."""

from __future__ import annotations

import numpy as np

import oracle as O


def rotate_keys(keys: np.ndarray, kv_heads: int, d: int, inv: np.ndarray, offset: int):
    """RoPE on keys [T, Hkv, d] at positions offset.. with the oracle
    (attention.rs:422-482 restated; the query slot is a throw-away copy)."""
    _, k = O.apply_rotary_with_offset(keys.copy(), keys, kv_heads, kv_heads, d, inv, offset)
    return k.reshape(keys.shape)


def to_dev(a: np.ndarray, device: int = 0):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(f"cuda:{device}")


def fill_history(caches, oracle_caches, lengths, layers, rng, inv, kv_heads, d):
    """Appends `lengths[i]` random tokens to every layer of cache i on both
    sides (GPU append with fused RoPE; oracle: rotate then append)."""
    for cache, oc, n in zip(caches, oracle_caches, lengths):
        if n == 0:
            continue
        for layer in range(layers):
            k = rng.standard_normal((n, kv_heads, d)).astype(np.float32)
            v = rng.standard_normal((n, kv_heads, d)).astype(np.float32)
            cache.append_layer(layer, to_dev(k), to_dev(v), n, rotate_keys=True)
            oc.append_layer(layer, rotate_keys(k, kv_heads, d, inv, 0), v, n)


def bits(a) -> np.ndarray:
    if hasattr(a, "detach"):
        a = a.detach().cpu().numpy()
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)

"""slm_batch_attention_exact against the oracle, bit for bit.

The kernel computes attention in the reference's operation order: each
score an in-order fma fold times (d as f32).sqrt().recip(), the softmax's
max, glibc's expf (restated), its sequential sum and division
(softmax.rs:26-44), each output an in-order fma fold over the positions
(attention.rs:195-399 for a prompt, 677-759 for a decoded token). The oracle
restates those functions in C with the host's glibc, so every output bit
must agree: prompt prefill from an empty cache, prefill after a cached
history, and decode steps (token counts 1 after the append), for every query
group size, over shuffled paged blocks.
"""

import numpy as np
import pytest

import oracle as O
from gpu_util import bits, fill_history, to_dev

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
slmkv = pytest.importorskip("slmkv")

D = 64


def _pool(hq, hkv, layers=1, seqs=8, ctx=512, blocks=256):
    pool = slmkv.KvPool(num_layers=layers, num_query_heads=hq, num_key_value_heads=hkv,
                        head_dimension=D, context_length=ctx, rope_theta=10000.0,
                        num_blocks=blocks, max_sequences=seqs, device=0)
    pool.shuffle(3)
    return pool


@pytest.mark.parametrize("hq,hkv", [(4, 2), (2, 2), (8, 2), (16, 2)])
def test_prefill_from_empty_is_bit_exact(hq, hkv):
    rng = np.random.default_rng(50 + hq)
    counts = [1, 5, 16, 17, 40, 130]
    pool = _pool(hq, hkv)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    caches = [pool.allocate_kv_cache(256) for _ in counts]
    T = sum(counts)
    q = rng.standard_normal((T, hq, D)).astype(np.float32)
    k = rng.standard_normal((T, hkv, D)).astype(np.float32)
    v = rng.standard_normal((T, hkv, D)).astype(np.float32)
    out = torch.empty((T, hq, D), dtype=torch.float32, device="cuda:0")
    with pool.begin(caches, counts) as b:
        b.append_layer(0, to_dev(k), to_dev(v), rotate_keys=True)
        b.attention_exact(0, to_dev(q), out, rotate_query=True)
    got = bits(out)
    row = 0
    for t in counts:
        rq, rk = O.apply_rotary_with_offset(q[row:row + t], k[row:row + t], hq, hkv, D, inv, 0)
        ref = O.prefill_attention(rq, rk, v[row:row + t], hq, hkv, D).reshape(t, hq, D)
        assert np.array_equal(got[row:row + t], bits(ref)), (t, row)
        row += t


def test_prefill_after_history_is_bit_exact():
    # the new tokens attend the cached history and each other (a prompt
    # extended after an attached prefix): equal to the full prompt's rows
    rng = np.random.default_rng(61)
    hq, hkv = 4, 2
    bases, counts = [3, 16, 40, 200], [7, 1, 33, 64]
    pool = _pool(hq, hkv)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    caches = [pool.allocate_kv_cache(512) for _ in bases]
    hist = []
    for c, n in zip(caches, bases):
        kk = rng.standard_normal((n, hkv, D)).astype(np.float32)
        vv = rng.standard_normal((n, hkv, D)).astype(np.float32)
        c.append_layer(0, to_dev(kk), to_dev(vv), n, rotate_keys=True)
        hist.append((kk, vv))
    T = sum(counts)
    q = rng.standard_normal((T, hq, D)).astype(np.float32)
    k = rng.standard_normal((T, hkv, D)).astype(np.float32)
    v = rng.standard_normal((T, hkv, D)).astype(np.float32)
    out = torch.empty((T, hq, D), dtype=torch.float32, device="cuda:0")
    with pool.begin(caches, counts) as b:
        b.append_layer(0, to_dev(k), to_dev(v), rotate_keys=True)
        b.attention_exact(0, to_dev(q), out, rotate_query=True)
    got = bits(out)
    row = 0
    for i, (base, t) in enumerate(zip(bases, counts)):
        qz = np.zeros((base, hq, D), np.float32)
        allq = np.concatenate([qz, q[row:row + t]])
        allk = np.concatenate([hist[i][0], k[row:row + t]])
        allv = np.concatenate([hist[i][1], v[row:row + t]])
        rq, rk = O.apply_rotary_with_offset(allq, allk, hq, hkv, D, inv, 0)
        ref = O.prefill_attention(rq, rk, allv, hq, hkv, D).reshape(base + t, hq, D)[base:]
        assert np.array_equal(got[row:row + t], bits(ref)), (base, t)
        row += t


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("hq,hkv", [(4, 2), (8, 2)])
def test_decode_steps_are_bit_exact(hq, hkv, fused):
    # append at the pre-append length, then attend the grown cache
    # (attention.rs:794-810); three steps over ragged shuffled caches, as
    # append + attention_exact and as the one-kernel decode_layer_exact
    rng = np.random.default_rng(70 + hq)
    lengths = [1, 15, 16, 17, 100, 300, 511 - 3]
    n = len(lengths)
    pool = _pool(hq, hkv, layers=2, seqs=n, blocks=512)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    caches = [pool.allocate_kv_cache(512) for _ in lengths]
    ocs = [O.DenseCache(2, 512, hkv, D) for _ in lengths]
    fill_history(caches, ocs, lengths, 2, rng, inv, hkv, D)
    for _ in range(3):
        with pool.begin(caches, 1) as b:
            for layer in range(2):
                q = rng.standard_normal((n, hq, D)).astype(np.float32)
                k = rng.standard_normal((n, hkv, D)).astype(np.float32)
                v = rng.standard_normal((n, hkv, D)).astype(np.float32)
                out = torch.empty((n, hq, D), dtype=torch.float32, device="cuda:0")
                if fused:
                    b.decode_layer_exact(layer, to_dev(q), to_dev(k), to_dev(v), out)
                else:
                    b.append_layer(layer, to_dev(k), to_dev(v), rotate_keys=True)
                    b.attention_exact(layer, to_dev(q), out, rotate_query=True)
                ref = O.forward_cached_attention_batch(ocs, layer, q, k, v, hq, inv, threads=8)
                assert np.array_equal(bits(out).reshape(n, -1), bits(ref).reshape(n, -1))
    assert [c.sequence_length() for c in caches] == [L + 3 for L in lengths]
    for c, oc in zip(caches, ocs):  # the appended rows, bit for bit
        for layer in range(2):
            assert np.array_equal(bits(c.layer_keys(layer)), bits(oc.layer_keys(layer)))
            assert np.array_equal(bits(c.layer_values(layer)), bits(oc.layer_values(layer)))


@pytest.mark.parametrize("n,max_len", [(64, 511), (100, 300)])
def test_fused_exact_decode_of_many_sequences_is_bit_exact(n, max_len):
    # more CTAs (sequences x 4 heads) than SMs: K passes through shared
    # memory in rounds of 128 positions, two buffers with an 8-deep V ring at
    # 256 CTAs (up to four rounds at these lengths), one buffer with a 4-deep
    # ring at 400
    rng = np.random.default_rng(77 + n)
    hq, hkv = 4, 2
    lengths = [int(x) for x in rng.integers(1, max_len, size=n)]
    n = len(lengths)
    pool = _pool(hq, hkv, layers=1, seqs=n, blocks=sum(L // 16 + 2 for L in lengths) + 8)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    caches = [pool.allocate_kv_cache(512) for _ in lengths]
    ocs = [O.DenseCache(1, 512, hkv, D) for _ in lengths]
    fill_history(caches, ocs, lengths, 1, rng, inv, hkv, D)
    q = rng.standard_normal((n, hq, D)).astype(np.float32)
    k = rng.standard_normal((n, hkv, D)).astype(np.float32)
    v = rng.standard_normal((n, hkv, D)).astype(np.float32)
    out = torch.empty((n, hq, D), dtype=torch.float32, device="cuda:0")
    with pool.begin(caches, 1) as b:
        b.decode_layer_exact(0, to_dev(q), to_dev(k), to_dev(v), out)
    ref = O.forward_cached_attention_batch(ocs, 0, q, k, v, hq, inv, threads=8)
    assert np.array_equal(bits(out).reshape(n, -1), bits(ref).reshape(n, -1))


def test_fused_exact_decode_rolls_back_non_finite_kv():
    rng = np.random.default_rng(75)
    pool = _pool(4, 2, layers=1, seqs=3)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    caches = [pool.allocate_kv_cache(64) for _ in range(3)]
    ocs = [O.DenseCache(1, 64, 2, D) for _ in range(3)]
    fill_history(caches, ocs, [15, 16, 3], 1, rng, inv, 2, D)
    q = rng.standard_normal((3, 4, D)).astype(np.float32)
    k = rng.standard_normal((3, 2, D)).astype(np.float32)
    v = rng.standard_normal((3, 2, D)).astype(np.float32)
    v[1, 1, 5] = np.inf
    out = torch.empty((3, 4, D), dtype=torch.float32, device="cuda:0")
    b = pool.begin(caches, 1)
    b.decode_layer_exact(0, to_dev(q), to_dev(k), to_dev(v), out)
    with pytest.raises(slmkv.InvalidInput) as e:
        b.end()
    assert "key/value" in str(e.value)
    assert b.statuses == [0, slmkv.ERR_NON_FINITE, 0]
    assert [c.sequence_length() for c in caches] == [16, 16, 4]


def test_exact_attention_flags_a_non_finite_query_and_needs_f32():
    rng = np.random.default_rng(80)
    pool = _pool(4, 2, seqs=2)
    caches = [pool.allocate_kv_cache(64) for _ in range(2)]
    k = rng.standard_normal((10, 2, D)).astype(np.float32)
    q = rng.standard_normal((10, 4, D)).astype(np.float32)
    q[7, 0, 0] = np.nan  # sequence 1
    out = torch.empty((10, 4, D), dtype=torch.float32, device="cuda:0")
    b = pool.begin(caches, [5, 5])
    b.append_layer(0, to_dev(k), to_dev(k), rotate_keys=True)
    b.attention_exact(0, to_dev(q), out, rotate_query=True)
    with pytest.raises(slmkv.InvalidInput) as e:
        b.end()
    assert "softmax" in str(e.value)
    assert b.statuses == [0, slmkv.ERR_NON_FINITE]
    assert [c.sequence_length() for c in caches] == [5, 0]
    bf = slmkv.KvPool(num_layers=1, num_query_heads=4, num_key_value_heads=2, head_dimension=D,
                      context_length=64, num_blocks=8, max_sequences=1, kv_dtype=slmkv.KV_BF16,
                      device=0)
    c = bf.allocate_kv_cache(16)
    b = bf.begin([c], [2])
    b.append_layer(0, to_dev(k[:2]), to_dev(k[:2]), rotate_keys=True)
    with pytest.raises(slmkv.InvalidInput):
        b.attention_exact(0, to_dev(q[:2]), out[:2])
    b.rollback()

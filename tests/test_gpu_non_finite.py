"""Non-finite attention scores on the GPU, as the reference rejects them.

softmax_in_place rejects a row holding a non-finite value and a sum that is
not finite and positive (softmax.rs:17-22,35-40). Through attend_cached_query
(attention.rs:731) a cached decode step then fails and truncates the layer
(attention.rs:814-815), and the model rolls the whole step back
(model.rs:390-396); a prompt prefill fails in causal_probabilities
(attention.rs:256-269) and the model clears the cache (model.rs:322-327).
Here: a query element that is NaN or infinite (host-made input, no device
fault) fails that sequence's step with SLM_ERR_NON_FINITE, leaves its length
as it was, and leaves its batch mates untouched.

Also: a failed append leaves zeros, not its non-finite values, in the pool
slots past the length, so a later prefill that stages those slots (the
tensor-core prefill loads whole 16-token blocks) still matches the oracle.
"""

import numpy as np
import pytest

import oracle as O
from gpu_util import fill_history, to_dev

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
slmkv = pytest.importorskip("slmkv")

D = 64


def _pool(kv_dtype=slmkv.KV_F32, layers=2, seqs=4, blocks=128):
    pool = slmkv.KvPool(num_layers=layers, num_query_heads=4, num_key_value_heads=2,
                        head_dimension=D, context_length=256, rope_theta=10000.0,
                        num_blocks=blocks, max_sequences=seqs, kv_dtype=kv_dtype, device=0)
    pool.shuffle(5)
    return pool


@pytest.mark.parametrize("kv_dtype", [slmkv.KV_F32, slmkv.KV_BF16])
@pytest.mark.parametrize("bad_value", [np.nan, np.inf, -np.inf])
def test_decode_with_a_non_finite_query_fails_that_sequence_only(kv_dtype, bad_value):
    rng = np.random.default_rng(1)
    q8 = kv_dtype == slmkv.KV_BF16
    pool = _pool(kv_dtype)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    lengths = [10, 40, 130]
    caches = [pool.allocate_kv_cache(256) for _ in lengths]
    ocs = [O.DenseCache(2, 256, 2, D, quantize_bf16=q8) for _ in lengths]
    fill_history(caches, ocs, lengths, 2, rng, inv, 2, D)
    batch = pool.begin(caches, 1)
    outs = []
    for layer in range(2):
        q = rng.standard_normal((3, 4, D)).astype(np.float32)
        k = rng.standard_normal((3, 2, D)).astype(np.float32)
        v = rng.standard_normal((3, 2, D)).astype(np.float32)
        ref = O.forward_cached_attention_batch([ocs[0], ocs[2]], layer, q[[0, 2]], k[[0, 2]],
                                               v[[0, 2]], 4, inv).reshape(2, 4, D)
        if layer == 1:
            q[1, 2, 33] = bad_value  # query head 2 of sequence 1 (KV head 1)
        out = torch.empty((3, 4, D), dtype=torch.float32, device="cuda:0")
        batch.decode_layer(layer, to_dev(q), to_dev(k), to_dev(v), out)
        outs.append((out, ref))
    with pytest.raises(slmkv.InvalidInput) as e:
        batch.end()
    assert e.value.code == slmkv.ERR_NON_FINITE
    assert "softmax" in str(e.value) and "finite" in str(e.value)
    assert batch.statuses == [0, slmkv.ERR_NON_FINITE, 0]
    assert [c.sequence_length() for c in caches] == [11, 40, 131]
    assert all(c.is_synchronized() for c in caches)
    tol = 2e-2 if q8 else 1e-4
    for out, ref in outs:  # the batch mates' attention is the oracle's
        got = out.cpu().numpy()[[0, 2]]
        assert np.abs(got - ref).max() <= tol
    # the failed sequence decodes normally afterwards
    with pool.begin(caches, 1) as b:
        for layer in range(2):
            out = torch.empty((3, 4, D), dtype=torch.float32, device="cuda:0")
            z = torch.zeros((3, 2, D), device="cuda:0")
            b.decode_layer(layer, torch.ones((3, 4, D), device="cuda:0"), z, z, out)
    assert [c.sequence_length() for c in caches] == [12, 41, 132]


def test_attend_cached_query_rejects_a_non_finite_query():
    rng = np.random.default_rng(2)
    pool = _pool()
    inv = O.rope_inverse_frequencies(D, 10000.0)
    cache = pool.allocate_kv_cache(256)
    oc = O.DenseCache(2, 256, 2, D)
    fill_history([cache], [oc], [77], 1, rng, inv, 2, D)
    q = rng.standard_normal((4, D)).astype(np.float32)
    q[3, 0] = np.nan
    with pytest.raises(slmkv.InvalidInput) as e:
        cache.attend_cached_query(0, to_dev(q))
    assert e.value.code == slmkv.ERR_NON_FINITE
    assert "invalid input for softmax: all input values must be finite" in str(e.value)
    assert cache.layer_sequence_length(0) == 77
    q[3, 0] = 0.25
    out = cache.attend_cached_query(0, to_dev(q))
    assert np.abs(out.cpu().numpy() - oc.attend_cached_query(0, q, 4)).max() <= 1e-4


@pytest.mark.parametrize("kv_dtype", [slmkv.KV_F32, slmkv.KV_BF16])
def test_prefill_with_a_non_finite_query_rolls_that_sequence_back(kv_dtype):
    # f32 pools prefill on CUDA cores, bf16 pools on the tensor cores
    rng = np.random.default_rng(3)
    pool = _pool(kv_dtype, layers=1)
    counts = [5, 140, 17]
    caches = [pool.allocate_kv_cache(256) for _ in counts]
    T = sum(counts)
    q = rng.standard_normal((T, 4, D)).astype(np.float32)
    k = rng.standard_normal((T, 2, D)).astype(np.float32)
    v = rng.standard_normal((T, 2, D)).astype(np.float32)
    q[5 + 131, 1, 9] = np.inf  # sequence 1, its token 131 (second K/V tile)
    out = torch.empty((T, 4, D), dtype=torch.float32, device="cuda:0")
    b = pool.begin(caches, counts)
    b.append_layer(0, to_dev(k), to_dev(v), rotate_keys=True)
    b.prefill_attention(0, to_dev(q), out, rotate_query=True)
    with pytest.raises(slmkv.InvalidInput) as e:
        b.end()
    assert e.value.code == slmkv.ERR_NON_FINITE and "softmax" in str(e.value)
    assert b.statuses == [0, slmkv.ERR_NON_FINITE, 0]
    assert [c.sequence_length() for c in caches] == [5, 0, 17]


def test_failed_append_leaves_no_non_finite_value_for_a_later_prefill():
    rng = np.random.default_rng(4)
    pool = _pool(slmkv.KV_BF16, layers=1, seqs=2)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    cache = pool.allocate_kv_cache(256)
    oc = O.DenseCache(1, 256, 2, D, quantize_bf16=True)
    fill_history([cache], [oc], [40], 1, rng, inv, 2, D)
    # a decode whose new V is NaN fails: slot 40 was written, then rolled back
    b = pool.begin([cache], 1)
    v = np.full((1, 2, D), np.nan, np.float32)
    out = torch.empty((1, 4, D), device="cuda:0")
    b.decode_layer(0, to_dev(rng.standard_normal((1, 4, D))), to_dev(np.ones((1, 2, D))),
                   to_dev(v), out)
    with pytest.raises(slmkv.InvalidInput):
        b.end()
    assert cache.sequence_length() == 40
    # back to 30 tokens, then a prefill of 5: its K/V tile stages block 2
    # (positions 32..47) whole, slot 40 included, with P = 0 there
    cache.truncate_all(30)
    oc.truncate_all(30)
    q = rng.standard_normal((5, 4, D)).astype(np.float32)
    k = rng.standard_normal((5, 2, D)).astype(np.float32)
    vv = rng.standard_normal((5, 2, D)).astype(np.float32)
    out = torch.empty((5, 4, D), dtype=torch.float32, device="cuda:0")
    with pool.begin([cache], [5]) as b:
        b.append_layer(0, to_dev(k), to_dev(vv), rotate_keys=True)
        b.prefill_attention(0, to_dev(q), out, rotate_query=True)
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    qz = np.zeros((30, 4, D), np.float32)
    qn, kn = O.apply_rotary_with_offset(q, k, 4, 2, D, inv, 30)
    kk = O.round_to_bfloat16_array(np.concatenate([oc.layer_keys(0), kn.reshape(5, 2, D)]))
    vh = O.round_to_bfloat16_array(np.concatenate([oc.layer_values(0), vv]))
    ref = O.prefill_attention(np.concatenate([qz, qn.reshape(5, 4, D)]), kk, vh, 4, 2,
                              D).reshape(35, 4, D)[30:]
    assert np.abs(got - ref).max() <= 2e-2

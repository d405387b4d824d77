"""GPU parity of the KV-cache hot path against the CPU oracle.

Bar: K/V append and block-table gathers bit-exact; decode / prefill attention
within 1e-4 max-abs for f32 KV and 2e-2 for bf16 KV (the oracle's bf16 cache
stores round_to_bfloat16 of the same values, linear.rs:14-23).
"""

import numpy as np
import pytest

import oracle as O
from gpu_util import bits, fill_history, rotate_keys, to_dev

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
slmkv = pytest.importorskip("slmkv")

D = 64
TOL = {slmkv.KV_F32: 1e-4, slmkv.KV_BF16: 2e-2}


def make_pool(kv_dtype=slmkv.KV_F32, layers=2, hq=4, hkv=2, ctx=512, blocks=1024, seqs=64,
              shuffle=7):
    pool = slmkv.KvPool(num_layers=layers, num_query_heads=hq, num_key_value_heads=hkv,
                        head_dimension=D, context_length=ctx, rope_theta=10000.0,
                        num_blocks=blocks, max_sequences=seqs, kv_dtype=kv_dtype, device=0)
    if shuffle is not None:
        pool.shuffle(shuffle)
    return pool


@pytest.mark.parametrize("kv_dtype", [slmkv.KV_F32, slmkv.KV_BF16])
def test_append_with_rope_is_bit_exact(kv_dtype):
    rng = np.random.default_rng(1)
    pool = make_pool(kv_dtype)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    cache = pool.allocate_kv_cache(300)
    oc = O.DenseCache(2, 300, 2, D, quantize_bf16=(kv_dtype == slmkv.KV_BF16))
    pos = 0
    for t in [37, 1, 1, 1, 20, 16, 64, 3]:  # ragged appends across block boundaries
        k = rng.standard_normal((t, 2, D)).astype(np.float32)
        v = rng.standard_normal((t, 2, D)).astype(np.float32)
        cache.append_layer(0, to_dev(k), to_dev(v), t, rotate_keys=True)
        oc.append_layer(0, rotate_keys(k, 2, D, inv, pos), v, t)
        pos += t
    torch.cuda.synchronize()
    assert cache.layer_sequence_length(0) == pos == oc.layer_sequence_length(0)
    assert cache.layer_sequence_length(1) == 0 and not cache.is_synchronized()
    assert np.array_equal(bits(cache.layer_keys(0)), bits(oc.layer_keys(0)))
    assert np.array_equal(bits(cache.layer_values(0)), bits(oc.layer_values(0)))
    # key_head / value_head views (kv_cache.rs:256-278)
    assert np.array_equal(bits(cache.key_head(0, 5, 1)), bits(oc.key_head(0, 5, 1)))
    assert np.array_equal(bits(cache.value_head(0, pos - 1, 0)), bits(oc.value_head(0, pos - 1, 0)))
    with pytest.raises(slmkv.InvalidInput):
        cache.key_head(0, pos, 0)


def test_append_without_rotation_stores_inputs_verbatim():
    rng = np.random.default_rng(2)
    pool = make_pool()
    cache = pool.allocate_kv_cache(64)
    k = rng.standard_normal((33, 2, D)).astype(np.float32)
    v = rng.standard_normal((33, 2, D)).astype(np.float32)
    cache.append_layer(1, to_dev(k), to_dev(v), 33, rotate_keys=False)
    assert np.array_equal(bits(cache.layer_keys(1)), bits(k))
    assert np.array_equal(bits(cache.layer_values(1)), bits(v))


def test_failed_append_does_not_mutate_the_cache():
    """kv_cache.rs:192-211 and its test at :473-483."""
    rng = np.random.default_rng(3)
    pool = make_pool()
    cache = pool.allocate_kv_cache(20)
    k = rng.standard_normal((16, 2, D)).astype(np.float32)
    v = rng.standard_normal((16, 2, D)).astype(np.float32)
    cache.append_layer(0, to_dev(k), to_dev(v), 16)
    free_before, _ = pool.stats()
    before_k, before_v = bits(cache.layer_keys(0)), bits(cache.layer_values(0))
    bad = rng.standard_normal((2, 2, D)).astype(np.float32)
    bad[1, 1, 7] = np.inf
    with pytest.raises(slmkv.InvalidInput) as e:
        cache.append_layer(0, to_dev(bad), to_dev(bad), 2)
    assert e.value.code == slmkv.ERR_NON_FINITE
    assert "must be finite" in str(e.value)
    assert cache.layer_sequence_length(0) == 16
    assert pool.stats()[0] == free_before
    assert np.array_equal(bits(cache.layer_keys(0)), before_k)
    assert np.array_equal(bits(cache.layer_values(0)), before_v)
    big = rng.standard_normal((5, 2, D)).astype(np.float32)
    with pytest.raises(slmkv.InvalidInput) as e:
        cache.append_layer(0, to_dev(big), to_dev(big), 5)
    assert e.value.code == slmkv.ERR_CAPACITY
    assert "exceeding capacity 20" in str(e.value)
    assert cache.layer_sequence_length(0) == 16


def _decode_case(kv_dtype, lengths, layers=2, hq=4, hkv=2, seed=5, ctx=512):
    rng = np.random.default_rng(seed)
    n = len(lengths)
    pool = make_pool(kv_dtype, layers=layers, hq=hq, hkv=hkv, ctx=ctx,
                     blocks=sum((L + 16) // 16 + 1 for L in lengths) + 8, seqs=n)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    q8 = kv_dtype == slmkv.KV_BF16
    caches = [pool.allocate_kv_cache(ctx) for _ in range(n)]
    ocs = [O.DenseCache(layers, ctx, hkv, D, quantize_bf16=q8) for _ in range(n)]
    fill_history(caches, ocs, lengths, layers, rng, inv, hkv, D)
    worst = 0.0
    with pool.begin(caches, 1) as batch:
        for layer in range(layers):
            q = rng.standard_normal((n, hq, D)).astype(np.float32)
            k = rng.standard_normal((n, hkv, D)).astype(np.float32)
            v = rng.standard_normal((n, hkv, D)).astype(np.float32)
            out = torch.empty((n, hq, D), dtype=torch.float32, device="cuda:0")
            batch.decode_layer(layer, to_dev(q), to_dev(k), to_dev(v), out)
            ref = O.forward_cached_attention_batch(ocs, layer, q, k, v, hq, inv, threads=8)
            got = out.cpu().numpy().reshape(n, hq * D)
            err = float(np.abs(got - ref.reshape(n, hq * D)).max())
            worst = max(worst, err)
    assert batch.statuses == [0] * n
    for c, oc, L in zip(caches, ocs, lengths):
        assert c.sequence_length() == L + 1 and c.is_synchronized()
        for layer in range(layers):
            assert np.array_equal(bits(c.layer_keys(layer)), bits(oc.layer_keys(layer)))
            assert np.array_equal(bits(c.layer_values(layer)), bits(oc.layer_values(layer)))
    return worst


@pytest.mark.parametrize("kv_dtype", [slmkv.KV_F32, slmkv.KV_BF16])
def test_fused_decode_matches_oracle_small(kv_dtype):
    lengths = [0, 1, 2, 15, 16, 17, 31, 63, 64, 65, 127, 128, 129, 200, 300, 511]
    err = _decode_case(kv_dtype, lengths)
    assert err <= TOL[kv_dtype], err


def test_fused_decode_many_short_sequences():
    """More sequences than decode warps have blocks: warps own zero or one
    block, every (sequence, head) is a single-block pair."""
    rng = np.random.default_rng(31)
    lengths = rng.choice([0, 1, 14, 15, 16], size=300).tolist()
    err = _decode_case(slmkv.KV_F32, lengths, layers=1, seed=33)
    assert err <= 1e-4, err


@pytest.mark.parametrize("hq,hkv", [(4, 4), (8, 2), (16, 2)])
def test_fused_decode_group_sizes(hq, hkv):
    err = _decode_case(slmkv.KV_F32, [3, 40, 257, 511], layers=1, hq=hq, hkv=hkv, seed=9)
    assert err <= 1e-4, err


@pytest.mark.parametrize("hq,hkv", [(4, 4), (4, 2), (8, 2), (16, 2)])
def test_fused_decode_group_sizes_bf16(hq, hkv):
    """bf16 KV runs its blocks on the tensor cores with Q and P split into
    bf16 (hi, lo) pairs: well inside the bf16 bar."""
    lengths = [1, 16, 17, 40, 257, 511]
    err = _decode_case(slmkv.KV_BF16, lengths, layers=2, hq=hq, hkv=hkv, seed=19)
    assert err <= 2e-2, err
    assert err <= 1e-3, err  # the split keeps ~16 mantissa bits of Q and P


def test_fused_decode_full_microbench_shape():
    """B=256 sequences, lengths U[1,511], Hq=4, Hkv=2, d=64, f32, shuffled
    16-token blocks — checked against the oracle for every sequence."""
    rng = np.random.default_rng(0)
    lengths = rng.integers(1, 512, size=256).tolist()
    lengths = [min(L, 511) for L in lengths]
    err = _decode_case(slmkv.KV_F32, lengths, layers=2, seed=17)
    assert err <= 1e-4, err


def test_long_context_bf16_split_k():
    """Long sequences exercise many split-K partials (the scaled-GQA shape:
    32 query / 8 KV heads, bf16 KV)."""
    err = _decode_case(slmkv.KV_BF16, [1024, 4097, 8191], layers=1, hq=32, hkv=8, seed=21,
                       ctx=8192)
    assert err <= 2e-2, err


def test_attend_cached_query_matches_oracle():
    """attention.rs:677-759 with an already-rotated query, no append."""
    rng = np.random.default_rng(4)
    pool = make_pool()
    inv = O.rope_inverse_frequencies(D, 10000.0)
    for L in [1, 16, 77, 512]:
        cache = pool.allocate_kv_cache(512)
        oc = O.DenseCache(2, 512, 2, D)
        fill_history([cache], [oc], [L], 1, rng, inv, 2, D)
        q = rng.standard_normal((4, D)).astype(np.float32)
        out = cache.attend_cached_query(0, to_dev(q))
        ref = oc.attend_cached_query(0, q, 4)
        assert np.abs(out.cpu().numpy() - ref).max() <= 1e-4
        assert cache.layer_sequence_length(0) == L
        cache.free()
    empty = pool.allocate_kv_cache(8)
    with pytest.raises(slmkv.InvalidInput):
        empty.attend_cached_query(0, to_dev(np.zeros((4, D), np.float32)))


@pytest.mark.parametrize("kv_dtype", [slmkv.KV_F32, slmkv.KV_BF16])
def test_prefill_attention_matches_oracle(kv_dtype):
    """Prompt prefill from an empty cache: attention.rs:859-868."""
    rng = np.random.default_rng(6)
    counts = [1, 5, 16, 17, 40, 100]
    n = len(counts)
    pool = make_pool(kv_dtype, layers=1, seqs=n)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    caches = [pool.allocate_kv_cache(256) for _ in range(n)]
    T = sum(counts)
    q = rng.standard_normal((T, 4, D)).astype(np.float32)
    k = rng.standard_normal((T, 2, D)).astype(np.float32)
    v = rng.standard_normal((T, 2, D)).astype(np.float32)
    out = torch.empty((T, 4, D), dtype=torch.float32, device="cuda:0")
    with pool.begin(caches, counts) as batch:
        batch.append_layer(0, to_dev(k), to_dev(v), rotate_keys=True)
        batch.prefill_attention(0, to_dev(q), out, rotate_query=True)
    got = out.cpu().numpy()
    row = 0
    for c, t in zip(caches, counts):
        rq, rk = O.apply_rotary_with_offset(q[row:row + t], k[row:row + t], 4, 2, D, inv, 0)
        vv = v[row:row + t]
        if kv_dtype == slmkv.KV_BF16:
            rk = O.round_to_bfloat16_array(rk)
            vv = O.round_to_bfloat16_array(vv)
        ref = O.prefill_attention(rq, rk, vv, 4, 2, D).reshape(t, 4, D)
        assert np.abs(got[row:row + t] - ref).max() <= TOL[kv_dtype]
        assert c.layer_sequence_length(0) == t
        assert np.array_equal(bits(c.layer_keys(0)),
                              bits(rk.reshape(t, 2, D) if kv_dtype == slmkv.KV_F32 else rk.reshape(t, 2, D)))
        row += t


def test_decode_step_rolls_back_non_finite_sequences():
    """model.rs:390-396: a failed step leaves that cache at its old length;
    the other sequences of the batch commit."""
    rng = np.random.default_rng(8)
    pool = make_pool(layers=2, seqs=4)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    caches = [pool.allocate_kv_cache(128) for _ in range(3)]
    ocs = [O.DenseCache(2, 128, 2, D) for _ in range(3)]
    fill_history(caches, ocs, [10, 20, 30], 2, rng, inv, 2, D)
    batch = pool.begin(caches, 1)
    for layer in range(2):
        q = rng.standard_normal((3, 4, D)).astype(np.float32)
        k = rng.standard_normal((3, 2, D)).astype(np.float32)
        v = rng.standard_normal((3, 2, D)).astype(np.float32)
        if layer == 1:
            v[1, 0, 3] = np.nan
        out = torch.empty((3, 4, D), dtype=torch.float32, device="cuda:0")
        batch.decode_layer(layer, to_dev(q), to_dev(k), to_dev(v), out)
    with pytest.raises(slmkv.InvalidInput):
        batch.end()
    assert batch.statuses == [0, slmkv.ERR_NON_FINITE, 0]
    assert [c.sequence_length() for c in caches] == [11, 20, 31]
    assert all(c.is_synchronized() for c in caches)


def test_batch_rejects_unsynchronized_and_full_caches():
    rng = np.random.default_rng(10)
    pool = make_pool(layers=2, seqs=4)
    a = pool.allocate_kv_cache(4)
    k = rng.standard_normal((4, 2, D)).astype(np.float32)
    a.append_layer(0, to_dev(k), to_dev(k), 4)
    with pytest.raises(slmkv.InvalidInput) as e:
        pool.begin([a], 1)
    assert "same length" in str(e.value)
    a.append_layer(1, to_dev(k), to_dev(k), 4)
    with pytest.raises(slmkv.InvalidInput) as e:
        pool.begin([a], 1)
    assert e.value.code == slmkv.ERR_CAPACITY
    assert a.sequence_length() == 4


def test_prefix_reuse_is_bit_exact_and_copy_on_write():
    rng = np.random.default_rng(12)
    pool = make_pool(layers=2, seqs=8, blocks=64, shuffle=3)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    prompt = rng.integers(0, 8192, size=40).tolist()
    a = pool.allocate_kv_cache(128)
    oa = O.DenseCache(2, 128, 2, D)
    fill_history([a], [oa], [40], 2, rng, inv, 2, D)
    assert a.publish_prefix(prompt) == 2  # two full blocks
    free0, idx0 = pool.stats()
    assert idx0 == 2
    b = pool.allocate_kv_cache(128)
    assert b.attach_prefix(prompt[:35] + [1, 2, 3]) == 32
    assert b.blocks()[:2] == a.blocks()[:2]
    assert pool.stats()[0] == free0  # no new blocks taken
    for layer in range(2):
        assert np.array_equal(bits(b.layer_keys(layer)), bits(oa.layer_keys(layer)[:32]))
        assert np.array_equal(bits(b.layer_values(layer)), bits(oa.layer_values(layer)[:32]))
    # b decodes past the prefix; a's cache is untouched
    ob = O.DenseCache(2, 128, 2, D)
    for layer in range(2):
        ob.append_layer(layer, oa.layer_keys(layer)[:32], oa.layer_values(layer)[:32], 32)
    with pool.begin([b], 1) as batch:
        for layer in range(2):
            q = rng.standard_normal((1, 4, D)).astype(np.float32)
            k = rng.standard_normal((1, 2, D)).astype(np.float32)
            v = rng.standard_normal((1, 2, D)).astype(np.float32)
            out = torch.empty((1, 4, D), dtype=torch.float32, device="cuda:0")
            batch.decode_layer(layer, to_dev(q), to_dev(k), to_dev(v), out)
            ref = O.forward_cached_attention_batch([ob], layer, q, k, v, 4, inv)
            assert np.abs(out.cpu().numpy().ravel() - ref).max() <= 1e-4
    assert b.sequence_length() == 33
    assert b.blocks()[:2] == a.blocks()[:2] and len(b.blocks()) == 3
    for layer in range(2):
        assert np.array_equal(bits(a.layer_keys(layer)), bits(oa.layer_keys(layer)))
    # Truncating b into the shared region, then writing, copies the block first.
    b.truncate_all(20)
    k = rng.standard_normal((1, 2, D)).astype(np.float32)
    for layer in range(2):
        b.append_layer(layer, to_dev(k), to_dev(k), 1)
    assert b.blocks()[0] == a.blocks()[0] and b.blocks()[1] != a.blocks()[1]
    for layer in range(2):
        assert np.array_equal(bits(a.layer_keys(layer)), bits(oa.layer_keys(layer)))
        assert np.array_equal(bits(b.layer_keys(layer)[:20]), bits(oa.layer_keys(layer)[:20]))

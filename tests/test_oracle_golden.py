"""Pin the CPU oracle to the reference before it is trusted as the checker.

Two sources: the known answers of small-lm-rs's own Rust unit tests
(tests/golden/known_answers.json, each case tagged with its file:line) and
vectors produced by the reference's NumPy decoder
(tests/golden/numpy_reference_vectors.json).
"""

import json
import math
from pathlib import Path

import numpy as np
import pytest

import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"
KA = json.loads((GOLDEN / "known_answers.json").read_text())
NV = json.loads((GOLDEN / "numpy_reference_vectors.json").read_text())


def _num(x):
    return float(x) if not isinstance(x, str) else float(x)


def test_rope_inverse_frequencies():
    c = KA["rope_inverse_frequencies"]
    inv = O.rope_inverse_frequencies(c["head_dim"], c["theta"])
    np.testing.assert_allclose(inv, c["expected"], atol=c["atol"], rtol=0)


def test_rope_position_zero_is_identity():
    c = KA["rope_position_zero_identity"]
    inv = O.rope_inverse_frequencies(c["head_dim"], c["theta"])
    out = O.rope_apply_head(c["head"], inv, c["position"])
    assert out.tolist() == c["expected"]


def test_rope_rotates_interleaved_pairs():
    c = KA["rope_interleaved_pairs"]
    inv = O.rope_inverse_frequencies(c["head_dim"], c["theta"])
    q = O.rope_apply_head(c["query"], inv, c["position"])
    k = O.rope_apply_head(c["key"], inv, c["position"])
    np.testing.assert_allclose(q, c["expected_query"], atol=c["atol"], rtol=0)
    np.testing.assert_allclose(k, c["expected_key"], atol=c["atol"], rtol=0)


def test_rope_multiple_heads_and_bad_shapes():
    c = KA["rope_multiple_heads_and_bad_shapes"]
    inv = O.rope_inverse_frequencies(c["head_dim"], c["theta"])
    O.rope_apply_heads(c["values"], c["num_heads_ok"], c["head_dim"], inv, c["position"])
    with pytest.raises(O.OracleError):
        O.rope_apply_heads(c["values"], c["num_heads_bad"], c["head_dim"], inv, c["position"])


def test_rope_rejects_bad_configuration():
    with pytest.raises(O.OracleError):
        O.rope_inverse_frequencies(3, 10000.0)
    with pytest.raises(O.OracleError):
        O.rope_inverse_frequencies(4, -1.0)


def test_softmax_known_answers():
    c = KA["softmax_large_logits"]
    out = O.softmax(c["values"])
    np.testing.assert_allclose(out, c["expected"], atol=c["atol"], rtol=0)
    assert abs(float(out.sum()) - 1.0) <= 1e-6
    c = KA["softmax_rows"]
    out = O.softmax_rows(c["values"], c["rows"], c["columns"])
    np.testing.assert_allclose(out, c["expected"], atol=c["atol"], rtol=0)
    with pytest.raises(O.OracleError):
        O.softmax([])
    with pytest.raises(O.OracleError):
        O.softmax([0.0, float("nan")])


def test_bf16_rounding_known_answers():
    for x, y in KA["bf16_rounding"]["cases"]:
        assert O.round_to_bfloat16(_num(x)) == _num(y)


def test_bf16_rounding_vector_matches_scalar():
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(4096).astype(np.float32),
                        np.array([0.0, -0.0, 1e-40, 3.4e38, -3.4e38, np.inf, -np.inf],
                                 np.float32)])
    vec = O.round_to_bfloat16_array(x)
    scal = np.array([O.round_to_bfloat16(float(v)) for v in x], np.float32)
    assert np.array_equal(vec.view(np.uint32), scal.view(np.uint32))


@pytest.mark.parametrize("name", ["linear_layout", "linear_bf16_single_row",
                                  "linear_bf16_multi_row"])
def test_linear_known_answers(name):
    c = KA[name]
    out = O.linear(c["input"], c["rows"], c["in"], c["weight"], c["out"])
    assert out.tolist() == c["expected"]


def test_linear_fp32_known_answer():
    c = KA["linear_fp32"]
    out = O.linear_fp32(c["input"], c["rows"], c["in"], c["weight"], c["out"])
    assert out.tolist() == c["expected"]
    bf = O.linear(c["input"], c["rows"], c["in"], c["weight"], c["out"])
    assert out.tolist() != bf.tolist()


def test_kv_cache_known_answers():
    c = KA["kv_cache_tiny"]
    L, H, d = c["num_layers"], c["kv_heads"], c["head_dim"]
    cache = O.DenseCache(L, 4, H, d)
    assert cache.sequence_length() == 0 and cache.is_empty() and cache.is_synchronized()
    assert cache.layer_keys(0).size == 0 and cache.layer_values(1).size == 0
    cache.append_layer(0, c["append_keys"], c["append_values"], 2)
    assert cache.layer_sequence_length(0) == 2 and cache.layer_sequence_length(1) == 0
    assert not cache.is_synchronized()
    assert cache.key_head(0, 1, 0).tolist() == c["key_head_0_1_0"]
    assert cache.value_head(0, 0, 0).tolist() == c["value_head_0_0_0"]

    small = O.DenseCache(L, 1, H, d)  # kv_cache.rs:473-483
    small.append_layer(0, [1.0, 2.0], [3.0, 4.0], 1)
    with pytest.raises(O.OracleError) as e:
        small.append_layer(0, [5.0, 6.0], [7.0, 8.0], 1)
    assert e.value.code == O.ERR_CAPACITY
    assert small.layer_sequence_length(0) == 1
    assert small.key_head(0, 0, 0).tolist() == [1.0, 2.0]

    cap = O.DenseCache(L, 4, H, d)  # kv_cache.rs:486-494
    assert cap.remaining_capacity() == 4
    cap.append_layer(0, [1.0, 2.0], [3.0, 4.0], 1)
    assert cap.remaining_capacity() == 3

    tr = O.DenseCache(L, 4, H, d)  # kv_cache.rs:497-510
    for layer in range(L):
        tr.append_layer(layer, [1.0, 2.0, 3.0, 4.0], [5.0, 6.0, 7.0, 8.0], 2)
    tr.truncate_all(1)
    assert tr.is_synchronized() and tr.sequence_length() == 1
    with pytest.raises(O.OracleError):
        tr.truncate_all(2)
    assert tr.sequence_length() == 1

    cl = O.DenseCache(L, 4, H, d)  # kv_cache.rs:513-526
    for layer in range(L):
        cl.append_layer(layer, [1.0, 2.0], [3.0, 4.0], 1)
    assert cl.sequence_length() == 1 and cl.is_synchronized()
    cl.clear()
    assert cl.is_empty() and cl.is_synchronized()


def test_kv_cache_rejects_non_finite_without_mutation():
    cache = O.DenseCache(1, 4, 1, 2)
    cache.append_layer(0, [1.0, 2.0], [3.0, 4.0], 1)
    with pytest.raises(O.OracleError) as e:
        cache.append_layer(0, [float("inf"), 2.0], [3.0, 4.0], 1)
    assert e.value.code == O.ERR_NON_FINITE
    assert cache.layer_sequence_length(0) == 1


def test_causal_scores_known_answer():
    c = KA["causal_scores"]
    s = O.causal_scores(c["query"], c["key"], c["q_heads"], c["kv_heads"], c["head_dim"])
    exp = np.array(c["expected"], np.float32)
    for i in c["masked_indices"]:
        assert s[i] == np.finfo(np.float32).min  # exactly f32::MIN
    keep = [i for i in range(len(exp)) if i not in c["masked_indices"]]
    np.testing.assert_allclose(s[keep], exp[keep], atol=c["atol"], rtol=0)


def test_causal_probabilities_known_answer():
    c = KA["causal_probabilities"]
    p = O.causal_probabilities(c["query"], c["key"], c["q_heads"], c["kv_heads"],
                               c["head_dim"])
    np.testing.assert_allclose(p, c["expected"], atol=c["atol"], rtol=0)
    assert p[1] == 0.0  # the masked entry is exactly zero


def test_gqa_value_aggregation_known_answer():
    c = KA["gqa_value_aggregation"]
    out = O.attend_values(c["probabilities"], c["value"], c["q_heads"], c["kv_heads"],
                          c["head_dim"])
    assert out.tolist() == c["expected"]


def test_rotary_offset_equals_prefill_position_bit_exact():
    c = KA["rotary_offset_equals_prefill_position"]
    inv = O.rope_inverse_frequencies(c["head_dim"], c["theta"])
    fq, fk = O.apply_rotary_with_offset(c["full_query"], c["full_key"], 1, 1,
                                        c["head_dim"], inv, 0)
    tq, tk = O.apply_rotary_with_offset(c["token_query"], c["token_key"], 1, 1,
                                        c["head_dim"], inv, c["offset"])
    assert tq.view(np.uint32).tolist() == fq[2:4].view(np.uint32).tolist()
    assert tk.view(np.uint32).tolist() == fk[2:4].view(np.uint32).tolist()


def test_rope_applies_to_queries_and_keys_only():
    c = KA["rope_queries_and_keys_only"]
    inv = O.rope_inverse_frequencies(c["head_dim"], c["theta"])
    q, k = O.apply_rotary_with_offset(c["query"], c["key"], c["q_heads"], c["kv_heads"],
                                      c["head_dim"], inv, 0)
    assert q[0:2].tolist() == c["expected_query_0_0"]
    np.testing.assert_allclose(q[4:6], c["expected_query_1_0"], atol=c["atol"], rtol=0)
    np.testing.assert_allclose(k[2:4], c["expected_key_1_0"], atol=c["atol"], rtol=0)


def test_single_token_attention_known_answer():
    c = KA["single_token_attention"]
    inv = O.rope_inverse_frequencies(c["head_dim"], c["theta"])
    cache = O.DenseCache(1, 8, c["kv_heads"], c["head_dim"])
    out, _, _ = cache.forward_cached_attention(0, c["query"], c["key"], c["value"],
                                               c["q_heads"], inv)
    assert out.tolist() == c["expected"]


def test_sequential_cached_attention_matches_fresh():
    """attention.rs:1262-1301 at the attention level: two cached decode steps
    equal the rows of a fresh causal prefill within 1e-6."""
    c = KA["sequential_cached_equals_fresh"]
    Hq, Hkv, d = c["q_heads"], c["kv_heads"], c["head_dim"]
    inv = O.rope_inverse_frequencies(d, c["theta"])
    hs = np.array(c["hidden_states"], np.float32).reshape(2, 4)
    q = hs.copy()
    k = hs[:, :2].copy()
    v = hs[:, :2].copy()
    rq, rk = O.apply_rotary_with_offset(q, k, Hq, Hkv, d, inv, 0)
    fresh = O.prefill_attention(rq, rk, v, Hq, Hkv, d)
    cache = O.DenseCache(1, 8, Hkv, d)
    o0, _, _ = cache.forward_cached_attention(0, q[0], k[0], v[0], Hq, inv)
    o1, _, _ = cache.forward_cached_attention(0, q[1], k[1], v[1], Hq, inv)
    np.testing.assert_allclose(np.concatenate([o0, o1]), fresh, atol=c["atol"], rtol=0)


def test_decode_equals_prefill_last_row_random():
    """The same property at the BASELINE head shape (Hq=4, Hkv=2, d=64)."""
    rng = np.random.default_rng(11)
    T, Hq, Hkv, d = 37, 4, 2, 64
    inv = O.rope_inverse_frequencies(d, 10000.0)
    q = rng.standard_normal((T, Hq, d)).astype(np.float32)
    k = rng.standard_normal((T, Hkv, d)).astype(np.float32)
    v = rng.standard_normal((T, Hkv, d)).astype(np.float32)
    rq, rk = O.apply_rotary_with_offset(q, k, Hq, Hkv, d, inv, 0)
    fresh = O.prefill_attention(rq, rk, v, Hq, Hkv, d).reshape(T, Hq * d)
    cache = O.DenseCache(1, T, Hkv, d)
    for t in range(T):
        out, qt, kt = cache.forward_cached_attention(0, q[t], k[t], v[t], Hq, inv)
        # RoPE at the cached offset is bit-identical to the prefill position
        assert np.array_equal(qt.ravel().view(np.uint32), rq[t].ravel().view(np.uint32))
        assert np.array_equal(kt.ravel().view(np.uint32), rk[t].ravel().view(np.uint32))
        np.testing.assert_allclose(out, fresh[t], atol=1e-5, rtol=0)


def test_oracle_rope_matches_numpy_reference():
    c = NV["rope"]
    pos = c["positions"]
    d, Hq, Hkv = c["head_dim"], c["q_heads"], c["kv_heads"]
    inv = O.rope_inverse_frequencies(d, c["theta"])
    q = np.array(c["query"], np.float32).reshape(len(pos), Hq * d)
    k = np.array(c["key"], np.float32).reshape(len(pos), Hkv * d)
    eq = np.array(c["rotated_query"], np.float32).reshape(len(pos), Hq * d)
    ek = np.array(c["rotated_key"], np.float32).reshape(len(pos), Hkv * d)
    for i, p in enumerate(pos):
        rq = O.rope_apply_heads(q[i], Hq, d, inv, p)
        rk = O.rope_apply_heads(k[i], Hkv, d, inv, p)
        # NumPy's float32 powf/sin/cos are not glibc's (inverse frequencies may
        # differ by 1 ulp), so the angle agrees to a few ulp of its magnitude:
        # the rotated values agree to |x| * (few ulp of pos) plus rounding.
        ulp_angle = np.spacing(np.float32(max(p, 1)))
        tol = 4.0 * float(ulp_angle) * 4.0 + 2e-6
        np.testing.assert_allclose(rq, eq[i], atol=tol, rtol=0)
        np.testing.assert_allclose(rk, ek[i], atol=tol, rtol=0)


def test_oracle_softmax_matches_numpy_reference():
    c = NV["softmax"]
    out = O.softmax_rows(c["values"], c["rows"], c["columns"])
    np.testing.assert_allclose(out, c["expected"], atol=1e-6, rtol=1e-5)


def test_oracle_prefill_attention_matches_numpy_reference():
    c = NV["causal_attention"]
    T, Hq, Hkv, d = c["tokens"], c["q_heads"], c["kv_heads"], c["head_dim"]
    inv = O.rope_inverse_frequencies(d, c["theta"])
    q = np.array(c["query"], np.float32).reshape(T, Hq, d)
    k = np.array(c["key"], np.float32).reshape(T, Hkv, d)
    v = np.array(c["value"], np.float32).reshape(T, Hkv, d)
    rq, rk = O.apply_rotary_with_offset(q, k, Hq, Hkv, d, inv, 0)
    out = O.prefill_attention(rq, rk, v, Hq, Hkv, d)
    np.testing.assert_allclose(out, c["expected"], atol=2e-5, rtol=0)


def test_oracle_decode_matches_numpy_reference_rows():
    """Cached decode over the same sequence reproduces every row of the
    NumPy reference's causal attention (the cached == fresh property)."""
    c = NV["causal_attention"]
    T, Hq, Hkv, d = c["tokens"], c["q_heads"], c["kv_heads"], c["head_dim"]
    inv = O.rope_inverse_frequencies(d, c["theta"])
    q = np.array(c["query"], np.float32).reshape(T, Hq * d)
    k = np.array(c["key"], np.float32).reshape(T, Hkv * d)
    v = np.array(c["value"], np.float32).reshape(T, Hkv * d)
    exp = np.array(c["expected"], np.float32).reshape(T, Hq * d)
    cache = O.DenseCache(1, T, Hkv, d)
    for t in range(T):
        out, _, _ = cache.forward_cached_attention(0, q[t], k[t], v[t], Hq, inv)
        np.testing.assert_allclose(out, exp[t], atol=2e-5, rtol=0)

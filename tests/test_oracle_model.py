"""The oracle's model-level functions against the reference's own unit tests
(rmsnorm.rs, situ_glu.rs, embedding.rs, greedy.rs, model.rs tests), on the
CPU: the RMSNorm and SiTU-GLU known answers, embedding order and vocabulary
check, the first-maximum argmax, and the model invariants the reference
asserts exactly: cached decode logits equal a fresh prefill's last-position
logits (model.rs:601-619) and cached and uncached greedy generation agree
(model.rs:622-632)."""

import numpy as np
import pytest

import oracle as O


def test_rmsnorm_known_answer():
    # rmsnorm.rs tests: normalizes_one_row_and_applies_weights (within 1e-6)
    out = O.rmsnorm_rows([1.0, -1.0, 1.0, -1.0], 1, 4, [1.0, 2.0, 3.0, 4.0], 1e-5)
    inv = np.float32(1.0) / np.sqrt(np.float32(1.0) + np.float32(1e-5))
    assert np.abs(out - inv * np.array([1, -2, 3, -4], np.float32)).max() <= 1e-6


def test_situ_branch_formulas():
    # situ_glu.rs tests: branch_formulas_match_the_reference_definition
    assert abs(O.situ_gate_activation(0.0, 4.0)) <= 1e-6
    assert abs(O.situ_up_activation(0.0, 25.0)) <= 1e-6
    g = 4.0 * np.tanh(np.float32(0.25)) / (1.0 + np.exp(np.float32(-1.0)))
    assert abs(O.situ_gate_activation(1.0, 4.0) - g) <= 1e-6
    assert abs(O.situ_up_activation(1.0, 25.0) - 25.0 * np.tanh(np.float32(0.04))) <= 1e-6


def test_situ_forward_with_identity_weights():
    # situ_glu.rs tests: complete_feed_forward_uses_exported_weight_layout
    eye = np.eye(2, dtype=np.float32)
    out = O.situ_glu([1.0, -1.0], 1, 2, 2, eye, eye, eye, 4.0, 25.0)
    for i, x in enumerate((1.0, -1.0)):
        p = O.situ_gate_activation(x, 4.0) * O.situ_up_activation(x, 25.0)
        assert abs(out[i] - O.round_to_bfloat16(p)) <= 1e-6


def test_embedding_order_and_vocabulary():
    # embedding.rs tests: gathers_rows_in_token_order, rejects_out_of_vocabulary_tokens
    table = np.array([1, 2, 3, 4, 5, 6], np.float32)
    assert O.embedding_lookup([2, 0], table, 3, 2).tolist() == [5.0, 6.0, 1.0, 2.0]
    with pytest.raises(O.OracleError):
        O.embedding_lookup([3], np.zeros(6, np.float32), 3, 2)


def test_argmax_first_maximum_and_non_finite():
    # greedy.rs tests
    assert O.argmax_finite([-1.0, 3.0, 2.0]) == 1
    assert O.argmax_finite([5.0, 1.0, 5.0]) == 0
    with pytest.raises(O.OracleError):
        O.argmax_finite([])
    with pytest.raises(O.OracleError):
        O.argmax_finite([0.0, float("nan")])


def tiny_model(seed=3, vocab=64, layers=2, hq=4, hkv=2, d=16, inter=40):
    hidden = hq * d
    cfg = dict(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter, num_layers=layers,
               num_query_heads=hq, num_key_value_heads=hkv, head_dimension=d,
               rms_norm_epsilon=1e-5, rope_theta=10000.0, situ_beta_gate=4.0, situ_beta_up=25.0)
    rng = np.random.default_rng(seed)
    kv = hkv * d
    shapes = [(vocab, hidden)]
    for _ in range(layers):
        shapes += [(hidden,), (hidden, hidden), (kv, hidden), (kv, hidden), (hidden, hidden),
                   (hidden,), (inter, hidden), (inter, hidden), (hidden, inter)]
    shapes.append((hidden,))
    tensors = [(1.0 + 0.1 * rng.standard_normal(s)).astype(np.float32) if len(s) == 1
               else (0.2 * rng.standard_normal(s)).astype(np.float32) for s in shapes]
    return O.Model(cfg, tensors), cfg


def test_cached_decode_logits_equal_fresh_prefill_logits():
    # model.rs:601-619 asserts exact equality
    model, cfg = tiny_model()
    cache = model.new_cache(16)
    model.prefill(cache, [1, 2])
    cached = model.decode(cache, 3)
    fresh = model.prefill(model.new_cache(16), [1, 2, 3])[-1]
    assert np.array_equal(cached, fresh)
    assert cache.sequence_length() == 3


def test_cached_and_uncached_greedy_generation_match():
    # model.rs:622-632
    model, cfg = tiny_model(seed=5)
    prompt, steps = [7, 1, 30, 2], 6
    seq = list(prompt)
    uncached = []
    for _ in range(steps):
        t = O.argmax_finite(model.prefill(model.new_cache(32), seq)[-1])
        uncached.append(t)
        seq.append(t)
    cache = model.new_cache(32)
    t = O.argmax_finite(model.prefill(cache, prompt)[-1])
    cached = [t]
    for _ in range(steps - 1):
        t = O.argmax_finite(model.decode(cache, t))
        cached.append(t)
    assert cached == uncached


def test_decode_needs_a_prefilled_cache_and_rolls_back_bad_tokens():
    # model.rs:686-700 (cached_decode_requires_prompt_state_and_capacity); an
    # out-of-vocabulary token fails before any layer advances
    model, cfg = tiny_model()
    with pytest.raises(O.OracleError):
        model.decode(model.new_cache(4), 1)
    cache = model.new_cache(3)
    model.prefill(cache, [1, 2, 3])
    with pytest.raises(O.OracleError):
        model.decode(cache, 1)  # no capacity left
    cache = model.new_cache(8)
    model.prefill(cache, [1, 2])
    with pytest.raises(O.OracleError):
        model.decode(cache, cfg["vocab_size"])
    assert cache.sequence_length() == 2 and cache.is_synchronized()

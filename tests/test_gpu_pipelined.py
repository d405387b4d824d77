"""Pipelined decode steps (slm_batch_submit / slm_batch_wait) against the CPU
oracle: a step may begin while the previous one still runs on the GPU, and a
sequence that fails in one step fails, and is rolled back, in every later step
that was planned on top of it (model.rs:390-396 applied across the pipeline).
"""

import numpy as np
import pytest

import oracle as O
from gpu_util import bits, fill_history, to_dev

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
slmkv = pytest.importorskip("slmkv")

D = 64
TOL = 1e-4  # f32 KV


def _pool(layers, hq, hkv, n, lengths, extra_steps):
    pool = slmkv.KvPool(num_layers=layers, num_query_heads=hq, num_key_value_heads=hkv,
                        head_dimension=D, context_length=512, rope_theta=10000.0,
                        num_blocks=sum((L + extra_steps + 15) // 16 + 1 for L in lengths) + 8,
                        max_sequences=n, device=0)
    pool.shuffle(11)
    return pool


def _step_inputs(rng, n, layers, hq, hkv):
    return [(rng.standard_normal((n, hq, D)).astype(np.float32),
             rng.standard_normal((n, hkv, D)).astype(np.float32),
             rng.standard_normal((n, hkv, D)).astype(np.float32)) for _ in range(layers)]


def _launch(batch, inputs, n, hq):
    outs = []
    for layer, (q, k, v) in enumerate(inputs):
        out = torch.empty((n, hq, D), dtype=torch.float32, device="cuda:0")
        batch.decode_layer(layer, to_dev(q), to_dev(k), to_dev(v), out)
        outs.append(out)
    return outs


def test_pipelined_steps_match_the_oracle():
    rng = np.random.default_rng(21)
    layers, hq, hkv = 2, 4, 2
    lengths = [1, 15, 16, 31, 47, 200, 333, 480]
    n, steps = len(lengths), 5
    pool = _pool(layers, hq, hkv, n, lengths, steps)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    caches = [pool.allocate_kv_cache(512) for _ in range(n)]
    ocs = [O.DenseCache(layers, 512, hkv, D) for _ in range(n)]
    fill_history(caches, ocs, lengths, layers, rng, inv, hkv, D)
    pending = []  # (batch, outputs, oracle outputs)
    worst = 0.0
    for _ in range(steps):
        inputs = _step_inputs(rng, n, layers, hq, hkv)
        batch = pool.begin(caches, 1)
        outs = _launch(batch, inputs, n, hq)
        batch.submit()
        refs = [O.forward_cached_attention_batch(ocs, layer, q, k, v, hq, inv, threads=8)
                for layer, (q, k, v) in enumerate(inputs)]
        pending.append((batch, outs, refs))
        if len(pending) == 2:  # keep one step in flight behind the open one
            b, o, r = pending.pop(0)
            assert b.wait() == [0] * n
            for got, ref in zip(o, r):
                worst = max(worst, float(np.abs(got.cpu().numpy().reshape(n, -1)
                                                - ref.reshape(n, -1)).max()))
    for b, o, r in pending:
        assert b.wait() == [0] * n
        for got, ref in zip(o, r):
            worst = max(worst, float(np.abs(got.cpu().numpy().reshape(n, -1)
                                            - ref.reshape(n, -1)).max()))
    assert worst <= TOL, worst
    for c, oc, L in zip(caches, ocs, lengths):
        assert c.sequence_length() == L + steps and c.is_synchronized()
        for layer in range(layers):
            assert np.array_equal(bits(c.layer_keys(layer)), bits(oc.layer_keys(layer)))
            assert np.array_equal(bits(c.layer_values(layer)), bits(oc.layer_values(layer)))


def test_failure_rolls_back_the_later_steps_that_hold_the_sequence():
    rng = np.random.default_rng(22)
    layers, hq, hkv = 2, 4, 2
    lengths = [10, 20, 30]
    n = len(lengths)
    pool = _pool(layers, hq, hkv, n, lengths, 4)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    caches = [pool.allocate_kv_cache(128) for _ in range(n)]
    ocs = [O.DenseCache(layers, 128, hkv, D) for _ in range(n)]
    fill_history(caches, ocs, lengths, layers, rng, inv, hkv, D)

    # step 1: sequence 1 appends a NaN value in layer 1; submitted, not waited
    in1 = _step_inputs(rng, n, layers, hq, hkv)
    in1[1][2][1, 0, 3] = np.nan
    b1 = pool.begin(caches, 1)
    _launch(b1, in1, n, hq)
    b1.submit()
    # step 2 is planned on step 1's lengths, before step 1 is known to fail
    in2 = _step_inputs(rng, n, layers, hq, hkv)
    b2 = pool.begin(caches, 1)
    _launch(b2, in2, n, hq)
    b2.submit()
    # waiting for the later step resolves the earlier one first
    with pytest.raises(slmkv.InvalidInput) as e:
        b2.wait()
    assert e.value.code == slmkv.ERR_NON_FINITE
    assert b2.statuses == [0, slmkv.ERR_NON_FINITE, 0]
    with pytest.raises(slmkv.InvalidInput):
        b1.wait()
    assert b1.statuses == [0, slmkv.ERR_NON_FINITE, 0]
    assert [c.sequence_length() for c in caches] == [12, 20, 32]
    assert all(c.is_synchronized() for c in caches)

    # the oracle commits steps 1 and 2 for sequences 0 and 2 only
    for inputs in (in1, in2):
        for layer, (q, k, v) in enumerate(inputs):
            for i in (0, 2):
                O.forward_cached_attention_batch([ocs[i]], layer, q[i:i + 1], k[i:i + 1],
                                                 v[i:i + 1], hq, inv, threads=1)
    # a third step over all three matches the oracle from the rolled-back state
    in3 = _step_inputs(rng, n, layers, hq, hkv)
    with pool.begin(caches, 1) as b3:
        outs = _launch(b3, in3, n, hq)
    worst = 0.0
    for layer, (q, k, v) in enumerate(in3):
        ref = O.forward_cached_attention_batch(ocs, layer, q, k, v, hq, inv, threads=4)
        worst = max(worst, float(np.abs(outs[layer].cpu().numpy().reshape(n, -1)
                                        - ref.reshape(n, -1)).max()))
    assert worst <= TOL, worst
    for c, oc in zip(caches, ocs):
        assert c.sequence_length() == oc.sequence_length()
        for layer in range(layers):
            assert np.array_equal(bits(c.layer_keys(layer)), bits(oc.layer_keys(layer)))


def test_in_flight_limit_and_sync_end_alongside():
    rng = np.random.default_rng(23)
    layers, hq, hkv = 1, 4, 2
    lengths = [5, 40]
    n = len(lengths)
    in_flight = 8  # the library's limit on submitted, unresolved batches
    pool = _pool(layers, hq, hkv, n, lengths, in_flight + 2)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    caches = [pool.allocate_kv_cache(128) for _ in range(n)]
    ocs = [O.DenseCache(layers, 128, hkv, D) for _ in range(n)]
    fill_history(caches, ocs, lengths, layers, rng, inv, hkv, D)
    subs = []
    for _ in range(in_flight):
        b = pool.begin(caches, 1)
        _launch(b, _step_inputs(rng, n, layers, hq, hkv), n, hq)
        subs.append(b.submit())
    b_extra = pool.begin(caches, 1)
    _launch(b_extra, _step_inputs(rng, n, layers, hq, hkv), n, hq)
    with pytest.raises(slmkv.InvalidInput) as e:
        b_extra.submit()
    assert f"at most {in_flight}" in str(e.value)
    # the refused step stays open; a synchronous end still has a readback slot
    assert b_extra.end() == [0, 0]
    assert [b.wait() for b in subs] == [[0, 0]] * in_flight
    assert [c.sequence_length() for c in caches] == [L + in_flight + 1 for L in lengths]

"""Continuous-batching scheduler logic on a host-only pool (no GPU): admission
order and cap, prompt chunking within the token budget, the first output token
at the end of the prompt, finishing after max_new_tokens, preemption with
recomputation when the pool runs out, capacity checks and failed statuses.
A committed step stands for the KV batches the caller would have run."""

import random

import pytest

import slmkv


def _pool(num_blocks=256, seqs=16, ctx=512):
    return slmkv.KvPool(num_layers=2, num_query_heads=4, num_key_value_heads=2,
                        context_length=ctx, num_blocks=num_blocks, max_sequences=seqs, device=None)


def _run(sched, steps=10_000, fail=None):
    """Plan / commit until idle; returns finished {id: (status, generated)}
    and the per-step plans."""
    done, plans = {}, []
    for _ in range(steps):
        nd, np_ = sched.plan()
        if nd == 0 and np_ == 0:
            break
        d, p = sched.decode_seqs(), sched.prefill_seqs()
        plans.append((d, p))
        ds = [0] * nd
        ps = [0] * np_
        if fail is not None:
            fail(d, p, ds, ps)
        for rid, st, gen in sched.commit(ds, ps):
            done[rid] = (st, gen)
    return done, plans


def test_admission_chunking_first_token_and_finish():
    pool = _pool()
    s = slmkv.Scheduler(pool, max_running=3, max_prefill_tokens=64)
    for rid, (prompt, new) in enumerate([(40, 3), (10, 1), (100, 2), (5, 4), (30, 2)]):
        s.submit(rid, prompt, new)
    s.plan()
    # the first three are admitted; prompts fill the 64-token budget in order
    assert s.decode_seqs() == []
    assert [c for _, c in s.prefill_seqs()] == [40, 10, 14]
    fin = s.commit(None, [0, 0, 0])
    # request 1 wanted one token: the end of its prompt gives it
    assert fin == [(1, 0, 1)]
    assert s.counts()["running"] == 2
    s.plan()
    # request 0 decodes; request 2 continues its prompt; request 3 is admitted
    assert len(s.decode_seqs()) == 1
    # (its prompt has no room left in this step's budget)
    assert [c for _, c in s.prefill_seqs()] == [64]
    s.commit([0], [0] * len(s.prefill_seqs()))
    done, _ = _run(s)
    done.update({1: (0, 1)})
    assert {k: v[1] for k, v in done.items()} == {0: 3, 1: 1, 2: 2, 3: 4, 4: 2}
    assert all(st == 0 for st, _ in done.values())
    c = s.counts()
    assert c["waiting"] == 0 and c["running"] == 0 and c["generated_tokens"] == 12
    assert pool.stats()[0] == 256  # every sequence was freed (no block was ever taken)


def test_budget_spreads_long_prompts_over_steps():
    pool = _pool()
    s = slmkv.Scheduler(pool, max_running=4, max_prefill_tokens=32)
    s.submit(7, 100, 1)
    counts = []
    while True:
        nd, np_ = s.plan()
        if nd == 0 and np_ == 0:
            break
        counts += [c for _, c in s.prefill_seqs()]
        s.commit([0] * nd, [0] * np_)
    assert counts == [32, 32, 32, 4]


def test_preemption_recomputes_and_everything_finishes():
    rng = random.Random(5)
    # 20 blocks = 320 tokens of cache for requests that need up to 100 each
    pool = _pool(num_blocks=20, seqs=8, ctx=128)
    s = slmkv.Scheduler(pool, max_running=8, max_prefill_tokens=128)
    want = {}
    for rid in range(30):
        prompt, new = rng.randint(8, 60), rng.randint(8, 40)
        want[rid] = new
        s.submit(rid, prompt, new)
    done, plans = _run(s)
    assert {k: v[1] for k, v in done.items()} == want
    assert s.counts()["preemptions"] > 0
    assert s.counts()["generated_tokens"] == sum(want.values())
    # no step ever planned more cache than the pool holds: the scheduler's
    # own accounting, replayed
    assert all(len(d) + len(p) <= 8 for d, p in plans)


def test_capacity_checks_and_duplicate_ids():
    pool = _pool(num_blocks=8, ctx=128)
    s = slmkv.Scheduler(pool, max_running=2, max_prefill_tokens=64)
    with pytest.raises(slmkv.InvalidInput) as e:
        s.submit(1, 100, 40)  # 140 > context 128 (kv_cache.rs:203-211)
    assert e.value.code == slmkv.ERR_CAPACITY
    with pytest.raises(slmkv.EngineError):
        s.submit(2, 0, 4)
    s.submit(3, 10, 4)
    with pytest.raises(slmkv.EngineError):
        s.submit(3, 10, 4)


def test_failed_sequence_finishes_with_its_status():
    pool = _pool()
    s = slmkv.Scheduler(pool, max_running=4, max_prefill_tokens=64)
    s.submit(1, 8, 5)
    s.submit(2, 8, 5)

    def fail(d, p, ds, ps):
        if d:
            ds[0] = slmkv.ERR_NON_FINITE  # the first decode of the batch fails

    done, _ = _run(s, fail=fail)
    assert done[1][0] == slmkv.ERR_NON_FINITE
    assert done[2] == (0, 5) or done[2][0] == slmkv.ERR_NON_FINITE
    assert s.counts()["running"] == 0


def test_plan_requests_report_ids_and_positions():
    pool = _pool()
    s = slmkv.Scheduler(pool, max_running=3, max_prefill_tokens=16)
    s.submit(10, 20, 3)
    s.submit(11, 5, 2)
    s.plan()
    assert s.plan_requests() == ([], [(10, 0)])  # 16 of request 10's 20 prompt tokens
    s.commit(None, [0])
    s.plan()
    # request 10 continues at position 16; request 11 starts at 0
    assert s.plan_requests() == ([], [(10, 16), (11, 0)])
    s.commit(None, [0, 0])
    s.plan()
    # both prompts are cached: each decode step feeds the token at its length
    assert s.plan_requests() == ([(10, 20), (11, 5)], [])
    dreq, dpos, preq, ppos = s.plan_request_arrays()  # the same as numpy views
    assert dreq.tolist() == [10, 11] and dpos.tolist() == [20, 5]
    assert preq.tolist() == [] and ppos.tolist() == []


def test_a_request_preempted_inside_its_prompt_prefills_the_whole_prompt_again():
    # A small prompt budget spreads prompts over several steps and a small
    # pool preempts requests inside their prompts. Replaying the plans'
    # positions: no request decodes before its whole prompt is cached (a
    # decode entry feeds position >= prompt length), a prefill entry always
    # starts where the request's cache ends, and the first token comes only
    # from the prompt's last position.
    rng = random.Random(11)
    pool = _pool(num_blocks=12, seqs=8, ctx=128)
    s = slmkv.Scheduler(pool, max_running=6, max_prefill_tokens=24)
    prompts, outs = {}, {}
    for rid in range(12):
        prompts[rid], outs[rid] = rng.randint(20, 60), rng.randint(4, 20)
        s.submit(rid, prompts[rid], outs[rid])
    cached = {rid: 0 for rid in prompts}
    generated = {rid: 0 for rid in prompts}
    mid_prompt_preemptions = 0
    for _ in range(5000):
        nd, np_ = s.plan()
        if nd == 0 and np_ == 0:
            break
        dreq, dpos, preq, ppos = s.plan_request_arrays()
        counts = [c for _, c in s.prefill_seqs()]
        for r, p in zip(dreq, dpos):
            r, p = int(r), int(p)
            assert p >= prompts[r], (r, p, prompts[r])
        for r, p, c in zip(preq, ppos, counts):
            r, p = int(r), int(p)
            if p == 0 and cached[r] > 0:  # recomputation after a preemption
                if cached[r] < prompts[r]:
                    mid_prompt_preemptions += 1
                cached[r] = 0
            assert p == cached[r], (r, p, cached[r])
            cached[r] += c
            if cached[r] == prompts[r] and generated[r] == 0:
                generated[r] = 1
        for r, p in zip(dreq, dpos):
            cached[int(r)] += 1
            generated[int(r)] += 1
        s.commit([0] * nd, [0] * np_)
    assert s.counts()["waiting"] == 0 and s.counts()["running"] == 0
    assert s.counts()["generated_tokens"] == sum(outs.values())
    assert mid_prompt_preemptions > 0

"""The continuous-batching serve path on the GPU against the oracle.

The scheduler (slmkv_sched.cpp) replaces the reference server's
one-request-at-a-time worker (rust/server/src/worker.rs:87-98): every step
it plans a decode batch and a batch of prompt chunks (a prompt may take
several steps), the caller runs slm_model_decode / slm_model_prefill on them
and commits the statuses; when the pool cannot hold a step the newest
requests are preempted and later recompute what they had cached.

Here ten requests of random prompts run through it on the 8M model's shape
(two layers, a 1024-token vocabulary, f32 pool) with a pool small enough to
force preemptions and a prompt budget small enough to chunk prompts, so
steps mix decode rows and prefill chunks. Each request's greedy tokens must
be the ones the oracle's model (model.rs:297-397 restated) chooses for that
request alone, from its prompt (GenerationService's order: the first token
from the prompt's last position, then one per decode step), and the logits
that chose every token must be within 1e-4 of the oracle's.
"""

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
slmkv = pytest.importorskip("slmkv")

VOCAB, HQ, HKV, D, INTER, LAYERS, CTX = 1024, 4, 2, 64, 704, 2, 128
HIDDEN = HQ * D
BAR = 1e-4


def random_model(seed):
    rng = np.random.default_rng(seed)
    kv, scale = HKV * D, 0.8 / np.sqrt(HIDDEN)
    shapes = [(VOCAB, HIDDEN)]
    for _ in range(LAYERS):
        shapes += [(HIDDEN,), (HIDDEN, HIDDEN), (kv, HIDDEN), (kv, HIDDEN), (HIDDEN, HIDDEN),
                   (HIDDEN,), (INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER)]
    shapes.append((HIDDEN,))
    return [(1.0 + 0.05 * rng.standard_normal(s)).astype(np.float32) if len(s) == 1
            else (scale * rng.standard_normal(s)).astype(np.float32) for s in shapes]


def test_scheduled_steps_with_preemption_match_the_oracle():
    rng = np.random.default_rng(90)
    tensors = random_model(91)
    n_req = 10
    prompts = [rng.integers(0, VOCAB, int(rng.integers(5, 61))).astype(np.int32)
               for _ in range(n_req)]
    outputs = [int(rng.integers(4, 21)) for _ in range(n_req)]
    pool = slmkv.KvPool(num_layers=LAYERS, num_query_heads=HQ, num_key_value_heads=HKV,
                        head_dimension=D, context_length=CTX, num_blocks=14, max_sequences=8,
                        device=0)
    pool.shuffle(92)
    model = slmkv.Model(pool, vocab_size=VOCAB, intermediate_size=INTER, tensors=tensors)
    sched = slmkv.Scheduler(pool, max_running=6, max_prefill_tokens=40)
    for i in range(n_req):
        sched.submit(i, len(prompts[i]), outputs[i])
    hist = [np.concatenate([p, np.zeros(o, np.int32)]) for p, o in zip(prompts, outputs)]
    # the logits behind each request's k-th output token
    chose = [dict() for _ in range(n_req)]
    first_done = set()
    stream = torch.cuda.current_stream()
    ones = slmkv._i32_array([1] * 8)
    finished, steps, mixed = 0, 0, 0
    while finished < n_req:
        nd, npf = sched.plan()
        dreq, dpos, preq, ppos = (a.copy() for a in sched.plan_request_arrays())
        counts = np.ctypeslib.as_array(sched._pcnt)[:npf].copy()
        mixed += int(nd > 0 and npf > 0)
        dst = pst = None
        if nd:
            ids = torch.tensor([hist[r][p] for r, p in zip(dreq, dpos)], dtype=torch.int32,
                               device="cuda:0")
            logits = torch.empty((nd, VOCAB), dtype=torch.float32, device="cuda:0")
            nxt = torch.empty(nd, dtype=torch.int32, device="cuda:0")
            b = slmkv.Batch.for_sequences(pool, nd, sched._dseq, ones, stream)
            model.decode(b, ids, logits, nxt)
            dst = b.end(raise_on_error=False)
            lg, nx = logits.cpu().numpy(), nxt.cpu().numpy()
            for i, (r, p) in enumerate(zip(dreq, dpos)):
                if dst[i] == 0:
                    hist[r][p + 1] = nx[i]
                    chose[r][p + 1 - len(prompts[r])] = lg[i]
        if npf:
            ids = torch.tensor(np.concatenate([hist[r][p:p + c] for r, p, c in
                                               zip(preq, ppos, counts)]), dtype=torch.int32,
                               device="cuda:0")
            logits = torch.empty((npf, VOCAB), dtype=torch.float32, device="cuda:0")
            nxt = torch.empty(npf, dtype=torch.int32, device="cuda:0")
            b = slmkv.Batch.for_sequences(pool, npf, sched._pseq, sched._pcnt, stream)
            model.prefill(b, ids, logits, nxt)
            pst = b.end(raise_on_error=False)
            lg, nx = logits.cpu().numpy(), nxt.cpu().numpy()
            for i, (r, p, c) in enumerate(zip(preq, ppos, counts)):
                if pst[i] == 0 and p + c == len(prompts[r]) and r not in first_done:
                    hist[r][p + c] = nx[i]  # the first token, from the prompt's end
                    chose[r][0] = lg[i]
                    first_done.add(int(r))
        fin = sched.commit(dst, pst)
        assert all(st == 0 for _, st, _ in fin), fin
        finished += len(fin)
        steps += 1
        assert steps < 2000
    c = sched.counts()
    assert c["preemptions"] > 0 and mixed > 0, (c, mixed)
    assert c["generated_tokens"] == sum(outputs)

    cfg = dict(vocab_size=VOCAB, hidden_size=HIDDEN, intermediate_size=INTER, num_layers=LAYERS,
               num_query_heads=HQ, num_key_value_heads=HKV, head_dimension=D,
               rms_norm_epsilon=1e-5, rope_theta=10000.0, situ_beta_gate=4.0, situ_beta_up=25.0)
    omodel = O.Model(cfg, tensors)
    threads = O.max_threads()
    worst = 0.0
    for r in range(n_req):
        P, gen = len(prompts[r]), hist[r][len(prompts[r]):]
        assert sorted(chose[r]) == list(range(outputs[r])), (r, sorted(chose[r]))
        cache = omodel.new_cache(CTX)
        ref = omodel.prefill(cache, [int(t) for t in prompts[r]], threads)[-1]
        for k in range(outputs[r]):
            assert O.argmax_finite(ref) == int(gen[k]), (r, k)
            worst = max(worst, float(np.abs(chose[r][k] - ref).max()))
            if k + 1 < outputs[r]:
                ref = omodel.decode(cache, int(gen[k]), threads)
    assert worst <= BAR, worst
    print(f"serve: {n_req} requests, {steps} steps ({mixed} mixed), "
          f"{c['preemptions']} preemptions, logits max abs {worst:.2e}")
    sched.close()
    model.close()
    pool.close()

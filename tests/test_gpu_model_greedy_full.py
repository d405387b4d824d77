"""The 8M model's cached greedy generation at its full length, against the
oracle, step by step.

The shape is the reference's 8M model (artifacts/small-lm-8m/config.json):
8 layers, hidden 256, 4 query / 2 KV heads of 64, SiTU-GLU FFN 704, vocab
8192, context 512, tied embeddings; random fp32 weights (seed 0: matrices and
embedding N(0, 0.02^2), norms 1), an f32 KV pool. Batch 1: a 64-token prompt
of random ids, then 448 greedy decode steps, which fill the 512-token
context. The reference's property is that cached greedy generation equals
uncached generation (model.rs:622-632, greedy.rs:103-141); the oracle's
model is pinned to it in the CPU tests. Here every one of the 449 chosen
tokens must be the oracle's, and every step's logits within 1e-4 max abs of
the oracle's (fp32 bar).
"""

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
slmkv = pytest.importorskip("slmkv")

VOCAB, HIDDEN, INTER, LAYERS, HQ, HKV, D, CTX = 8192, 256, 704, 8, 4, 2, 64, 512
PROMPT, STEPS = 64, 448
BAR = 1e-4


def model_tensors(seed=0):
    rng = np.random.default_rng(seed)
    out = []
    for _, shape in slmkv.model_tensor_shapes(vocab_size=VOCAB, hidden_size=HIDDEN,
                                              intermediate_size=INTER, num_layers=LAYERS,
                                              kv_width=HKV * D):
        out.append(np.ones(shape, np.float32) if len(shape) == 1
                   else (0.02 * rng.standard_normal(shape)).astype(np.float32))
    return out


def test_8m_model_greedy_448_steps_equals_the_oracle():
    tensors = model_tensors(0)
    prompt = [int(x) for x in np.random.default_rng(0).integers(0, VOCAB, size=PROMPT)]
    cfg = dict(vocab_size=VOCAB, hidden_size=HIDDEN, intermediate_size=INTER, num_layers=LAYERS,
               num_query_heads=HQ, num_key_value_heads=HKV, head_dimension=D,
               rms_norm_epsilon=1e-5, rope_theta=10000.0, situ_beta_gate=4.0, situ_beta_up=25.0)
    omodel = O.Model(cfg, tensors)
    ocache = omodel.new_cache(CTX)
    threads = O.max_threads()

    pool = slmkv.KvPool(num_layers=LAYERS, num_query_heads=HQ, num_key_value_heads=HKV,
                        head_dimension=D, context_length=CTX, num_blocks=CTX // 16 + 4,
                        max_sequences=1, device=0)
    pool.shuffle(1)
    model = slmkv.Model(pool, vocab_size=VOCAB, intermediate_size=INTER, tensors=tensors)
    cache = pool.allocate_kv_cache(CTX)
    logits = torch.empty((1, VOCAB), dtype=torch.float32, device="cuda:0")
    tok = [torch.zeros(1, dtype=torch.int32, device="cuda:0") for _ in range(2)]
    with pool.begin([cache], [PROMPT]) as b:
        model.prefill(b, torch.tensor(prompt, dtype=torch.int32, device="cuda:0"), logits, tok[0])
    ref = omodel.prefill(ocache, prompt, threads)[-1]
    worst, steps_checked = 0.0, 0
    gpu_tokens, cpu_tokens = [], []
    for i in range(STEPS + 1):
        got = logits.cpu().numpy()[0]
        g_tok, c_tok = int(tok[i % 2].cpu()[0]), O.argmax_finite(ref)
        gpu_tokens.append(g_tok)
        cpu_tokens.append(c_tok)
        err = float(np.abs(got - ref).max())
        worst = max(worst, err)
        assert g_tok == c_tok, (i, g_tok, c_tok)
        assert err <= BAR, (i, err)
        steps_checked += 1
        if i == STEPS:
            break
        with pool.begin([cache], 1) as b:
            model.decode(b, tok[i % 2], logits, tok[(i + 1) % 2])
        ref = omodel.decode(ocache, c_tok, threads)
    assert cache.sequence_length() == CTX == ocache.sequence_length()
    assert gpu_tokens == cpu_tokens and steps_checked == STEPS + 1
    print(f"8M model, {STEPS} greedy steps: tokens equal, logits max abs {worst:.2e}")
    model.close()
    pool.close()

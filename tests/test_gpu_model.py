"""Full-model steps (slm_model_prefill / slm_model_decode) against the
oracle's model (model.rs:297-397): a seeded random model in the reference
layout, prompts of several lengths prefilled in one batch, then greedy decode
steps for all of them in one batch per step.

Bars: every greedy token must be the oracle's, and the logits must meet
  - max abs <= 1e-4 with an f32 pool on the exact-order projections (the
    default up to 1024 rows: each output is the reference's own fma fold over
    bf16-rounded operands, linear.rs:98-103);
  - max abs <= 2e-2 with a bf16 pool (the oracle's bf16 cache stores the same
    values rounded; the reference's prefill attends its unrounded K/V);
and, on top, the reference's own GPU-versus-CPU logit thresholds
(parity/runner.rs:33-43: max abs 0.1, mean abs 0.01, RMS 0.02, cosine >=
0.9999, top-1 agreement 1.0). The tensor-core projection path (another
accumulation order: a 1-ulp fp32 difference can flip a bf16 operand rounding,
which moves a logit by ~1e-3) is an option outside the fp32 parity claim and
is held to the reference's thresholds only.
Also: a token outside the vocabulary fails the step and rolls it back."""

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
slmkv = pytest.importorskip("slmkv")


def random_model(seed, vocab, hidden, hkv, inter, layers, d=64, scale=0.05):
    rng = np.random.default_rng(seed)
    kv = hkv * d
    shapes = [(vocab, hidden)]
    for _ in range(layers):
        shapes += [(hidden,), (hidden, hidden), (kv, hidden), (kv, hidden), (hidden, hidden),
                   (hidden,), (inter, hidden), (inter, hidden), (hidden, inter)]
    shapes.append((hidden,))
    # norms near 1, matrices N(0, scale^2) so the logits spread out
    return [(1.0 + 0.05 * rng.standard_normal(s)).astype(np.float32) if len(s) == 1
            else (scale * rng.standard_normal(s)).astype(np.float32) for s in shapes]


def _run(kv_dtype, prompts, steps=4, seed=7, ctx=128, exact_rows=None,
         dims=(1024, 4, 2, 64, 704, 2)):
    vocab, hq, hkv, d, inter, layers = dims
    hidden = hq * d
    threads = O.max_threads()
    # matrices scaled with the width so activations stay as at hidden 256
    tensors = random_model(seed, vocab, hidden, hkv, inter, layers, scale=0.8 / np.sqrt(hidden))
    ocfg = dict(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter, num_layers=layers,
                num_query_heads=hq, num_key_value_heads=hkv, head_dimension=d,
                rms_norm_epsilon=1e-5, rope_theta=10000.0, situ_beta_gate=4.0, situ_beta_up=25.0)
    omodel = O.Model(ocfg, tensors)
    pool = slmkv.KvPool(num_layers=layers, num_query_heads=hq, num_key_value_heads=hkv,
                        head_dimension=d, context_length=ctx, rope_theta=10000.0,
                        num_blocks=len(prompts) * (ctx // 16) + 4, max_sequences=len(prompts),
                        kv_dtype=kv_dtype, device=0)
    pool.shuffle(seed)
    model = slmkv.Model(pool, vocab_size=vocab, intermediate_size=inter, tensors=tensors)
    if exact_rows is not None:
        model.set_exact_rows(exact_rows)
    caches = [pool.allocate_kv_cache(ctx) for _ in prompts]
    ocaches = [omodel.new_cache(ctx, quantize_bf16=(kv_dtype == slmkv.KV_BF16)) for _ in prompts]
    n = len(prompts)
    ids = torch.tensor(np.concatenate(prompts), dtype=torch.int32, device="cuda:0")
    logits = torch.empty((n, vocab), dtype=torch.float32, device="cuda:0")
    nxt = torch.empty(n, dtype=torch.int32, device="cuda:0")
    with pool.begin(caches, [len(p) for p in prompts]) as b:
        model.prefill(b, ids, logits, nxt)
    got_all, ref_all = [], []
    ref = np.stack([omodel.prefill(oc, p, threads)[-1] for oc, p in zip(ocaches, prompts)])
    got_all.append(logits.cpu().numpy())
    ref_all.append(ref)
    tokens = nxt.cpu().numpy()
    assert tokens.tolist() == [int(np.argmax(r)) for r in ref]
    for _ in range(steps):
        cur = torch.tensor(tokens, dtype=torch.int32, device="cuda:0")
        with pool.begin(caches, 1) as b:
            model.decode(b, cur, logits, nxt)
        ref = np.stack([omodel.decode(oc, int(t), threads) for oc, t in zip(ocaches, tokens)])
        got_all.append(logits.cpu().numpy())
        ref_all.append(ref)
        tokens = nxt.cpu().numpy()
        assert tokens.tolist() == [int(np.argmax(r)) for r in ref]
    assert [c.sequence_length() for c in caches] == [len(p) + steps for p in prompts]
    model.close()
    return parity_metrics(np.concatenate(got_all), np.concatenate(ref_all))


def parity_metrics(got, ref):
    """parity/metrics.rs: scalar errors, flattened cosine, per-row top-1."""
    d = (got.astype(np.float64) - ref.astype(np.float64))
    g, r = got.astype(np.float64).ravel(), ref.astype(np.float64).ravel()
    return dict(max_abs=float(np.abs(d).max()), mean_abs=float(np.abs(d).mean()),
                rms=float(np.sqrt((d * d).mean())),
                cosine=float(g @ r / (np.linalg.norm(g) * np.linalg.norm(r))),
                top1=float(np.mean(np.argmax(got, 1) == np.argmax(ref, 1))))


def check_thresholds(m):
    # parity/runner.rs:33-43 defaults
    assert m["max_abs"] <= 0.1 and m["mean_abs"] <= 0.01 and m["rms"] <= 0.02, m
    assert m["cosine"] >= 0.9999 and m["top1"] == 1.0, m


F32_BAR, BF16_BAR = 1e-4, 2e-2  # logits max abs: fp32 KV, bf16 KV


def check_f32(m):
    check_thresholds(m)
    assert m["max_abs"] <= F32_BAR, m


def check_bf16(m):
    check_thresholds(m)
    assert m["max_abs"] <= BF16_BAR, m


PROMPTS = [np.array(p, np.uint32) for p in ([5, 900, 17, 3, 3], list(range(100, 117)),
                                             [int(x) for x in np.arange(33) * 31 % 1024])]


def test_model_prefill_and_decode_match_the_oracle_f32():
    m = _run(slmkv.KV_F32, PROMPTS)
    check_f32(m)
    print("f32 KV logits vs oracle:", m)


def test_model_prefill_and_decode_match_the_oracle_bf16():
    m = _run(slmkv.KV_BF16, PROMPTS)
    check_bf16(m)
    print("bf16 KV logits vs oracle:", m)


def test_batched_prefill_of_1024_rows_stays_exact():
    # 4 x 256 prompt rows = 1024: the largest step the exact-order kernels take
    rng = np.random.default_rng(12)
    prompts = [rng.integers(0, 1024, 256).astype(np.uint32) for _ in range(4)]
    m = _run(slmkv.KV_F32, prompts, steps=2, ctx=512)
    check_f32(m)
    print("1024-row prefill, f32 KV logits vs oracle:", m)


def test_long_prefill_on_the_tensor_core_path():
    # 3 x 400 prompt rows > 1024: the prefill's projections run as tensor-core
    # GEMMs (another accumulation order, outside the fp32 bar), the decode
    # steps as the exact-order kernels
    rng = np.random.default_rng(11)
    prompts = [rng.integers(0, 1024, 400).astype(np.uint32) for _ in range(3)]
    m = _run(slmkv.KV_F32, prompts, steps=2, ctx=512)
    check_thresholds(m)
    print("long prefill, f32 KV logits vs oracle:", m)


def test_every_step_on_the_tensor_core_path():
    # exact-order rows 0: prefill and decode projections all as GEMMs (an
    # option outside the fp32 bar)
    m = _run(slmkv.KV_F32, PROMPTS, exact_rows=0)
    check_thresholds(m)
    print("GEMM projections, f32 KV logits vs oracle:", m)


@pytest.mark.parametrize("exact_rows", [None, 0])
def test_scaled_gqa_shape_bf16(exact_rows):
    # the scaled GQA model's widths (hidden 2048 = 32 x 64, 8 KV heads, FFN
    # 5632, bf16 KV) on two layers and a small vocabulary: the exact-order
    # kernels at their widest staging (5632 down-projection inputs) and the
    # tensor-core GEMMs
    prompts = [np.array(p, np.uint32) for p in ([7, 1000, 3], list(range(200, 213)), [5] * 6)]
    m = _run(slmkv.KV_BF16, prompts, steps=3, exact_rows=exact_rows,
             dims=(1024, 32, 8, 64, 5632, 2))
    if exact_rows is None:
        check_bf16(m)
    else:
        check_thresholds(m)
    print(f"scaled GQA shape, exact rows {exact_rows}, bf16 KV logits vs oracle:", m)


def test_exact_rows_range_is_checked():
    pool = slmkv.KvPool(num_layers=1, num_query_heads=4, num_key_value_heads=2, head_dimension=64,
                        context_length=64, num_blocks=8, max_sequences=1, device=0)
    model = slmkv.Model(pool, vocab_size=64, intermediate_size=64,
                        tensors=random_model(1, 64, 256, 2, 64, 1))
    for bad in (-1, 1025):
        with pytest.raises(slmkv.InvalidInput):
            model.set_exact_rows(bad)
    model.set_exact_rows(0)
    model.set_exact_rows(1024)
    model.close()
    pool.close()


def test_out_of_vocabulary_token_fails_and_rolls_back():
    vocab, hq, hkv, d, inter, layers = 256, 4, 2, 64, 64, 1
    tensors = random_model(3, vocab, hq * d, hkv, inter, layers)
    pool = slmkv.KvPool(num_layers=layers, num_query_heads=hq, num_key_value_heads=hkv,
                        head_dimension=d, context_length=64, num_blocks=16, max_sequences=2,
                        device=0)
    model = slmkv.Model(pool, vocab_size=vocab, intermediate_size=inter, tensors=tensors)
    caches = [pool.allocate_kv_cache(64) for _ in range(2)]
    with pool.begin(caches, [3, 4]) as b:
        model.prefill(b, torch.tensor([1, 2, 3, 4, 5, 6, 7], dtype=torch.int32, device="cuda:0"))
    b = pool.begin(caches, 1)
    model.decode(b, torch.tensor([9, vocab], dtype=torch.int32, device="cuda:0"))
    with pytest.raises(slmkv.InvalidInput) as e:
        b.end()
    assert "vocabulary" in str(e.value)
    assert [c.sequence_length() for c in caches] == [3, 4]
    # the context is still usable
    nxt = torch.empty(2, dtype=torch.int32, device="cuda:0")
    with pool.begin(caches, 1) as b:
        model.decode(b, torch.tensor([9, 10], dtype=torch.int32, device="cuda:0"), None, nxt)
    assert [c.sequence_length() for c in caches] == [4, 5]
    assert all(0 <= t < vocab for t in nxt.cpu().tolist())
    model.close()


def test_model_loaded_from_safetensors_equals_the_array_model(tmp_path):
    # the same weights through slm_model_load_safetensors (weights.rs:117-190)
    # give bit-identical logits: names, shapes and little-endian values land
    # where slm_model_create puts them
    from test_weights_safetensors import write_safetensors

    vocab, hq, hkv, d, inter, layers = 512, 4, 2, 64, 128, 2
    tensors = random_model(5, vocab, hq * d, hkv, inter, layers)
    names = [n for n, _ in slmkv.model_tensor_shapes(vocab_size=vocab, hidden_size=hq * d,
                                                      intermediate_size=inter, num_layers=layers,
                                                      kv_width=hkv * d)]
    path = tmp_path / "w.safetensors"
    write_safetensors(path, dict(zip(names, tensors)), order=names[::-1])
    outs = []
    for build in ("arrays", "file"):
        pool = slmkv.KvPool(num_layers=layers, num_query_heads=hq, num_key_value_heads=hkv,
                            head_dimension=d, context_length=64, num_blocks=16, max_sequences=1,
                            device=0)
        if build == "arrays":
            model = slmkv.Model(pool, vocab_size=vocab, intermediate_size=inter, tensors=tensors)
        else:
            model = slmkv.Model.from_safetensors(pool, path, vocab_size=vocab,
                                                 intermediate_size=inter,
                                                 expected_parameter_count=sum(t.size for t in tensors))
        cache = pool.allocate_kv_cache(64)
        logits = torch.empty((1, vocab), dtype=torch.float32, device="cuda:0")
        with pool.begin([cache], [5]) as b:
            model.prefill(b, torch.tensor([3, 1, 4, 1, 5], dtype=torch.int32, device="cuda:0"), logits)
        first = logits.cpu().numpy().copy()
        with pool.begin([cache], 1) as b:
            model.decode(b, torch.tensor([9], dtype=torch.int32, device="cuda:0"), logits)
        outs.append((first, logits.cpu().numpy().copy()))
        model.close()
        pool.close()
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])

"""slm_decode_attention_noalloc: the decode attention entry point for callers
that cannot allocate device memory. An engine that owns all device memory as
one arena of its own, or a plugin inside a host that forbids new device
allocations after start-up, cannot let the library call cudaMalloc; this
entry point keeps its working memory in a fixed array the library holds.

Its output must equal the CPU oracle's attend_cached_query
(attention.rs:677-759 restated) within the decode tolerance, and the existing
entry point's (slm_attend_cached_query) on the same KV contents, on two calls
in a row (the calls share the library's fixed scratch array). This file is
collected last so that a run stopping at the first failure has run every
other test.
"""

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
slmkv = pytest.importorskip("slmkv")

D = 64
TOL = 1e-4  # f32 KV, as for every decode-attention parity test


def _case(seed, hq=4, hkv=2, lengths=(1, 15, 16, 17, 130, 300, 511)):
    rng = np.random.default_rng(seed)
    n = len(lengths)
    dev = "cuda:0"
    pool = slmkv.KvPool(num_layers=1, num_query_heads=hq, num_key_value_heads=hkv,
                        head_dimension=D, context_length=512, num_blocks=256, max_sequences=n,
                        device=0)
    pool.shuffle(seed)
    caches = [pool.allocate_kv_cache(512) for _ in range(n)]
    ocaches = [O.DenseCache(1, 512, hkv, D) for _ in range(n)]
    keys = [rng.standard_normal((L, hkv, D)).astype(np.float32) for L in lengths]
    vals = [rng.standard_normal((L, hkv, D)).astype(np.float32) for L in lengths]
    for c, oc, k, v in zip(caches, ocaches, keys, vals):
        c.append_layer(0, torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev), len(k),
                       rotate_keys=False)
        oc.append_layer(0, k, v, len(k))

    # The caller's own paged cache holding the same rows, with its own blocks.
    max_blocks = 32
    num_blocks = sum((L + 15) // 16 for L in lengths) + 5
    ids = rng.permutation(num_blocks).astype(np.int32)
    table = np.zeros((n, max_blocks), np.int32)
    kp = np.zeros((num_blocks, hkv, 16, D), np.float32)
    vp = np.zeros_like(kp)
    cur = 0
    for i, L in enumerate(lengths):
        for j in range((L + 15) // 16):
            table[i, j] = ids[cur]
            cur += 1
        for t in range(L):
            kp[table[i, t // 16], :, t % 16] = keys[i][t]
            vp[table[i, t // 16], :, t % 16] = vals[i][t]
    return pool, caches, ocaches, torch.from_numpy(kp).to(dev), torch.from_numpy(vp).to(dev), \
        table, np.array(lengths, np.int32), rng


def _existing(caches, query):
    return torch.stack([c.attend_cached_query(0, query[i]).view(-1, D)
                        for i, c in enumerate(caches)])


def _oracle(ocaches, query, hq):
    q = query.cpu().numpy()
    return np.stack([oc.attend_cached_query(0, q[i], hq).reshape(-1, D)
                     for i, oc in enumerate(ocaches)])


@pytest.mark.parametrize("hq,hkv", [(2, 2), (4, 2), (8, 2), (16, 2)])
def test_noalloc_matches_the_oracle_and_the_existing_entry_point_on_two_calls(hq, hkv):
    pool, caches, ocaches, kp, vp, table, lens, rng = _case(41, hq=hq, hkv=hkv)
    for call in range(2):
        q = torch.from_numpy(rng.standard_normal((len(lens), hq, D)).astype(np.float32)).cuda()
        got = slmkv.decode_attention_noalloc(kp, vp, table, lens, q)
        want = _existing(caches, q)
        torch.cuda.synchronize()
        err_existing = float((got - want).abs().max())
        err_oracle = float(np.abs(got.cpu().numpy() - _oracle(ocaches, q, hq)).max())
        assert err_existing <= TOL and err_oracle <= TOL, (call, err_existing, err_oracle)
    pool.close()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    pool, caches, ocaches, kp, vp, table, lens, rng = _case(43)
    q = torch.zeros((len(lens), 4, D), device="cuda:0")
    with pytest.raises(slmkv.InvalidInput) as e:  # 2100 sequences x 2 heads > 4096 pairs
        slmkv.decode_attention_noalloc(kp, vp, np.zeros((2100, 32), np.int32),
                                       np.ones(2100, np.int32),
                                       torch.zeros((2100, 4, D), device="cuda:0"))
    assert "fixed scratch" in str(e.value)
    # 512 sequences x 2 heads = 1024 pairs, but 512 x 130 blocks x 2 heads =
    # 133 120 blocks to read > 131 072
    with pytest.raises(slmkv.InvalidInput) as e:
        slmkv.decode_attention_noalloc(kp, vp, np.zeros((512, 130), np.int32),
                                       np.full(512, 130 * 16, np.int32),
                                       torch.zeros((512, 4, D), device="cuda:0"))
    assert "blocks to read" in str(e.value)
    bad = table.copy()
    bad[0, 0] = kp.shape[0]  # outside the caller's pool
    with pytest.raises(slmkv.InvalidInput):
        slmkv.decode_attention_noalloc(kp, vp, bad, lens, q)
    with pytest.raises(slmkv.InvalidInput):  # lengths shorter than the query's rows
        slmkv.decode_attention_noalloc(kp, vp, table, lens[:-1], q)
    # the shared scratch still serves a valid call afterwards
    q = torch.from_numpy(rng.standard_normal((len(lens), 4, D)).astype(np.float32)).cuda()
    got = slmkv.decode_attention_noalloc(kp, vp, table, lens, q)
    assert float((got - _existing(caches, q)).abs().max()) <= TOL
    pool.close()


def test_noalloc_rejects_a_non_finite_query():
    # softmax.rs:17-22: a non-finite score fails attend_cached_query
    pool, caches, ocaches, kp, vp, table, lens, rng = _case(44)
    q = torch.from_numpy(rng.standard_normal((len(lens), 4, D)).astype(np.float32)).cuda()
    q[2, 1, 7] = float("nan")
    with pytest.raises(slmkv.InvalidInput) as e:
        slmkv.decode_attention_noalloc(kp, vp, table, lens, q)
    assert "finite" in str(e.value)
    q[2, 1, 7] = 0.5
    got = slmkv.decode_attention_noalloc(kp, vp, table, lens, q)
    assert float(np.abs(got.cpu().numpy() - _oracle(ocaches, q, 4)).max()) <= TOL
    pool.close()

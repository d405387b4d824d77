"""slm_decode_attention_noalloc: the decode attention entry point for callers
that cannot allocate device memory (graph capture, arena-managed engines,
hosts that forbid allocations after start-up).

It must give the same result as the existing entry point,
slm_attend_cached_query, on the same KV contents, on two calls in a row
(the calls share the library's fixed scratch array). This file is collected
last so that a run stopping at the first failure has run every other test.
"""

import numpy as np
import pytest

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
    keys = [rng.standard_normal((L, hkv, D)).astype(np.float32) for L in lengths]
    vals = [rng.standard_normal((L, hkv, D)).astype(np.float32) for L in lengths]
    for c, k, v in zip(caches, keys, vals):
        c.append_layer(0, torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev), len(k),
                       rotate_keys=False)

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
    return pool, caches, torch.from_numpy(kp).to(dev), torch.from_numpy(vp).to(dev), table, \
        np.array(lengths, np.int32), rng


def _existing(caches, query):
    return torch.stack([c.attend_cached_query(0, query[i]).view(-1, D)
                        for i, c in enumerate(caches)])


@pytest.mark.parametrize("hq,hkv", [(4, 2), (8, 2)])
def test_noalloc_matches_the_existing_entry_point_on_two_calls(hq, hkv):
    pool, caches, kp, vp, table, lens, rng = _case(41, hq=hq, hkv=hkv)
    for call in range(2):
        q = torch.from_numpy(rng.standard_normal((len(lens), hq, D)).astype(np.float32)).cuda()
        got = slmkv.decode_attention_noalloc(kp, vp, table, lens, q)
        want = _existing(caches, q)
        torch.cuda.synchronize()
        err = float((got - want).abs().max())
        assert err <= TOL, (call, err)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    pool, caches, kp, vp, table, lens, rng = _case(43)
    q = torch.zeros((len(lens), 4, D), device="cuda:0")
    with pytest.raises(slmkv.InvalidInput) as e:  # 2100 sequences x 2 heads > 4096 pairs
        slmkv.decode_attention_noalloc(kp, vp, np.zeros((2100, 32), np.int32),
                                       np.ones(2100, np.int32),
                                       torch.zeros((2100, 4, D), device="cuda:0"))
    assert "fixed scratch" in str(e.value)
    bad = table.copy()
    bad[0, 0] = kp.shape[0]  # outside the caller's pool
    with pytest.raises(slmkv.InvalidInput):
        slmkv.decode_attention_noalloc(kp, vp, bad, lens, q)
    # the shared scratch still serves a valid call afterwards
    q = torch.from_numpy(rng.standard_normal((len(lens), 4, D)).astype(np.float32)).cuda()
    got = slmkv.decode_attention_noalloc(kp, vp, table, lens, q)
    assert float((got - _existing(caches, q)).abs().max()) <= TOL

"""Prefill attention over a bf16 cache on the tensor cores (tcgen05) against
the oracle: prompts spanning several 128-token K/V tiles, a cached history
before the new tokens (attention of the new tokens over the whole cache, as
forward_prefill_with_cache does, attention.rs:835-870), every supported query
group size. The oracle stores the same values rounded to bf16 and computes
the causal prefill in f32 (attention.rs:195-399)."""

import numpy as np
import pytest

import oracle as O
from gpu_util import to_dev

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
slmkv = pytest.importorskip("slmkv")

D = 64
TOL = 2e-2  # bf16 KV


def _case(hq, hkv, counts, bases, seed):
    rng = np.random.default_rng(seed)
    n = len(counts)
    ctx = 512
    pool = slmkv.KvPool(num_layers=1, num_query_heads=hq, num_key_value_heads=hkv,
                        head_dimension=D, context_length=ctx, rope_theta=10000.0,
                        num_blocks=sum((b + c + 15) // 16 + 1 for b, c in zip(bases, counts)) + 8,
                        max_sequences=n, kv_dtype=slmkv.KV_BF16, device=0)
    pool.shuffle(seed)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    caches = [pool.allocate_kv_cache(ctx) for _ in range(n)]
    # history (its own batch, only the sequences that have one)
    hist = [(rng.standard_normal((b, hkv, D)).astype(np.float32),
             rng.standard_normal((b, hkv, D)).astype(np.float32)) for b in bases]
    with_hist = [i for i, b in enumerate(bases) if b > 0]
    if with_hist:
        hk = np.concatenate([hist[i][0] for i in with_hist])
        hv = np.concatenate([hist[i][1] for i in with_hist])
        with pool.begin([caches[i] for i in with_hist], [bases[i] for i in with_hist]) as b:
            b.append_layer(0, to_dev(hk), to_dev(hv), rotate_keys=True)
    # the new tokens: append, then attention over the grown cache
    T = sum(counts)
    q = rng.standard_normal((T, hq, D)).astype(np.float32)
    k = rng.standard_normal((T, hkv, D)).astype(np.float32)
    v = rng.standard_normal((T, hkv, D)).astype(np.float32)
    out = torch.empty((T, hq, D), dtype=torch.float32, device="cuda:0")
    with pool.begin(caches, counts) as b:
        b.append_layer(0, to_dev(k), to_dev(v), rotate_keys=True)
        b.prefill_attention(0, to_dev(q), out, rotate_query=True)
    got = out.cpu().numpy()
    worst, row = 0.0, 0
    for i, (c, base) in enumerate(zip(counts, bases)):
        qz = np.zeros((base, hq, D), np.float32)
        kh = (O.apply_rotary_with_offset(qz, hist[i][0], hq, hkv, D, inv, 0)[1] if base
              else np.zeros((0, hkv, D), np.float32))
        qn, kn = O.apply_rotary_with_offset(q[row:row + c], k[row:row + c], hq, hkv, D, inv, base)
        kk = O.round_to_bfloat16_array(np.concatenate([kh.reshape(base, hkv, D),
                                                       kn.reshape(c, hkv, D)]))
        vv = O.round_to_bfloat16_array(np.concatenate([hist[i][1], v[row:row + c]]))
        qq = np.concatenate([qz, qn.reshape(c, hq, D)])
        ref = O.prefill_attention(qq, kk, vv, hq, hkv, D).reshape(base + c, hq, D)[base:]
        worst = max(worst, float(np.abs(got[row:row + c] - ref).max()))
        row += c
    return worst


@pytest.mark.parametrize("hq,hkv", [(2, 2), (4, 2), (8, 2), (16, 2)])
def test_prefill_bf16_multi_tile_matches_oracle(hq, hkv):
    err = _case(hq, hkv, counts=[1, 127, 128, 129, 300], bases=[0, 0, 0, 0, 0], seed=41)
    assert err <= TOL, err


@pytest.mark.parametrize("hq,hkv", [(4, 2), (8, 2)])
def test_prefill_bf16_after_cached_history_matches_oracle(hq, hkv):
    err = _case(hq, hkv, counts=[3, 64, 130, 200], bases=[200, 5, 130, 250], seed=43)
    assert err <= TOL, err

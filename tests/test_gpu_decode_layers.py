"""slm_batch_decode_layers: a step's decode layers as one launch.

The layers of a step share one plan, so with an f32 pool one kernel runs up
to eight of them (each warp takes its slice of the step's blocks in every
layer in turn; bf16 pools launch once per layer). Its
results must equal the one-layer calls' bit for bit (outputs and appended
K/V), and through them the oracle's forward_cached_token cache part
(attention.rs:794-810) within the decode bar (1e-4 f32, 2e-2 bf16 KV).
"""

import numpy as np
import pytest

import oracle as O
from gpu_util import bits, fill_history, to_dev

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
slmkv = pytest.importorskip("slmkv")

D = 64
TOL = {slmkv.KV_F32: 1e-4, slmkv.KV_BF16: 2e-2}


def _setup(kv_dtype, lengths, layers, hq, hkv, seed, ctx=512):
    rng = np.random.default_rng(seed)
    n = len(lengths)
    pool = slmkv.KvPool(num_layers=layers, num_query_heads=hq, num_key_value_heads=hkv,
                        head_dimension=D, context_length=ctx, rope_theta=10000.0,
                        num_blocks=sum((L + 16) // 16 + 1 for L in lengths) + 8, max_sequences=n,
                        kv_dtype=kv_dtype, device=0)
    pool.shuffle(seed)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    caches = [pool.allocate_kv_cache(ctx) for _ in range(n)]
    ocs = [O.DenseCache(layers, ctx, hkv, D, quantize_bf16=(kv_dtype == slmkv.KV_BF16))
           for _ in range(n)]
    fill_history(caches, ocs, lengths, layers, rng, inv, hkv, D)
    qs = rng.standard_normal((layers, n, hq, D)).astype(np.float32)
    ks = rng.standard_normal((layers, n, hkv, D)).astype(np.float32)
    vs = rng.standard_normal((layers, n, hkv, D)).astype(np.float32)
    return pool, caches, ocs, inv, qs, ks, vs


def _one_layer_calls(pool, caches, qs, ks, vs):
    layers, n, hq, _ = qs.shape
    outs = torch.empty((layers, n, hq, D), device="cuda:0")
    with pool.begin(caches, 1) as b:
        for layer in range(layers):
            b.decode_layer(layer, to_dev(qs[layer]), to_dev(ks[layer]), to_dev(vs[layer]),
                           outs[layer])
    assert b.statuses == [0] * n
    return outs


def _snapshot(caches, layers):
    return [(bits(c.layer_keys(l)), bits(c.layer_values(l))) for c in caches for l in range(layers)]


def _compare(kv_dtype, lengths, layers, hq, hkv, seed, splits=None, oracle=True, ctx=512):
    pool, caches, ocs, inv, qs, ks, vs = _setup(kv_dtype, lengths, layers, hq, hkv, seed, ctx)
    base = [c.sequence_length() for c in caches]
    ref = _one_layer_calls(pool, caches, qs, ks, vs)
    ref_pool = _snapshot(caches, layers)
    for c, L in zip(caches, base):
        c.truncate_all(L)
    dq, dk, dv = to_dev(qs), to_dev(ks), to_dev(vs)
    outs = torch.full_like(ref, float("nan"))
    launches0 = pool.launch_count()
    with pool.begin(caches, 1) as b:
        first = 0
        for cnt in (splits or [layers]):
            b.decode_layers(first, [(dq[l], dk[l], dv[l], outs[l]) for l in range(first, first + cnt)])
            first += cnt
    assert b.statuses == [0] * len(lengths)
    launched = pool.launch_count() - launches0
    assert np.array_equal(bits(outs), bits(ref))
    assert all(np.array_equal(a[0], b_[0]) and np.array_equal(a[1], b_[1])
               for a, b_ in zip(_snapshot(caches, layers), ref_pool))
    if oracle:
        worst = 0.0
        for layer in range(layers):
            r = O.forward_cached_attention_batch(ocs, layer, qs[layer], ks[layer], vs[layer], hq,
                                                 inv, threads=8)
            got = outs[layer].cpu().numpy().reshape(len(lengths), hq * D)
            worst = max(worst, float(np.abs(got - r.reshape(len(lengths), hq * D)).max()))
        assert worst <= TOL[kv_dtype], worst
    return launched


@pytest.mark.parametrize("kv_dtype", [slmkv.KV_F32, slmkv.KV_BF16])
def test_eight_layers_as_one_launch_equal_the_one_layer_calls(kv_dtype):
    lengths = [0, 1, 2, 15, 16, 17, 31, 63, 64, 65, 127, 128, 129, 200, 300, 511]
    launched = _compare(kv_dtype, lengths, layers=8, hq=4, hkv=2, seed=3)
    assert launched == (1 if kv_dtype == slmkv.KV_F32 else 8)  # bf16: a launch per layer


@pytest.mark.parametrize("hq,hkv", [(4, 4), (8, 2), (16, 2)])
def test_group_sizes(hq, hkv):
    _compare(slmkv.KV_F32, [3, 40, 257, 511, 90], layers=4, hq=hq, hkv=hkv, seed=9)


def test_bf16_scaled_gqa_heads():
    _compare(slmkv.KV_BF16, [1, 16, 17, 40, 257, 511, 700], layers=3, hq=32, hkv=8, seed=11,
             ctx=1024)


def test_layer_ranges_and_more_layers_than_one_launch_holds():
    """Ten layers in calls of 3 and 7: the 7 go out as one launch, and a
    call of 10 as 8 + 2."""
    lengths = [5, 77, 300, 12, 511, 256]
    assert _compare(slmkv.KV_F32, lengths, layers=10, hq=4, hkv=2, seed=13, splits=[3, 7],
                    oracle=False) == 2
    assert _compare(slmkv.KV_F32, lengths, layers=10, hq=4, hkv=2, seed=14, oracle=False) == 2


def test_microbench_shape_eight_layers():
    """B=256, lengths U[1,511], Hq=4, Hkv=2, f32, 8 layers: the headline
    step as one launch, equal to the eight one-layer launches."""
    rng = np.random.default_rng(0)
    lengths = rng.integers(1, 512, size=256).tolist()
    assert _compare(slmkv.KV_F32, lengths, layers=8, hq=4, hkv=2, seed=17, oracle=False) == 1


def test_slices_beyond_one_window_fall_back_to_one_launch_per_layer():
    """256 sequences of ~500 tokens with 8 KV heads: ~37 blocks per warp,
    more than a warp's 32-entry window, so each layer is its own launch."""
    rng = np.random.default_rng(23)
    lengths = rng.integers(480, 511, size=256).tolist()
    assert _compare(slmkv.KV_F32, lengths, layers=2, hq=8, hkv=8, seed=23, oracle=False) == 2


def test_non_finite_query_fails_only_its_sequence():
    lengths = [40, 300, 17, 511]
    layers, hq, hkv = 6, 4, 2
    pool, caches, ocs, inv, qs, ks, vs = _setup(slmkv.KV_F32, lengths, layers, hq, hkv, 29)
    qs[4, 2, 1, 7] = np.nan  # layer 4, sequence 2
    dq, dk, dv = to_dev(qs), to_dev(ks), to_dev(vs)
    outs = torch.empty((layers, len(lengths), hq, D), device="cuda:0")
    b = pool.begin(caches, 1)
    b.decode_layers(0, [(dq[l], dk[l], dv[l], outs[l]) for l in range(layers)])
    st = b.end(raise_on_error=False)
    assert st[2] == slmkv.ERR_NON_FINITE and st[0] == st[1] == st[3] == 0
    assert [c.sequence_length() for c in caches] == [41, 301, 17, 512]


def test_rejects_overlapping_layer_buffers_before_launching():
    lengths = [10, 20]
    pool, caches, ocs, inv, qs, ks, vs = _setup(slmkv.KV_F32, lengths, 3, 4, 2, 31)
    dq, dk, dv = to_dev(qs), to_dev(ks), to_dev(vs)
    outs = torch.empty((3, 2, 4, D), device="cuda:0")
    launches0 = pool.launch_count()
    b = pool.begin(caches, 1)
    with pytest.raises(slmkv.InvalidInput):
        b.decode_layers(0, [(dq[0], dk[0], dv[0], outs[0]), (dq[1], dk[1], dv[1], dq[0])])
    with pytest.raises(slmkv.InvalidInput):
        b.decode_layers(1, [(dq[1], dk[1], dv[1], outs[1]), (dq[2], dk[2], dv[2], outs[1])])
    assert pool.launch_count() == launches0
    b.rollback()
    assert [c.sequence_length() for c in caches] == lengths


def test_host_buffers_equal_the_device_call_with_steps_in_flight():
    """slm_batch_decode_layers_host: inputs copied in from pinned host memory,
    outputs copied back before the batch's wait returns; three steps
    submitted before any is waited for (each its own staging and host
    buffers), every output equal to the device-buffer call's bit for bit."""
    lengths = [0, 3, 16, 17, 200, 505, 45, 130]
    layers, hq, hkv = 8, 4, 2
    pool, caches, ocs, inv, qs, ks, vs = _setup(slmkv.KV_F32, lengths, layers, hq, hkv, 37)
    base = [c.sequence_length() for c in caches]
    rng = np.random.default_rng(38)
    steps = 3
    hq_ = [torch.from_numpy(rng.standard_normal(qs.shape).astype(np.float32)).pin_memory()
           for _ in range(steps)]
    hk_ = [torch.from_numpy(rng.standard_normal(ks.shape).astype(np.float32)).pin_memory()
           for _ in range(steps)]
    hv_ = [torch.from_numpy(rng.standard_normal(vs.shape).astype(np.float32)).pin_memory()
           for _ in range(steps)]
    hout = [torch.full(qs.shape, float("nan")).pin_memory() for _ in range(steps)]
    # step 0's inputs as one pinned block (Q, K, V back to back: one copy in)
    blk = torch.cat([hq_[0].reshape(-1), hk_[0].reshape(-1), hv_[0].reshape(-1)]).pin_memory()
    nq, nk = hq_[0].numel(), hk_[0].numel()
    hq_[0] = blk[:nq].view(qs.shape)
    hk_[0] = blk[nq:nq + nk].view(ks.shape)
    hv_[0] = blk[nq + nk:].view(vs.shape)
    inflight = []
    for i in range(steps):
        b = pool.begin(caches, 1)
        b.decode_layers_host(0, layers, hq_[i], hk_[i], hv_[i], hout[i])
        inflight.append(b.submit())
    for b in inflight:
        assert b.wait() == [0] * len(lengths)
    got = [h.clone() for h in hout]
    # the same three steps from device buffers
    for c, L in zip(caches, base):
        c.truncate_all(L)
    for i in range(steps):
        dq, dk, dv = hq_[i].cuda(), hk_[i].cuda(), hv_[i].cuda()
        out = torch.empty_like(dq)
        with pool.begin(caches, 1) as b:
            b.decode_layers(0, [(dq[l], dk[l], dv[l], out[l]) for l in range(layers)])
        assert np.array_equal(bits(got[i]), bits(out))
    assert [c.sequence_length() for c in caches] == [L + steps for L in base]

"""CPU checks of the C ABI: the library loads, exports every declared symbol,
and the host bookkeeping follows the reference's KvCache contract on a
host-only context (device -1: no compute calls are made)."""

import re
from pathlib import Path

import pytest

import slmkv

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "slmkv.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:slm_status|const char\*)\s+(slm_\w+)\s*\(", text,
                                 re.M)))


def test_library_exports_every_declared_symbol():
    lib = slmkv.lib()
    names = declared_symbols()
    assert len(names) >= 30
    for name in names:
        assert hasattr(lib, name), name
    assert sorted(slmkv.SIGNATURES) == names


def host_pool(**kw):
    args = dict(num_layers=2, num_query_heads=2, num_key_value_heads=1, head_dimension=64,
                context_length=8, num_blocks=16, max_sequences=3, device=None)
    args.update(kw)
    return slmkv.KvPool(**args)


@pytest.mark.parametrize("kw,needle", [
    (dict(num_layers=0), "greater than zero"),
    (dict(num_query_heads=3, num_key_value_heads=2), "divisible"),
    (dict(head_dimension=32), "head_dimension 64"),
    (dict(rope_theta=-1.0), "theta"),
    (dict(num_query_heads=3, num_key_value_heads=1), "1, 2, 4 or 8"),
    (dict(num_blocks=0), "num_blocks"),
    (dict(kv_dtype=7), "kv_dtype"),
])
def test_invalid_configurations_are_rejected(kw, needle):
    with pytest.raises(slmkv.InvalidConfiguration) as e:
        host_pool(**kw)
    assert "invalid model configuration" in str(e.value)
    assert needle in str(e.value)


def test_cache_allocation_limits():
    """kv_cache.rs:27-41: 1..=context_length."""
    pool = host_pool()
    with pytest.raises(slmkv.InvalidConfiguration):
        pool.allocate_kv_cache(0)
    with pytest.raises(slmkv.InvalidConfiguration) as e:
        pool.allocate_kv_cache(9)
    assert "1..=8" in str(e.value)
    caches = [pool.allocate_kv_cache(4) for _ in range(3)]
    with pytest.raises(slmkv.InvalidInput):
        pool.allocate_kv_cache(4)
    caches[0].free()
    pool.allocate_kv_cache(4)


def test_fresh_cache_state():
    """kv_cache.rs:446-456"""
    pool = host_pool()
    c = pool.allocate_kv_cache(4)
    assert c.sequence_length() == 0 and c.is_empty() and c.is_synchronized()
    assert c.layer_sequence_length(0) == 0 and c.layer_sequence_length(1) == 0
    assert c.remaining_capacity() == 4
    assert c.blocks() == []
    with pytest.raises(slmkv.InvalidInput) as e:
        c.layer_sequence_length(2)
    assert "layer index 2 is outside 0..2" in str(e.value)


def test_truncation_rules():
    """kv_cache.rs:302-346 on an empty cache: cannot grow while truncating."""
    pool = host_pool()
    c = pool.allocate_kv_cache(4)
    c.truncate_all(0)
    with pytest.raises(slmkv.InvalidInput) as e:
        c.truncate_all(1)
    assert "cannot restore all layers to 1" in str(e.value)
    with pytest.raises(slmkv.InvalidInput) as e:
        c.truncate_layer(1, 2)
    assert "cannot extend layer 1 from 0 to 2" in str(e.value)
    c.clear()
    assert c.is_empty()
    pool.truncate_many([c], [0])


def test_compute_calls_need_a_device():
    pool = host_pool()
    c = pool.allocate_kv_cache(4)
    rc = slmkv.lib().slm_append_layer(pool.handle, c.seq_id, 0, None, None, 1, 1, None)
    assert rc == slmkv.ERR_NO_DEVICE
    assert "no device" in slmkv.lib().slm_last_error(pool.handle).decode()
    with pytest.raises(slmkv.DeviceError):
        pool.begin([c], 1)
    assert c.sequence_length() == 0


def test_prefix_index_starts_empty_and_shuffle_needs_an_idle_pool():
    pool = host_pool()
    c = pool.allocate_kv_cache(8)
    assert c.attach_prefix(list(range(8))) == 0
    assert pool.stats() == (16, 0)
    pool.shuffle(123)
    assert pool.stats() == (16, 0)
    assert c.publish_prefix([]) == 0
    with pytest.raises(slmkv.InvalidInput):
        c.publish_prefix([1] * 16)  # longer than the cache


def test_launch_counter_starts_at_zero():
    assert host_pool().launch_count() == 0

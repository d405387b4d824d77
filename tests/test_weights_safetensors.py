"""SafeTensors weight loading (slm_safetensors_check / slm_model_load_safetensors)
against ModelWeights::load (weights.rs:117-190), on the CPU: files written
here in the format's published layout (8-byte little-endian header length,
JSON header, byte buffer), the 8M model's expected parameter count
(artifacts/small-lm-8m/config.json: 7 999 744), and every rejection the
reference makes: missing and unexpected names, a non-F32 dtype, a wrong
shape, a wrong parameter count; plus the format's own rules (truncated file,
header past the end, holes in the buffer, offsets that do not match the
shape)."""

import json
import struct

import numpy as np
import pytest

import slmkv

SMALL = dict(vocab_size=32, hidden_size=128, intermediate_size=40, num_layers=2,
             num_key_value_heads=1, head_dimension=64)


def layout(vocab_size, hidden_size, intermediate_size, num_layers, num_key_value_heads,
           head_dimension):
    return slmkv.model_tensor_shapes(vocab_size=vocab_size, hidden_size=hidden_size,
                                     intermediate_size=intermediate_size, num_layers=num_layers,
                                     kv_width=num_key_value_heads * head_dimension)


def write_safetensors(path, tensors, dtypes=None, order=None, pad=0, offsets=None):
    """tensors: {name: float32 array}; writes them back to back in `order`."""
    names = order or list(tensors)
    header, buf, at = {}, bytearray(), 0
    for n in names:
        a = np.ascontiguousarray(tensors[n])
        raw = a.astype("<f4").tobytes() if a.dtype == np.float32 else a.tobytes()
        header[n] = {"dtype": (dtypes or {}).get(n, "F32"), "shape": list(a.shape),
                     "data_offsets": [at, at + len(raw)]}
        buf += raw
        at += len(raw)
    if offsets:
        for n, off in offsets.items():
            header[n]["data_offsets"] = off
    header["__metadata__"] = {"format": "pt"}
    h = json.dumps(header).encode() + b" " * pad
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + bytes(buf))


def random_tensors(cfg, seed=0):
    rng = np.random.default_rng(seed)
    return {n: rng.standard_normal(s).astype(np.float32) for n, s in layout(**cfg)}


def check(path, cfg, expected=0):
    return slmkv.check_safetensors(path, expected_parameter_count=expected, **cfg)


def test_eight_m_model_parameter_count(tmp_path):
    cfg = dict(vocab_size=8192, hidden_size=256, intermediate_size=704, num_layers=8,
               num_key_value_heads=2, head_dimension=64)
    n = sum(int(np.prod(s)) for _, s in layout(**cfg))
    assert n == 7_999_744  # artifacts/small-lm-8m/config.json expected_parameter_count
    p = tmp_path / "m.safetensors"
    write_safetensors(p, {k: np.zeros(s, np.float32) for k, s in layout(**cfg)})
    assert check(p, cfg, 7_999_744) == 7_999_744


def test_valid_file_any_order_and_padding(tmp_path):
    t = random_tensors(SMALL)
    p = tmp_path / "ok.safetensors"
    write_safetensors(p, t, order=sorted(t, reverse=True), pad=7)
    assert check(p, SMALL) == sum(a.size for a in t.values())


@pytest.mark.parametrize("case", ["missing", "unexpected", "dtype", "shape", "count"])
def test_reference_rejections(tmp_path, case):
    t = random_tensors(SMALL)
    dtypes, expected = None, 0
    if case == "missing":
        del t["layers.1.up_proj.weight"]
    elif case == "unexpected":
        t["lm_head.weight"] = np.zeros((2, 2), np.float32)
    elif case == "dtype":
        t["final_norm.weight"] = t["final_norm.weight"].astype(np.float16)
        dtypes = {"final_norm.weight": "F16"}
    elif case == "shape":
        t["layers.0.k_proj.weight"] = t["layers.0.k_proj.weight"].T.copy()
    elif case == "count":
        expected = 12345
    p = tmp_path / f"{case}.safetensors"
    write_safetensors(p, t, dtypes=dtypes)
    with pytest.raises(slmkv.InvalidInput) as e:
        check(p, SMALL, expected)
    msg = str(e.value)
    assert "invalid weights" in msg
    if case == "missing":
        assert "missing=[layers.1.up_proj.weight]" in msg
    if case == "unexpected":
        assert "unexpected=[lm_head.weight]" in msg
    if case == "dtype":
        assert "must have dtype F32" in msg
    if case == "shape":
        assert "has shape" in msg
    if case == "count":
        assert "expected 12345" in msg


@pytest.mark.parametrize("case", ["truncated", "header_past_end", "hole", "span"])
def test_format_rejections(tmp_path, case):
    t = random_tensors(SMALL)
    p = tmp_path / f"{case}.safetensors"
    if case == "hole":
        # move the last tensor 4 bytes later: a hole and a span past the buffer
        last = list(t)[-1]
        b = 4 * sum(a.size for a in t.values()) - 4 * t[last].size
        write_safetensors(p, t, offsets={last: [b + 4, b + 4 + 4 * t[last].size]})
    elif case == "span":
        first = list(t)[0]
        write_safetensors(p, t, offsets={first: [0, 8]})
    else:
        write_safetensors(p, t)
        raw = p.read_bytes()
        if case == "truncated":
            p.write_bytes(raw[:-3])
        else:
            p.write_bytes(struct.pack("<Q", len(raw)) + raw[8:])
    with pytest.raises(slmkv.InvalidInput) as e:
        check(p, SMALL)
    assert "invalid weights" in str(e.value)

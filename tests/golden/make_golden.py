"""Generate the committed golden fixtures that pin the CPU oracle.

Two files are written next to this script:

known_answers.json
    The known-answer cases of small-lm-rs's own Rust unit tests for the hot
    path (rope.rs, softmax.rs, linear.rs, kv_cache.rs, attention.rs), with the
    inputs and expected outputs those tests state, each tagged with its
    file:line. Expected values that the Rust tests define by a formula (for
    example the bf16 projection cases) are evaluated here in exact rational
    arithmetic, independently of the oracle.

numpy_reference_vectors.json
    Seeded vectors computed by importing the reference's independent NumPy
    decoder (src/smalllm/reference.py: apply_rope, _softmax, rms_norm,
    situ_glu) from a checkout of the reference. That module runs only in the
    build container; the vectors it produced are committed so the GPU box
    never needs the reference.

Run from the repository root:  python tests/golden/make_golden.py [REF_ROOT]
"""

from __future__ import annotations

import json
import math
import sys
from fractions import Fraction
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
F32_MIN = float(np.finfo(np.float32).min)


def f32(x) -> float:
    return float(np.float32(x))


def bf16(x: float) -> float:
    """linear.rs:14-23, on the exact float32 bit pattern."""
    bits = int(np.array([x], np.float32).view(np.uint32)[0])
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) & 0xFFFFFFFF) & 0xFFFF0000
    return float(np.array([rounded], np.uint32).view(np.float32)[0])


def fma_exact(a: float, b: float, c: float) -> float:
    """Correctly rounded f32 fma: round(a*b + c) once, via exact rationals."""
    exact = Fraction(a) * Fraction(b) + Fraction(c)
    d = float(exact)  # exact here: operands carry <= 24-bit mantissas
    assert Fraction(d) == exact, "not exactly representable in double"
    return f32(d)


def known_answers() -> dict:
    s1, c1 = f32(math.sin(1.0)), f32(math.cos(1.0))
    inv_sqrt2 = f32(1.0 / math.sqrt(2.0))
    e1 = f32(math.exp(1.0))
    first = f32(1.0 / (1.0 + e1))

    # linear.rs:177-200
    lin_x = [1.0039062, -0.99609375]
    lin_w = [0.33398438, 0.66796875, -0.25, 0.125]
    lin_x = [f32(v) for v in lin_x]
    lin_w = [f32(v) for v in lin_w]
    lin_expected = []
    for row in (lin_w[0:2], lin_w[2:4]):
        acc = 0.0
        for i in range(2):
            acc = fma_exact(bf16(lin_x[i]), bf16(row[i]), acc)
        lin_expected.append(acc)

    # linear.rs:203-230
    mr_x = [f32(v) for v in [1.0039062, -0.99609375, 0.50390625, 1.9960938]]
    mr_w = [f32(v) for v in [0.33398438, 0.66796875, -0.25195312, 0.12695312]]
    mr_expected = []
    for xr in (mr_x[0:2], mr_x[2:4]):
        for wr in (mr_w[0:2], mr_w[2:4]):
            prod = f32(Fraction(bf16(xr[1])) * Fraction(bf16(wr[1])))
            mr_expected.append(fma_exact(bf16(xr[0]), bf16(wr[0]), prod))

    # linear.rs:233-243
    fp_x = lin_x
    fp_w = [f32(0.33398438), f32(0.66796875)]
    fp_expected = fma_exact(fp_x[0], fp_w[0], f32(Fraction(fp_x[1]) * Fraction(fp_w[1])))

    return {
        "rope_inverse_frequencies": {
            "source": "rust/engine/src/rope.rs:158-164",
            "head_dim": 4, "theta": 10000.0, "expected": [1.0, 0.01], "atol": 1e-6},
        "rope_position_zero_identity": {
            "source": "rust/engine/src/rope.rs:166-174",
            "head_dim": 4, "theta": 10000.0, "head": [1.0, 2.0, 3.0, 4.0], "position": 0,
            "expected": [1.0, 2.0, 3.0, 4.0], "exact": True},
        "rope_interleaved_pairs": {
            "source": "rust/engine/src/rope.rs:176-188",
            "head_dim": 2, "theta": 10000.0, "position": 1,
            "query": [1.0, 0.0], "key": [0.0, 1.0],
            "expected_query": [c1, s1], "expected_key": [-s1, c1], "atol": 1e-6},
        "rope_multiple_heads_and_bad_shapes": {
            "source": "rust/engine/src/rope.rs:190-198",
            "head_dim": 2, "theta": 10000.0, "values": [1.0, 0.0, 0.0, 1.0],
            "num_heads_ok": 2, "num_heads_bad": 3, "position": 1},
        "softmax_large_logits": {
            "source": "rust/engine/src/softmax.rs:271-280",
            "values": [1000.0, 1001.0], "expected": [first, f32(1.0 - first)], "atol": 1e-6},
        "softmax_rows": {
            "source": "rust/engine/src/softmax.rs:282-292",
            "values": [0.0, 0.0, 2.0, 2.0], "rows": 2, "columns": 2,
            "expected": [0.5, 0.5, 0.5, 0.5], "atol": 1e-6},
        "softmax_rejects": {
            "source": "rust/engine/src/softmax.rs:294-298",
            "empty": [], "non_finite": [0.0, "nan"]},
        "bf16_rounding": {
            "source": "rust/engine/src/linear.rs:158-163",
            "cases": [[1.0, 1.0], [-2.0, -2.0], ["inf", "inf"]]},
        "linear_layout": {
            "source": "rust/engine/src/linear.rs:165-174",
            "input": [1.0, 2.0], "rows": 1, "in": 2, "weight": [3.0, 4.0, 5.0, 6.0],
            "out": 2, "expected": [11.0, 17.0]},
        "linear_bf16_single_row": {
            "source": "rust/engine/src/linear.rs:176-200",
            "input": lin_x, "rows": 1, "in": 2, "weight": lin_w, "out": 2,
            "expected": lin_expected},
        "linear_bf16_multi_row": {
            "source": "rust/engine/src/linear.rs:202-230",
            "input": mr_x, "rows": 2, "in": 2, "weight": mr_w, "out": 2,
            "expected": mr_expected},
        "linear_fp32": {
            "source": "rust/engine/src/linear.rs:232-243",
            "input": fp_x, "rows": 1, "in": 2, "weight": fp_w, "out": 1,
            "expected": [fp_expected]},
        "kv_cache_tiny": {
            "source": "rust/engine/src/kv_cache.rs:419-526",
            "num_layers": 2, "kv_heads": 1, "head_dim": 2,
            "append_keys": [1.0, 2.0, 3.0, 4.0], "append_values": [5.0, 6.0, 7.0, 8.0],
            "key_head_0_1_0": [3.0, 4.0], "value_head_0_0_0": [5.0, 6.0]},
        "causal_scores": {
            "source": "rust/engine/src/attention.rs:1005-1038",
            "tokens": 2, "q_heads": 2, "kv_heads": 1, "head_dim": 2,
            "query": [1.0, 0.0, 0.0, 1.0, 1.0, 1.0, 1.0, -1.0], "key": [1.0, 0.0, 0.0, 1.0],
            "expected": [inv_sqrt2, F32_MIN, inv_sqrt2, inv_sqrt2,
                         0.0, F32_MIN, inv_sqrt2, -inv_sqrt2],
            "masked_indices": [1, 5], "atol": 1e-6},
        "causal_probabilities": {
            "source": "rust/engine/src/attention.rs:1040-1067",
            "tokens": 2, "q_heads": 1, "kv_heads": 1, "head_dim": 2,
            "query": [1.0, 0.0, 1.0, 1.0], "key": [1.0, 0.0, 0.0, 1.0],
            "expected": [1.0, 0.0, 0.5, 0.5], "atol": 1e-6},
        "gqa_value_aggregation": {
            "source": "rust/engine/src/attention.rs:1069-1099",
            "tokens": 2, "q_heads": 2, "kv_heads": 1, "head_dim": 2,
            "value": [10.0, 20.0, 30.0, 40.0],
            "probabilities": [1.0, 0.0, 0.25, 0.75, 1.0, 0.0, 0.5, 0.5],
            "expected": [10.0, 20.0, 10.0, 20.0, 25.0, 35.0, 20.0, 30.0]},
        "rotary_offset_equals_prefill_position": {
            "source": "rust/engine/src/attention.rs:1101-1131",
            "head_dim": 2, "theta": 10000.0,
            "full_query": [1.0, 0.0, 1.0, 0.0], "full_key": [0.0, 1.0, 0.0, 1.0],
            "token_query": [1.0, 0.0], "token_key": [0.0, 1.0], "offset": 1},
        "rope_queries_and_keys_only": {
            "source": "rust/engine/src/attention.rs:1133-1169",
            "tokens": 2, "q_heads": 2, "kv_heads": 1, "head_dim": 2, "theta": 10000.0,
            "query": [1.0, 0.0, 0.0, 1.0, 1.0, 0.0, 0.0, 1.0], "key": [1.0, 0.0, 0.0, 1.0],
            "value": [5.0, 6.0, 7.0, 8.0],
            "expected_query_0_0": [1.0, 0.0], "expected_query_1_0": [c1, s1],
            "expected_key_1_0": [-s1, c1], "atol": 1e-6},
        "single_token_attention": {
            "source": "rust/engine/src/attention.rs:1197-1222",
            "q_heads": 2, "kv_heads": 1, "head_dim": 2, "theta": 10000.0,
            "query": [1.0, 2.0, 3.0, 4.0], "key": [1.0, 2.0], "value": [1.0, 2.0],
            "expected": [1.0, 2.0, 1.0, 2.0]},
        "sequential_cached_equals_fresh": {
            "source": "rust/engine/src/attention.rs:1262-1301",
            "q_heads": 2, "kv_heads": 1, "head_dim": 2, "theta": 10000.0,
            "hidden_states": [1.0, 2.0, 3.0, 4.0, -1.0, 0.5, 2.0, -0.25],
            "note": "identity q/o projections, k/v = first two hidden dims", "atol": 1e-6},
    }


def numpy_reference_vectors(ref_root: Path) -> dict:
    sys.path.insert(0, str(ref_root / "src"))
    from smalllm import reference as R  # the reference's own NumPy decoder

    rng = np.random.default_rng(20240601)
    out: dict = {"source": "src/smalllm/reference.py (imported from the reference)"}

    # apply_rope: reference.py:24-50 on [1, T, H, d] with arbitrary positions.
    positions = np.array([0, 1, 2, 3, 15, 16, 17, 100, 255, 256, 511, 1000, 4095, 8191],
                         np.int32)
    d = 64
    q = rng.standard_normal((1, positions.size, 4, d)).astype(np.float32)
    k = rng.standard_normal((1, positions.size, 2, d)).astype(np.float32)
    rq, rk = R.apply_rope(q, k, positions=positions, theta=10_000.0)
    out["rope"] = {"positions": positions.tolist(), "head_dim": d, "theta": 10000.0,
                   "query": q.ravel().tolist(), "key": k.ravel().tolist(),
                   "rotated_query": rq.ravel().tolist(), "rotated_key": rk.ravel().tolist(),
                   "q_heads": 4, "kv_heads": 2,
                   "note": "NumPy float32 sin/cos; compare with a ~1e-5 tolerance"}

    # _softmax: reference.py:79-82 on rows of causal-style scores.
    x = (rng.standard_normal((6, 37)) * 3.0).astype(np.float32)
    out["softmax"] = {"rows": 6, "columns": 37, "values": x.ravel().tolist(),
                      "expected": R._softmax(x).ravel().tolist()}

    # Masked causal attention in the reference's NumPy formulation
    # (reference.py:123-135: rope, scores / sqrt(d), -inf mask, softmax, PV).
    T, Hq, Hkv = 9, 4, 2
    q = rng.standard_normal((1, T, Hq, d)).astype(np.float32)
    k = rng.standard_normal((1, T, Hkv, d)).astype(np.float32)
    v = rng.standard_normal((1, T, Hkv, d)).astype(np.float32)
    pos = np.arange(T, dtype=np.int32)
    rq, rk = R.apply_rope(q, k, positions=pos, theta=10_000.0)
    g = Hq // Hkv
    qg = rq.reshape(1, T, Hkv, g, d)
    scores = np.einsum("btkgh,bskh->bkgts", qg, rk).astype(np.float32)
    scores /= np.float32(math.sqrt(d))
    causal = np.arange(T)[:, None] >= np.arange(T)[None, :]
    scores = np.where(causal[None, None, None], scores, np.float32(-np.inf))
    probs = R._softmax(scores)
    att = np.einsum("bkgts,bskh->btkgh", probs, v).reshape(T, Hq, d).astype(np.float32)
    out["causal_attention"] = {
        "tokens": T, "q_heads": Hq, "kv_heads": Hkv, "head_dim": d, "theta": 10000.0,
        "query": q.ravel().tolist(), "key": k.ravel().tolist(), "value": v.ravel().tolist(),
        "expected": att.ravel().tolist(),
        "note": "query/key unrotated; expected uses the reference's rope + -inf mask"}
    return out


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <small-lm-rs checkout>")
    ref_root = Path(sys.argv[1])
    if not (ref_root / "src" / "smalllm" / "reference.py").exists():
        sys.exit(f"{ref_root}: not a small-lm-rs checkout (src/smalllm/reference.py missing)")
    (HERE / "known_answers.json").write_text(json.dumps(known_answers(), indent=1) + "\n")
    vec = numpy_reference_vectors(ref_root)
    (HERE / "numpy_reference_vectors.json").write_text(json.dumps(vec) + "\n")


if __name__ == "__main__":
    main()

"""Live kernel timeline of a model decode step (profiling builds only).

ncu serializes the launches it measures, so it cannot show how the chained
kernels of a step (programmatic dependent launch) overlap on the GPU. The
timeline build of the library (`make -C small-lm-rs_b200/csrc timeline`:
slmkv/libslmkv_timeline.so, compiled with SLMKV_TIMELINE) has every warp of
every kernel record its kernel kind, SM and %globaltimer at entry and exit;
this module runs the scaled GQA model's decode steps on it and prints, per
kernel, where a step's time goes:

    python -m slmkv.timeline [--workload gqa-model|model|prefix] [--steps 6] [--batch 16]

(run from the repository root with small-lm-rs_b200 on sys.path, as the
tests do). The numbers are of the timeline build, whose records cost a few
percent; the bench's own figures come from the product library.
"""

from __future__ import annotations

import argparse
import ctypes as C
import sys
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
ROOT = PKG.parents[1]

RECORD = np.dtype([("kind", "<u2"), ("sm", "<u2"), ("block", "<u4"), ("t0", "<u8"), ("t1", "<u8")])
NAMES = {1: "decode", 2: "decode (layers)", 3: "append", 5: "prefill", 6: "exact attention", 7: "apply",
         8: "embed", 9: "rmsnorm", 10: "round", 11: "situ", 12: "proj", 13: "head", 14: "argmax",
         15: "proj1", 16: "prefill_tc", 17: "mlp1 (cluster)", 32: "gemm_qkv", 33: "gemm_o", 34: "gemm_gu",
         35: "gemm_down", 36: "gemm_head"}
MARK_WAITED, MARK_SLICE_DONE = 24, 25  # decode warps (slmkv_timeline.h)
EXACT_MARKS = {26: "past the wait", 28: "scored", 29: "summed", 27: "softmax done", 30: "folded"}
MLP_MARKS = {56: "past the wait", 57: "weights in", 58: "O + barrier", 59: "FFN norm",
             60: "gate/up + barrier", 61: "down + barrier", 62: "attn norm"}


def is_mark(kind):
    return ((kind >= 24) & (kind < 32)) | (kind >= 40)


def launches(rec):
    """Consecutive records of one kind (sorted by entry) as launches:
    {kind, t0 (first entry), t1 (last exit), n (warps)}."""
    runs = []
    for r in rec:
        if runs and runs[-1]["kind"] == r["kind"] and r["t0"] <= runs[-1]["t1"] + 2000:
            g = runs[-1]
            g["t1"] = max(g["t1"], int(r["t1"]))
            g["n"] += 1
        else:
            runs.append({"kind": int(r["kind"]), "t0": int(r["t0"]), "t1": int(r["t1"]), "n": 1})
    return runs


def run_steps(workload: str, steps: int, batch: int):
    """bench.py's gqa-model workload (the scaled GQA model, 16 sequences of
    1-8 k tokens, row-GEMM projections), model workload (the 8M model,
    batch 1, a 64-token prompt, exact-order projections) or prefix workload's
    decode shape (the 8M model, 64 sequences of 384 tokens), one GPU: prefill,
    10 untimed decode steps, then `steps` recorded ones. Returns the records
    sorted by entry time."""
    import torch

    import slmkv

    slmkv.LIB_PATH = PKG / "libslmkv_timeline.so"
    if not slmkv.LIB_PATH.exists():
        raise SystemExit(f"{slmkv.LIB_PATH} is missing: make -C small-lm-rs_b200/csrc timeline")
    sys.path.insert(0, str(ROOT))
    import bench

    gqa = workload == "gqa-model"
    bench.select_workload(workload, batch)
    B = bench.B
    dev = torch.device("cuda:0")
    if gqa:
        lens = [int(x) for x in np.random.default_rng(0).integers(bench.LEN_LO, bench.LEN_HI + 1,
                                                                 size=B * 8)[:B]]
    else:
        lens = [bench.LEN_LO] * B
    prng = np.random.default_rng(1)
    prompts = [prng.integers(0, bench.MODEL_VOCAB, size=L).astype(np.int32) for L in lens]
    pool = slmkv.KvPool(num_layers=bench.LAYERS, num_query_heads=bench.HQ,
                        num_key_value_heads=bench.HKV, head_dimension=bench.D,
                        context_length=bench.CTX,
                        num_blocks=sum(-(-(L + 256) // 16) for L in lens) + 8, max_sequences=B,
                        kv_dtype=slmkv.KV_BF16 if gqa else slmkv.KV_F32, device=0)
    pool.shuffle(1)
    inter = bench.GQA_MODEL_INTER if gqa else bench.MODEL_INTER
    model = slmkv.Model(pool, vocab_size=bench.MODEL_VOCAB, intermediate_size=inter,
                        tensors=bench.model_tensors(0, inter))
    if gqa:
        model.set_exact_rows(0)
    caches = [pool.allocate_kv_cache(bench.CTX) for _ in lens]
    tok = [torch.zeros(B, dtype=torch.int32, device=dev) for _ in range(2)]
    with pool.begin(caches, lens) as b:
        model.prefill(b, torch.from_numpy(np.concatenate(prompts)).to(dev), None, tok[0])
    plan = pool.step_plan(caches, 1)

    def decode(n):
        inflight = []
        for i in range(n):
            b = plan.begin()
            model.decode(b, tok[i % 2], None, tok[(i + 1) % 2])
            inflight.append(b.submit())
            while len(inflight) > 1:
                inflight.pop(0).wait()
        for b in inflight:
            b.wait()

    decode(10)
    torch.cuda.synchronize()
    cap = 1 << 20
    buf = torch.zeros(cap * RECORD.itemsize, dtype=torch.uint8, device=dev)
    cnt = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = slmkv.lib()
    if lib.slmkv_timeline_set(C.c_void_p(buf.data_ptr()), C.c_void_p(cnt.data_ptr()), C.c_uint32(cap)):
        raise SystemExit("slmkv_timeline_set failed")
    decode(steps)
    torch.cuda.synchronize()
    lib.slmkv_timeline_set(None, None, C.c_uint32(0))
    n = int(cnt.item())
    if n >= cap:
        raise SystemExit("timeline buffer full: fewer --steps")
    rec = np.frombuffer(buf[: n * RECORD.itemsize].cpu().numpy().tobytes(), dtype=RECORD)
    pool.close()
    return np.sort(rec, order="t0")


def pct(a, ps=(0, 0.1, 0.5, 0.9, 0.99, 1.0)):
    a = np.sort(a)
    return " / ".join(f"{a[int(p * (len(a) - 1))]:.1f}" for p in ps)


def report(rec):
    mk = is_mark(rec["kind"])
    marks = rec[mk]
    runs = launches(rec[~mk])
    steps = []
    for g in runs:
        if g["kind"] == 8:  # embed opens a step
            steps.append([])
        if steps:
            steps[-1].append(g)
    full = steps[1:-1]  # whole steps only
    print(f"steps: {len(full)}; step time (embed to embed, us): " +
          ", ".join(f"{(steps[i + 1][0]['t0'] - steps[i][0]['t0']) / 1e3:.1f}"
                    for i in range(len(steps) - 1)))
    print("per kernel: launches a step, mean duration (first entry to last exit), and the time "
          "from its first entry to the next kernel's (its share of the step), us")
    tot = {}
    for st in full:
        for i, g in enumerate(st):
            d = tot.setdefault(NAMES.get(g["kind"], str(g["kind"])), [0, 0.0, 0.0])
            d[0] += 1
            d[1] += (g["t1"] - g["t0"]) / 1e3
            if i + 1 < len(st):
                d[2] += (st[i + 1]["t0"] - g["t0"]) / 1e3
    for k, (c, dur, share) in sorted(tot.items(), key=lambda x: -x[1][2]):
        print(f"  {k:16s} {c / len(full):5.1f}  {dur / c:7.2f}  {share / len(full):8.1f}")
    st = full[len(full) // 2]
    base = st[0]["t0"]
    print("one step's first layer (entry / exit, us from the step's start):")
    for g in st[:12]:
        print(f"  {NAMES.get(g['kind'], g['kind']):16s} {(g['t0'] - base) / 1e3:8.2f} "
              f"{(g['t1'] - base) / 1e3:8.2f}")
    gemm_marks = [(32 + md, {48 + md: "producer past the wait", 40 + md: "MMAs done",
                                64 + md: "partials", 72 + md: "stored"}) for md in range(4)]
    for kind, names in [(6, EXACT_MARKS), (17, MLP_MARKS)] + gemm_marks:
        gs = [g for s in full for g in s if g["kind"] == kind]
        if not gs:
            continue
        print(f"{NAMES[kind]}: phases, median over launches of the first / last warp's time "
              "from the launch's first entry (us)")
        row = []
        for k, nm in names.items():
            ts = []
            for g in gs:
                t = marks[(marks["kind"] == k) & (marks["t0"] >= g["t0"]) & (marks["t0"] <= g["t1"])]["t0"]
                if len(t):
                    ts.append(((int(t.min()) - g["t0"]) / 1e3, (int(t.max()) - g["t0"]) / 1e3))
            if ts:
                ts = np.array(ts)
                row.append(f"{nm} {np.median(ts[:, 0]):.2f} / {np.median(ts[:, 1]):.2f}")
        row.append(f"exit {np.median([(g['t1'] - g['t0']) / 1e3 for g in gs]):.2f}")
        print("  " + "; ".join(row))
    dec = [g for s in full for g in s if g["kind"] == 1]
    if dec:
        print("decode launches, warps' times from the launch's first entry (p0 / 10 / 50 / 90 / "
              "99 / 100, us):")
        for g in dec[:3]:
            sel = lambda k: marks[(marks["kind"] == k) & (marks["t0"] >= g["t0"]) &
                                  (marks["t0"] <= g["t1"])]["t0"]
            w = rec[(rec["kind"] == 1) & (rec["t0"] >= g["t0"]) & (rec["t1"] <= g["t1"])]
            f = lambda x: (x.astype(np.int64) - g["t0"]) / 1e3
            print(f"  past the wait {pct(f(sel(MARK_WAITED)))}; slice done "
                  f"{pct(f(sel(MARK_SLICE_DONE)))}; exit {pct(f(w['t1']))}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", choices=["gqa-model", "model", "prefix"], default="gqa-model")
    ap.add_argument("--steps", type=int, default=6)
    ap.add_argument("--batch", type=int, default=None)
    a = ap.parse_args()
    report(run_steps(a.workload, a.steps, a.batch))


if __name__ == "__main__":
    main()

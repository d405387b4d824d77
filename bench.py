#!/usr/bin/env python
"""Decode-step benchmark of the KV-cache hot path (append + GQA decode attention).

Workload (the batched KV-cached decode microbench): B=256 sequences per GPU,
cached lengths uniform in [1, 511] (seeded), 4 query / 2 KV heads, head_dim
64, f32 KV, 16-token paged blocks handed out from a shuffled free list, 8
layers. One step = one decode token for every sequence through all 8 layers:
`slm_batch_begin`, `slm_batch_decode_layers` over the 8 layers (RoPE on Q and
K, paged append, split-K attention over the grown cache; one launch runs all
8, since every layer's inputs are given), `slm_batch_submit`. The same step
with one `slm_batch_decode_layer` launch per layer, as a model step issues
them, is timed beside it ("one_layer_launches"). After each
step the sequences return to their drawn lengths (host bookkeeping only), so
every step does the same work. One step reads ~544 MB of K/V, far more than
the 126 MB L2, so no flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload microbench|gqa-bf16|model|prefix|serve|gqa-model]

Multi-GPU (torchrun, one process per GPU): every rank runs its own 256
sequences (weak scaling, no collective on the data path); the timed region is
bracketed by barriers and the slowest rank's time is reported.

The default run (no --workload) then runs the benchmark's other
configurations, each in a process of its own per GPU, and attaches their
result lines under "configs": the 8M model end to end (batch 1, 64-token
prompt, 448 greedy steps), prefix reuse (64 requests sharing a 384-token
prefix, 96 greedy steps), continuous batching (4096 Poisson requests over the
GPUs) and the scaled GQA model (16 sequences of 1-8k tokens per GPU, 256
greedy steps). Each line has its own value, e2e, and at one GPU its CPU
baseline and greedy-token parity against the oracle.

`--impl reference` times the reference's CPU path for the same workload: the
oracle restatement of rust/engine (the Rust engine cannot be built here), all
host threads, one sampled batch of sequences per step.
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "small-lm-rs_b200"))

METRIC = "decode tok/s and KV-attn HBM GB/s (% of peak) at 1/2/4/8 B200 vs host CPU"
BLOCK = 16
APPEND_REPS = 5
REF_SAMPLE = 32  # sequences per reference-arm step
# Steps the headline loop keeps submitted ahead of the GPU (the library's
# limit on unresolved batches): the host plans and queues step i + DEPTH - 1
# while the GPU runs step i, so a stall of the host thread shorter than that
# many steps leaves the GPU busy.
DEPTH = 8

# Per-GPU workloads. "microbench" is the isolated decode-attention + append
# microbench (the headline); "gqa-bf16" is the scaled GQA shape (Hq 32 / Hkv 8,
# bf16 KV, 8k context; 128 sequences over 8 GPUs = 16 per GPU; cached lengths
# stop at 8191 so the appended token fits the 8192-token context).
WORKLOADS = {
    "microbench": dict(B=256, LEN_LO=1, LEN_HI=511, LAYERS=8, HQ=4, HKV=2, D=64, CTX=512,
                       BF16=False),
    "gqa-bf16": dict(B=16, LEN_LO=1024, LEN_HI=8191, LAYERS=8, HQ=32, HKV=8, D=64, CTX=8192,
                     BF16=True),
    # continuous batching: the request trace below through the scheduler
    "serve": dict(B=512, LEN_LO=8, LEN_HI=256, LAYERS=8, HQ=4, HKV=2, D=64, CTX=512, BF16=False),
    # prefix reuse: 64 requests, a shared 384-token prefix + 32 own tokens each
    "prefix": dict(B=64, LEN_LO=384, LEN_HI=32, LAYERS=8, HQ=4, HKV=2, D=64, CTX=512, BF16=False),
    # the 8M model end to end: batch 1, a 64-token prompt, 448 greedy decode steps
    "model": dict(B=1, LEN_LO=64, LEN_HI=448, LAYERS=8, HQ=4, HKV=2, D=64, CTX=512, BF16=False),
    # the scaled GQA model end to end: 16 sequences a GPU, prompts of
    # U[1024, 8192 - 256] random tokens, then 256 greedy decode steps
    "gqa-model": dict(B=16, LEN_LO=1024, LEN_HI=8192 - 256, LAYERS=8, HQ=32, HKV=8, D=64,
                      CTX=8192, BF16=True),
}
# the 8M model (artifacts/small-lm-8m/config.json): vocab 8192, hidden 256,
# SiTU-GLU FFN 704, RMSNorm eps 1e-5, SiTU betas 4 / 25, tied embeddings
MODEL_VOCAB, MODEL_INTER = 8192, 704
# the scaled GQA model: hidden 2048 (32 x 64), FFN 5632, same vocabulary
GQA_MODEL_INTER, GQA_MODEL_STEPS = 5632, 256
PREFIX_DECODE_STEPS = 96
# "serve": 4096 requests in total (shared by the ranks), Poisson arrivals at
# SERVE_RATE requests/s (seeded), prompts U[8,256], outputs U[16,256], at
# most 512 running per GPU, the 8M model's KV shape.
SERVE_REQUESTS, SERVE_RATE, SERVE_OUT_LO, SERVE_OUT_HI = 4096, 50000.0, 16, 256
SERVE_PREFILL_TOKENS = 1024  # prompt tokens a step: the exact-order projections' row limit


def select_workload(name: str, batch: int | None = None) -> None:
    global B, LEN_LO, LEN_HI, LAYERS, HQ, HKV, D, CTX, BF16, S_KV, WORKLOAD, WORKLOAD_NAME
    w = WORKLOADS[name]
    B, LEN_LO, LEN_HI = (batch or w["B"]), w["LEN_LO"], w["LEN_HI"]
    LAYERS, HQ, HKV, D, CTX, BF16 = w["LAYERS"], w["HQ"], w["HKV"], w["D"], w["CTX"], w["BF16"]
    S_KV = 2 if BF16 else 4
    WORKLOAD_NAME = name
    kind = "batched decode microbench" if name == "microbench" else "scaled GQA decode"
    WORKLOAD = (f"{kind}: B={B} per GPU, cached lengths U[{LEN_LO},{LEN_HI}], Hq={HQ}, "
                f"Hkv={HKV}, d={D}, {'bf16' if BF16 else 'f32'} KV, {BLOCK}-token paged blocks, "
                f"shuffled block table, {LAYERS} layers, 1 appended token per sequence per step")


select_workload("microbench")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="headline workload only: skip the other configurations' runs")
    ap.add_argument("--pg-timeout", type=int, default=300,
                    help="process-group timeout in seconds (multi-GPU)")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="microbench")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per GPU instead of the workload's (smaller cases for profiling)")
    ap.add_argument("--exact-rows", type=int, default=None,
                    help="model workloads: steps of up to this many token rows project in the "
                         "reference's accumulation order, larger ones on tensor-core GEMMs "
                         "(default: the 8M model at batch 1: 1024; serve and prefix: 1; the scaled "
                         "GQA model: 0)")
    args = ap.parse_args()
    select_workload(args.workload, args.batch)
    return args


def dist_env():
    """(rank, world size, local rank) from the torchrun environment."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init_dist(world: int, dev, seconds: int) -> None:
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=seconds),
                                device_id=dev)


def close_dist(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def pin_rank_cores(local: int, local_world: int) -> list[int]:
    """Binds this rank's process to its own share of the host cores it may
    use (rank r of n takes the r-th of n equal slices), so that the ranks'
    host loops do not migrate across one another's cores. Returns them."""
    try:
        cores = sorted(os.sched_getaffinity(0))
    except AttributeError:
        return []
    if local_world <= 1 or len(cores) < local_world:
        return cores
    k = len(cores) // local_world
    mine = cores[local * k:(local + 1) * k]
    os.sched_setaffinity(0, mine)
    return mine


def host_threads() -> int:
    """Host cores this process may run on (torchrun sets OMP_NUM_THREADS=1,
    so the oracle is always given this count explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def sum_over_ranks(value: float, device) -> float:
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t)
    return float(t.item())


# The other configurations of the benchmark, each run by `python bench.py`
# (no --workload) in a process of its own after the headline microbench, on
# the same GPUs, and attached to the headline line under "configs":
#   model     the 8M model end to end, batch 1: 64-token prompt, 448 greedy
#             steps (each GPU its own replica: weak scaling)
#   prefix    prefix reuse: 64 requests sharing a 384-token prefix + 32 own
#             tokens, 96 greedy steps (64 requests per GPU: weak scaling)
#   serve     continuous batching of 4096 Poisson requests over the GPUs
#             (strong scaling)
#   gqa_model the scaled GQA model, 16 sequences per GPU, 256 greedy steps
CONFIG_RUNS = [
    ("model", "model", ["--steps", "448"]),
    ("prefix", "prefix", []),
    ("serve", "serve", []),
    ("gqa_model", "gqa-model", ["--steps", "256"]),
]
CONFIGS_BUDGET_S = 700.0  # all configuration runs of one bench.py invocation


def last_json_line(text: str):
    for line in reversed(text.splitlines()):
        line = line.strip()
        if line.startswith("{"):
            try:
                return json.loads(line)
            except ValueError:
                continue
    return None


def run_configs(args, world: int) -> dict:
    """Runs CONFIG_RUNS one after another, each as a child process per rank
    (a fresh CUDA context and, with several GPUs, a process group of its own
    on its own port). Returns rank 0's result line of each, or its error."""
    env = dict(os.environ)
    # the children host their own rendezvous store (rank 0 child)
    env.pop("TORCHELASTIC_USE_AGENT_STORE", None)
    base_port = int(env.get("MASTER_PORT", "29500"))
    out, t_begin = {}, time.time()
    for k, (key, workload, extra) in enumerate(CONFIG_RUNS):
        left = CONFIGS_BUDGET_S - (time.time() - t_begin)
        if left < 30:
            out[key] = {"error": "skipped: the configurations' time budget is spent"}
            continue
        env["MASTER_PORT"] = str(base_port + 1 + k)
        cmd = [sys.executable, str(ROOT / "bench.py"), "--workload", workload, "--warmup", "3",
               "--gpus", str(world), "--seed", str(args.seed), "--pg-timeout", "180", *extra]
        if args.no_cpu_baseline:
            cmd.append("--no-cpu-baseline")
        t0 = time.time()
        try:
            p = subprocess.run(cmd, env=env, capture_output=True, text=True,
                               timeout=min(400.0, left))
            line = last_json_line(p.stdout)
            if p.returncode != 0 or (line is None and int(env.get("RANK", "0")) == 0):
                tail = (p.stderr or p.stdout or "").strip().splitlines()[-3:]
                line = {"error": f"exit {p.returncode}: " + " | ".join(tail)}
        except subprocess.TimeoutExpired:
            line = {"error": f"timed out after {min(400.0, left):.0f} s"}
        if line is not None:
            line["wall_s"] = round(time.time() - t0, 1)
        out[key] = line
    return out


def draw_lengths(seed: int):
    import numpy as np

    rng = np.random.default_rng(seed)
    return rng.integers(LEN_LO, LEN_HI + 1, size=B).astype(np.int64)


def algorithmic_bytes(lengths, s_kv: int | None = None) -> int:
    """Bytes one decode launch must move for the batch (one layer):
    K+V over L_i+1 positions, Q read + O write, new K/V read, the append
    write, and the block-table entries."""
    s_kv = S_KV if s_kv is None else s_kv
    total = 0
    for L in lengths:
        Lp = int(L) + 1
        total += (2 * HKV * D * s_kv * Lp + 2 * HQ * D * 4 + 2 * HKV * D * 4 + 2 * HKV * D * s_kv
                  + 4 * math.ceil(Lp / BLOCK))
    return total


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def ncu_traffic_per_launch():
    """(dram bytes read + written per decode launch, where they come from)
    from the committed ncu summary of this workload's decode kernel: a figure
    of one capture of the kernel version the summary names, not a counter of
    this run. (None, None) without one."""
    name = "microbench" if WORKLOAD_NAME == "microbench" else "gqa_bf16"
    p = ROOT / "profiles" / f"decode_kernel_{name}.md"
    if not p.exists():
        return None, None
    traffic, version = None, None
    for line in p.read_text().splitlines():
        key, _, val = line.strip().partition(":")
        if key == "traffic_bytes_per_launch":
            try:
                traffic = int(float(val.strip()))
            except ValueError:
                return None, None
        elif key == "traffic_kernel_version":
            version = val.strip()
    src = f"profiles/{p.name}" + (f", kernel version {version}" if version else "")
    return traffic, src


class ClockSampler:
    """nvidia-smi sampling of SM clock / throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.2)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[4:]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        busy = [r for r in rows if r[2] > 200.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in busy for i, v in enumerate(r[3][1:5])
                          if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in busy),
                "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(busy), "power_w_max": max(r[2] for r in rows)}


def cpu_baseline(lengths, seed: int, threads: int, budget_s: float = 8.0):
    """The oracle (a restatement of the reference's decode path) on a bounded
    sample: REF_SAMPLE sequences, all layers, repeated until ~budget_s."""
    import numpy as np

    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O

    rng = np.random.default_rng(seed + 99)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    sample = [int(x) for x in lengths[:REF_SAMPLE]]
    caches = [O.DenseCache(LAYERS, CTX, HKV, D, quantize_bf16=BF16) for _ in sample]
    for c, L in zip(caches, sample):
        for layer in range(LAYERS):
            k = rng.standard_normal((L, HKV, D)).astype(np.float32)
            c.append_layer(layer, k, k, L)
    n = len(sample)
    q = rng.standard_normal((LAYERS, n, HQ, D)).astype(np.float32)
    kv = rng.standard_normal((LAYERS, n, HKV, D)).astype(np.float32)

    def one_step():
        for layer in range(LAYERS):
            O.forward_cached_attention_batch(caches, layer, q[layer], kv[layer], kv[layer], HQ,
                                             inv, threads=threads)
        for c, L in zip(caches, sample):
            c.truncate_all(L)

    one_step()
    reps, t0 = 0, time.perf_counter()
    while True:
        one_step()
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return n * reps / el, reps, el


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O

    lengths = draw_lengths(args.seed)
    threads = host_threads()
    rng = np.random.default_rng(args.seed + 7)
    inv = O.rope_inverse_frequencies(D, 10000.0)
    sample = [int(x) for x in lengths[:REF_SAMPLE]]
    caches = [O.DenseCache(LAYERS, CTX, HKV, D, quantize_bf16=BF16) for _ in sample]
    for c, L in zip(caches, sample):
        for layer in range(LAYERS):
            k = rng.standard_normal((L, HKV, D)).astype(np.float32)
            _, kr = O.apply_rotary_with_offset(k.copy(), k, HKV, HKV, D, inv, 0)
            c.append_layer(layer, kr, k, L)
    n = len(sample)
    q = rng.standard_normal((LAYERS, n, HQ, D)).astype(np.float32)
    kv = rng.standard_normal((LAYERS, n, HKV, D)).astype(np.float32)

    def step():
        for layer in range(LAYERS):
            O.forward_cached_attention_batch(caches, layer, q[layer], kv[layer], kv[layer], HQ,
                                             inv, threads=threads)
        for c, L in zip(caches, sample):
            c.truncate_all(L)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    value = n * args.steps / el
    sample_desc = (f"{n} of the {B} seeded sequences per step (lengths {min(sample)}..{max(sample)}),"
                   f" all {LAYERS} layers, oracle restatement of rust/engine "
                   "(attention.rs:794-816 per sequence), OpenMP over sequences")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "reference_sample_sequences": n},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sample_desc},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    import slmkv
    from slmkv.shard import max_over_ranks

    rank, world, local = dist_env()
    pinned = pin_rank_cores(local, int(os.environ.get("LOCAL_WORLD_SIZE", str(world))))
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    init_dist(world, dev, args.pg_timeout)

    def barrier():
        if world > 1:
            dist.barrier()

    seed = args.seed + 1000 * rank
    lengths = draw_lengths(seed)
    need_blocks = int(sum(math.ceil((int(L) + 1) / BLOCK) for L in lengths))
    pool = slmkv.KvPool(num_layers=LAYERS, num_query_heads=HQ, num_key_value_heads=HKV,
                        head_dimension=D, context_length=CTX, rope_theta=10000.0,
                        num_blocks=need_blocks + B + 64, max_sequences=B,
                        kv_dtype=slmkv.KV_BF16 if BF16 else slmkv.KV_F32, device=local)
    pool.shuffle(seed + 1)
    caches = [pool.allocate_kv_cache(CTX) for _ in range(B)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed + 2)
    total = int(lengths.sum())
    hist_k = [torch.randn((total, HKV, D), generator=gen, device=dev) for _ in range(LAYERS)]
    hist_v = [torch.randn((total, HKV, D), generator=gen, device=dev) for _ in range(LAYERS)]
    counts = [int(x) for x in lengths]

    def append_history(b):
        for layer in range(LAYERS):
            b.append_layer(layer, hist_k[layer], hist_v[layer], rotate_keys=True)

    # Append kernel (RoPE on K + paged scatter of the whole history, one
    # launch per layer): timed over rolled-back repeats of the history
    # prefill, 8 launches each, then the history is appended for real.
    a_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(APPEND_REPS)]
    # bf16 pools: the prompt prefill's attention (layer 0, every sequence's
    # whole prompt, causal) runs on the tensor cores; timed in the same repeats.
    p_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(APPEND_REPS)] if BF16 else []
    if BF16:
        pq = torch.randn((total, HQ, D), generator=gen, device=dev)
        pout = torch.empty_like(pq)
    for r in range(3 + APPEND_REPS):
        b = pool.begin(caches, counts)
        if r >= 3:
            a_ev[r - 3][0].record(torch.cuda.current_stream())
        append_history(b)
        if r >= 3:
            a_ev[r - 3][1].record(torch.cuda.current_stream())
        if BF16:
            if r >= 3:
                p_ev[r - 3][0].record(torch.cuda.current_stream())
            b.prefill_attention(0, pq, pout, rotate_query=True)
            if r >= 3:
                p_ev[r - 3][1].record(torch.cuda.current_stream())
        b.rollback()
    torch.cuda.synchronize()
    append_ms = sum(x.elapsed_time(y) for x, y in a_ev) / (APPEND_REPS * LAYERS)
    prefill_ms = (sum(x.elapsed_time(y) for x, y in p_ev) / APPEND_REPS) if BF16 else None
    if BF16:
        del pq, pout
    with pool.begin(caches, counts) as b:
        append_history(b)
    del hist_k, hist_v
    torch.cuda.synchronize()
    q = torch.randn((LAYERS, B, HQ, D), generator=gen, device=dev)
    kn = torch.randn((LAYERS, B, HKV, D), generator=gen, device=dev)
    vn = torch.randn((LAYERS, B, HKV, D), generator=gen, device=dev)
    out = torch.empty((LAYERS, B, HQ, D), device=dev)
    base = [int(x) for x in lengths]
    stream = torch.cuda.current_stream()
    plan = pool.step_plan(caches, 1)
    base_arr = plan.lengths(base)
    ptrs = [(q[l].data_ptr(), kn[l].data_ptr(), vn[l].data_ptr(), out[l].data_ptr())
            for l in range(LAYERS)]
    io = slmkv.layer_io_array(ptrs)
    # Decode-kernel timing, live in every timed step: a step's layers go out
    # as one launch (slm_batch_decode_layers) and a CUDA event records its
    # completion; the host queues steps ahead of the GPU, so the interval
    # between consecutive steps' completions is the launch's duration back to
    # back (each launch's prologue overlaps the previous one's tail).
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]

    # Steps are pipelined (slm_batch_submit / slm_batch_wait): a step is
    # submitted without waiting for the GPU, the next one is planned and
    # queued while it runs, and its statuses are collected one step later.
    # Every step's statuses are checked.
    inflight = []

    def collect(keep):
        while len(inflight) > keep:
            st = inflight.pop(0).wait()
            if any(st):
                raise RuntimeError(f"decode step failed: {st}")

    host_s = [0.0, 0.0]  # seconds in begin..submit, and waiting in collect

    def step(timed_index=None, layer_io=io):
        t0 = time.perf_counter()
        batch = plan.begin()
        batch.decode_layers_array(0, LAYERS, layer_io)
        if timed_index is not None:
            ev[timed_index].record(stream)
        inflight.append(batch.submit())
        t1 = time.perf_counter()
        collect(DEPTH - 1)
        plan.truncate_all(base_arr)
        if timed_index is not None:
            host_s[0] += t1 - t0
            host_s[1] += time.perf_counter() - t1

    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    for _ in range(max(args.warmup, 3)):
        step()
    collect(0)
    torch.cuda.synchronize()
    barrier()
    launches0 = pool.launch_count()
    t_start = torch.cuda.Event(enable_timing=True)
    t_stop = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        step(i)
    t_stop.record(stream)
    collect(0)
    torch.cuda.synchronize()
    barrier()
    launches = pool.launch_count() - launches0
    clocks = sampler.stop() if sampler else None
    ms = t_start.elapsed_time(t_stop)
    kern_avg_ms = ev[0].elapsed_time(ev[-1]) / max(1, args.steps - 1)

    # The same step with one launch per layer (slm_batch_decode_layer), as a
    # model step issues them between its projections: completion of layer 0's
    # and of the last layer's kernel, interval / (LAYERS - 1).
    chain_steps = min(args.steps, 50)
    cev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(chain_steps)]
    for i in range(3 + chain_steps):
        batch = plan.begin()
        for layer in range(LAYERS):
            batch.decode_layer_ptr(layer, *ptrs[layer])
            if i >= 3 and layer in (0, LAYERS - 1):
                cev[i - 3][0 if layer == 0 else 1].record(stream)
        inflight.append(batch.submit())
        collect(DEPTH - 1)
        plan.truncate_all(base_arr)
    collect(0)
    torch.cuda.synchronize()
    chain_ms = sum(a.elapsed_time(b) for a, b in cev) / (chain_steps * (LAYERS - 1))
    # every rank's own step time and host time per step, for the line
    mine = torch.tensor([ms / args.steps, kern_avg_ms, host_s[0] / args.steps * 1e3,
                         host_s[1] / args.steps * 1e3], dtype=torch.float64, device=dev)
    per_rank = [mine]
    if world > 1:
        per_rank = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(per_rank, mine)
    per_rank = [[round(float(x), 4) for x in t.tolist()] for t in per_rank]
    ms, kern_avg_ms, chain_ms = max_over_ranks([ms, kern_avg_ms, chain_ms], device=dev)

    # End to end through the public API with host buffers: every step hands
    # slm_batch_decode_layers_host its inputs in pinned host memory (Q, new K,
    # new V of every layer) and a pinned output buffer; the library copies
    # them in on its own stream, runs the step, and copies the outputs back
    # before the step's statuses, so a step is complete on the host when its
    # wait returns. DEPTH steps are in flight, each with its own output buffer.
    # (one pinned block: Q, then K, then V, so the library copies it in at once)
    h_in = torch.cat([q.reshape(-1), kn.reshape(-1), vn.reshape(-1)]).cpu().pin_memory()
    h_q = h_in[:q.numel()].view_as(q)
    h_k = h_in[q.numel():q.numel() + kn.numel()].view_as(kn)
    h_v = h_in[q.numel() + kn.numel():].view_as(vn)
    ho_ = [torch.empty_like(out, device="cpu").pin_memory() for _ in range(DEPTH)]
    hin = [C.c_void_p(t.data_ptr()) for t in (h_q, h_k, h_v)]
    hout = [C.c_void_p(t.data_ptr()) for t in ho_]
    e2e_i = [0]

    def e2e_step():
        j = e2e_i[0] % DEPTH
        e2e_i[0] += 1
        batch = plan.begin()
        batch.decode_layers_host_ptr(0, LAYERS, *hin, hout[j])
        inflight.append(batch.submit())
        collect(DEPTH - 1)
        plan.truncate_all(base_arr)

    for _ in range(3):
        e2e_step()
    collect(0)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    collect(0)  # every step's outputs are on the host
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    (e2e_ms,) = max_over_ranks([e2e_ms], device=dev)
    # the link's own rates for a step's bytes, copied alone (CUDA events)
    dq_, do_ = torch.empty_like(q), torch.empty_like(out)
    ho_probe = torch.empty_like(out, device="cpu").pin_memory()
    pe = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    pe[0].record(stream)
    for _ in range(5):
        dq_.copy_(h_q, non_blocking=True)
    pe[1].record(stream)
    for _ in range(5):
        ho_probe.copy_(do_, non_blocking=True)
    pe[2].record(stream)
    torch.cuda.synchronize()
    h2d_gbs = 5 * q.numel() * 4 / (pe[0].elapsed_time(pe[1]) / 1e3) / 1e9
    d2h_gbs = 5 * out.numel() * 4 / (pe[1].elapsed_time(pe[2]) / 1e3) / 1e9
    ref_out = out.cpu()
    if not all(torch.equal(h, ref_out) for h in ho_[:min(DEPTH, e2e_i[0])]):
        raise RuntimeError("end-to-end outputs differ from the device-resident run")

    append_bytes = total * HKV * D * (4 + 4 + 2 * S_KV)  # K, V in (f32) and out (pool type)
    (append_ms,) = max_over_ranks([append_ms], device=dev)
    if BF16:
        (prefill_ms,) = max_over_ranks([prefill_ms], device=dev)
        # causal QK^T and PV: 2 flops per multiply-add, d per score / output
        prefill_flops = sum(int(L) * (int(L) + 1) // 2 for L in lengths) * HQ * 4 * D
    tokens = B * world * args.steps
    value = tokens / (ms / 1e3)
    e2e_value = tokens / (e2e_ms / 1e3)
    peaks, peak_kind = measured_peaks()
    alg = algorithmic_bytes(lengths)  # one layer
    achieved = LAYERS * alg / (kern_avg_ms / 1e3) / 1e9  # a launch runs every layer
    chain_achieved = alg / (chain_ms / 1e3) / 1e9
    traffic, traffic_src = ncu_traffic_per_launch()
    result = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "name": WORKLOAD_NAME, "batch_per_gpu": B,
                   "layers": LAYERS, "kv_dtype": "bf16" if BF16 else "f32",
                   "l2": f"inputs larger than L2 ({LAYERS * alg / 1e6:.0f} MB of K/V per step)",
                   "seed": args.seed},
        "kv_attn_hbm_gbs": achieved,
        "kv_attn_hbm_frac": achieved / peaks["hbm_gbs"],
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     "traffic": traffic, "traffic_source": traffic_src, "peak_source": peak_kind,
                     "kernel": ("decode_stream_kernel (fused RoPE + paged append + split-K GQA "
                                f"attention), all {LAYERS} layers of a step in one launch "
                                "(slm_batch_decode_layers)"),
                     "algorithmic_bytes_per_launch": LAYERS * alg, "avg_launch_ms": kern_avg_ms,
                     "timing": ("CUDA events at each timed step's launch completion; mean "
                                "interval between consecutive steps' completions")},
        "one_layer_launches": {
            "what": ("the same step as one slm_batch_decode_layer launch per layer, as a model "
                     "step issues them between its projections"),
            "avg_launch_ms": chain_ms, "algorithmic_bytes_per_launch": alg,
            "achieved": chain_achieved, "unit": "GB/s", "frac": chain_achieved / peaks["hbm_gbs"],
            "timing": (f"completion of layer 0's to layer {LAYERS - 1}'s kernel, "
                       f"/ {LAYERS - 1}, over {chain_steps} steps")},
        "e2e": {"value": e2e_value, "unit": "tok/s",
                "h2d_bytes_per_step": int(q.numel() + kn.numel() + vn.numel()) * 4,
                "d2h_bytes_per_step": int(out.numel()) * 4,
                "api": ("slm_batch_decode_layers_host from pinned host buffers: the library "
                        "copies the inputs in and the outputs out on its own streams, "
                        f"{DEPTH} steps in flight"),
                "ms_per_step": e2e_ms / args.steps,
                "timing": ("CUDA events around the steps; the end event is recorded after "
                           "the host has every step's outputs"),
                "link_h2d_gbs": h2d_gbs, "link_d2h_gbs": d2h_gbs,
                "link": "a step's Q rows alone host to device and its outputs alone back, "
                        "5 copies each, CUDA events"},
        "append_kernel": {"achieved": append_bytes / (append_ms / 1e3) / 1e9, "unit": "GB/s",
                          "frac": append_bytes / (append_ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                          "avg_launch_ms": append_ms, "bytes_per_launch": append_bytes,
                          "workload": f"history prefill: {total} tokens x {HKV} KV heads, "
                                      f"RoPE on K, f32 in, {'bf16' if BF16 else 'f32'} pool"},
        **({"prefill_kernel": {
            "bound": "tensor", "unit": "TFLOP/s",
            "achieved": prefill_flops / (prefill_ms / 1e3) / 1e12,
            "peak": peaks.get("bf16_tflops", 1590.0),
            "frac": prefill_flops / (prefill_ms / 1e3) / 1e12 / peaks.get("bf16_tflops", 1590.0),
            "avg_launch_ms": prefill_ms, "flops_per_launch": prefill_flops,
            "workload": (f"prompt prefill attention, one layer: {B} prompts of the drawn lengths "
                         f"({total} tokens), Hq={HQ}, Hkv={HKV}, causal, bf16 KV, tcgen05")}}
           if BF16 else {}),
        "gpu_launches": launches,
        "kernel_timing": ("CUDA events at the completion of every timed step's decode launch "
                          "(all layers); mean interval between consecutive completions"),
        "per_rank": {"fields": ["ms_per_step", "decode_kernel_ms", "host_submit_ms_per_step",
                                "host_wait_ms_per_step"], "values": per_rank,
                     "host_cores_per_rank": len(pinned)},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, str(ROOT / "oracle"))
        cv, reps, el = cpu_baseline(lengths, args.seed, threads=1)
        result["cpu_baseline"] = {
            "value": cv, "unit": "tok/s", "cores": 1, "kind": "port",
            "sample": (f"{min(REF_SAMPLE, B)} of the {B} seeded sequences x {LAYERS} layers per step, "
                       f"{reps} steps in {el:.1f} s, single thread (the reference's decode "
                       "attention is serial per sequence)")}
    pool.close()
    close_dist(world)
    return result if rank == 0 else None


def serve_trace(seed: int):
    """(arrival s, prompt length, output length) of every request, seeded."""
    import numpy as np

    rng = np.random.default_rng(seed + 4242)
    arrivals = np.cumsum(rng.exponential(1.0 / SERVE_RATE, size=SERVE_REQUESTS))
    prompts = rng.integers(LEN_LO, LEN_HI + 1, size=SERVE_REQUESTS)
    outputs = rng.integers(SERVE_OUT_LO, SERVE_OUT_HI + 1, size=SERVE_REQUESTS)
    return arrivals, prompts, outputs


def oracle_generate_check(tensors, prompt, generated, threads):
    """The oracle model (model.rs:297-397 restated) prefills `prompt` and then
    decodes the GPU's `generated` tokens one by one (the reference has no
    prefix cache or batching: every request alone, from scratch); returns
    (every greedy choice equal to the GPU's next token, seconds)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O

    cfg = dict(vocab_size=MODEL_VOCAB, hidden_size=HQ * D, intermediate_size=MODEL_INTER,
               num_layers=LAYERS, num_query_heads=HQ, num_key_value_heads=HKV, head_dimension=D,
               rms_norm_epsilon=1e-5, rope_theta=10000.0, situ_beta_gate=4.0, situ_beta_up=25.0)
    m = O.Model(cfg, tensors)
    cache = m.new_cache(CTX)
    generated = [int(t) for t in generated]
    t0 = time.perf_counter()
    ok = O.argmax_finite(m.prefill(cache, [int(t) for t in prompt], threads)[-1]) == generated[0]
    for j in range(len(generated) - 1):
        ok = ok and O.argmax_finite(m.decode(cache, generated[j], threads)) == generated[j + 1]
    return bool(ok), time.perf_counter() - t0


def run_serve(args):
    """Continuous batching of the request trace on the 8M model: every step the
    scheduler plans a decode batch and a prefill batch (prompt chunks within a
    token budget); the decode batch runs slm_model_decode, the prefill batch
    slm_model_prefill, and their statuses are committed. Each request's tokens
    (its random prompt, then the greedy tokens the model chose) live in a
    device history indexed by request and position: a step gathers its input
    tokens from it and writes the chosen tokens back, so a preempted request
    recomputes from its own tokens. Requests arrive on the host clock.
    Throughput = output tokens of all ranks / slowest rank's device time.
    Every step stays on the exact-order projections (steps of at most 1024
    rows: a 512-row decode batch and a 1024-token prefill budget). The e2e
    run copies each request's prompt in from pinned host memory when it
    arrives and each step's chosen tokens out. At one GPU the oracle replays
    sampled requests from their prompts: every greedy token must agree."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import slmkv
    from slmkv.shard import max_over_ranks, rank_share

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    init_dist(world, dev, args.pg_timeout)
    arrivals, prompts, outputs = serve_trace(args.seed)
    mine = rank_share([int(p + o) for p, o in zip(prompts, outputs)], world, rank)
    pool = slmkv.KvPool(num_layers=LAYERS, num_query_heads=HQ, num_key_value_heads=HKV,
                        head_dimension=D, context_length=CTX, num_blocks=B * (CTX // BLOCK),
                        max_sequences=B, device=local)
    pool.shuffle(args.seed + 1)
    tensors = model_tensors(args.seed)
    model = slmkv.Model(pool, vocab_size=MODEL_VOCAB, intermediate_size=MODEL_INTER,
                        tensors=tensors)
    exact_rows = 1024 if args.exact_rows is None else args.exact_rows
    model.set_exact_rows(exact_rows)
    # token history: row per request of this rank, prompt tokens first
    row_of = {rid: k for k, rid in enumerate(mine)}
    W = CTX + 1
    rng = np.random.default_rng(args.seed + 11)
    h_hist = np.zeros((max(1, len(mine)), W), np.int32)
    for rid, k in row_of.items():
        h_hist[k, :prompts[rid]] = rng.integers(0, MODEL_VOCAB, size=int(prompts[rid]))
    p_hist = torch.from_numpy(h_hist).pin_memory()  # the prompts, on the host
    hist = torch.zeros(h_hist.size, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    ones = slmkv._i32_array([1] * B)
    # staging for the per-step gather / scatter indices (pinned, copied async)
    h_idx = torch.zeros(B + SERVE_PREFILL_TOKENS + B, dtype=torch.int64).pin_memory()
    d_idx = torch.zeros_like(h_idx, device=dev)
    sel_h = torch.zeros(B, dtype=torch.int64).pin_memory()  # prefill rows whose first token is due
    sel_d = torch.zeros_like(sel_h, device=dev)
    row_arr = np.full(len(prompts), -1, np.int64)  # request id -> history row
    for rid, k in row_of.items():
        row_arr[rid] = k
    nxt_dec = torch.zeros(B, dtype=torch.int32, device=dev)
    nxt_pre = torch.zeros(B, dtype=torch.int32, device=dev)
    h_out = torch.zeros(2 * B, dtype=torch.int32).pin_memory()  # a step's chosen tokens
    copied = {"h2d": 0, "d2h": 0}

    def run_step(sched, first_done, e2e):
        # the decode batch is submitted and the prefill batch queued behind it:
        # one wait per step
        nd, npf = sched.plan()
        dreq, dpos, preq, ppos = sched.plan_request_arrays()
        counts = np.ctypeslib.as_array(sched._pcnt)[:npf]
        rows = int(counts.sum())
        # indices: decode inputs [0, nd), prefill inputs [nd, nd + rows),
        # first-token writes after them
        hv = h_idx.numpy()
        hv[:nd] = row_arr[dreq] * W + dpos
        at = nd
        firsts = []
        for i in range(npf):
            rid, pos, c = int(preq[i]), int(ppos[i]), int(counts[i])
            base = int(row_arr[rid]) * W + pos
            hv[at:at + c] = np.arange(base, base + c)
            at += c
            if pos + c == prompts[rid] and rid not in first_done:
                firsts.append((i, base + c))
                first_done.add(rid)
        for j, (i, dst) in enumerate(firsts):
            hv[at + j] = dst
            sel_h.numpy()[j] = i
        n_idx = at + len(firsts)
        if n_idx:
            d_idx[:n_idx].copy_(h_idx[:n_idx], non_blocking=True)
        if firsts:
            sel_d[:len(firsts)].copy_(sel_h[:len(firsts)], non_blocking=True)
        dst = pst = None
        dec = None
        if nd:
            dec = slmkv.Batch.for_sequences(pool, nd, sched._dseq, ones, stream)
            model.decode(dec, hist.index_select(0, d_idx[:nd]).to(torch.int32), None, nxt_dec[:nd])
            hist.index_copy_(0, d_idx[:nd] + 1, nxt_dec[:nd])
            if e2e:
                h_out[:nd].copy_(nxt_dec[:nd], non_blocking=True)
                copied["d2h"] += 4 * nd
            dec.submit()
        if npf:
            b = slmkv.Batch.for_sequences(pool, npf, sched._pseq, sched._pcnt, stream)
            model.prefill(b, hist.index_select(0, d_idx[nd:nd + rows]).to(torch.int32), None,
                          nxt_pre[:npf])
            if firsts:
                firsts_tok = nxt_pre.index_select(0, sel_d[:len(firsts)])
                hist.index_copy_(0, d_idx[nd + rows:n_idx], firsts_tok)
                if e2e:
                    h_out[B:B + len(firsts)].copy_(firsts_tok, non_blocking=True)
                    copied["d2h"] += 4 * len(firsts)
            pst = b.end(raise_on_error=False)
        if dec is not None:
            dst = dec.wait(raise_on_error=False)
        if e2e:
            stream.synchronize()  # the chosen tokens are on the host
        return nd, npf, sched.commit(dst, pst)

    def serve_once(e2e):
        """The whole trace once; returns (device ms, steps, output tokens,
        preemptions, launches)."""
        sched = slmkv.Scheduler(pool, max_running=B, max_prefill_tokens=SERVE_PREFILL_TOKENS)
        first_done = set()
        if not e2e:  # the prompts are resident before the timed region
            hist.copy_(p_hist.view(-1))
        else:
            hist.zero_()
        order = sorted(mine, key=lambda i: arrivals[i])
        l0 = pool.launch_count()
        t_start = torch.cuda.Event(enable_timing=True)
        t_stop = torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t_start.record(stream)
        t0 = time.perf_counter()
        nxt, finished, failed, steps = 0, 0, 0, 0
        while finished < len(order):
            now = time.perf_counter() - t0
            while nxt < len(order) and arrivals[order[nxt]] <= now:
                i = order[nxt]
                if e2e:  # the request's prompt arrives from the host
                    k, P = row_of[i], int(prompts[i])
                    hist[k * W:k * W + P].copy_(p_hist[k, :P], non_blocking=True)
                    copied["h2d"] += 4 * P
                sched.submit(i, int(prompts[i]), int(outputs[i]))
                nxt += 1
            nd, npf, fin = run_step(sched, first_done, e2e)
            steps += 1
            finished += len(fin)
            failed += sum(1 for _, st, _ in fin if st != 0)
            if nd == 0 and npf == 0 and nxt < len(order):
                time.sleep(max(0.0, arrivals[order[nxt]] - (time.perf_counter() - t0)))
        t_stop.record(stream)
        torch.cuda.synchronize()
        if failed:
            raise RuntimeError(f"{failed} requests failed")
        c = sched.counts()
        sched.close()
        return (t_start.elapsed_time(t_stop), steps, c["generated_tokens"], c["preemptions"],
                pool.launch_count() - l0)

    # warm-up on throwaway sequences (both batch kinds at the timed shapes)
    warm = [pool.allocate_kv_cache(CTX) for _ in range(4)]
    wid = torch.ones(SERVE_PREFILL_TOKENS, dtype=torch.int32, device=dev)
    with pool.begin(warm, [SERVE_PREFILL_TOKENS // 4] * 4) as b:
        model.prefill(b, wid)
    with pool.begin(warm, 1) as b:
        model.decode(b, wid[:4])
    for c in warm:
        c.free()
    # and the whole trace once, untimed: its steps take every batch size up to
    # 512 rows, so every kernel variant they select is loaded and configured
    # (first launches of a variant cost milliseconds) before the timed pass
    serve_once(False)

    ms, steps, generated, preemptions, launches = serve_once(False)
    hist_done = hist.view(-1, W).cpu().numpy().copy()
    copied["h2d"] = copied["d2h"] = 0
    e2e_ms, e2e_steps, _, _, _ = serve_once(True)
    if not np.array_equal(hist.view(-1, W).cpu().numpy(), hist_done):
        raise RuntimeError("the e2e run generated other tokens than the device-resident run")
    ms, e2e_ms = max_over_ranks([ms, e2e_ms], device=dev)
    tokens = sum_over_ranks(generated, dev)
    result = {
        "metric": METRIC, "value": tokens / (ms / 1e3), "unit": "tok/s",
        "n_gpus": world, "steps": steps, "warmup": 0, "ms_per_step": ms / max(1, steps),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": (f"continuous batching: {SERVE_REQUESTS} requests shared by the "
                                f"GPUs, Poisson arrivals {SERVE_RATE:.0f}/s, prompts "
                                f"U[{LEN_LO},{LEN_HI}], outputs U[{SERVE_OUT_LO},{SERVE_OUT_HI}], "
                                f"<= {B} running per GPU, {SERVE_PREFILL_TOKENS} prompt tokens "
                                f"per step; the 8M model ({LAYERS} layers, hidden {HQ * D}, FFN "
                                f"{MODEL_INTER}, Hq={HQ}, Hkv={HKV}, d={D}, vocab {MODEL_VOCAB}, "
                                "f32 KV, random N(0, 0.02^2) weights), random prompt ids, "
                                "greedy decoding"),
                   "name": "serve", "requests_per_rank": len(mine), "seed": args.seed,
                   "exact_rows": exact_rows},
        "output_tokens": int(tokens), "preemptions": preemptions,
        "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": copied["h2d"] // max(1, e2e_steps),
                "d2h_bytes_per_step": copied["d2h"] // max(1, e2e_steps),
                "loop": "each request's prompt ids copied in from pinned host memory on "
                        "arrival, each step's chosen tokens copied out and synchronized "
                        "(plus the step's gather indices, as in the device-resident run)"},
        "gpu_launches": launches,
        "projections": ("this library's fused exact-order projection kernels (bf16 operands, "
                        "the reference's fp32 fold order) for every step" if exact_rows >= 1024
                        else f"exact order up to {exact_rows} rows, tensor-core GEMMs beyond "
                             "(outside the fp32 parity bar)"),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # the three cheapest requests of this rank, replayed by the oracle
        sample = sorted(mine, key=lambda i: int(prompts[i] + outputs[i]))[:3]
        ok, secs, toks = True, 0.0, 0
        for rid in sample:
            k, P, Ou = row_of[rid], int(prompts[rid]), int(outputs[rid])
            good, t = oracle_generate_check(tensors, hist_done[k, :P], list(hist_done[k, P:P + Ou]),
                                            host_threads())
            ok, secs, toks = ok and good, secs + t, toks + Ou
        result["parity"] = {"greedy_tokens_match_cpu": ok, "requests_checked": len(sample),
                            "tokens_checked": toks,
                            "oracle": "oracle model replaying each request alone from its prompt"}
        result["cpu_baseline"] = {
            "value": toks / secs, "unit": "tok/s", "cores": host_threads(), "kind": "port",
            "sample": (f"{len(sample)} requests ({toks} output tokens) served one at a time as the "
                       "reference server does (worker.rs:87-98): oracle prefill of the prompt, "
                       "then greedy decode; OpenMP projections, serial attention")}
    if rank == 0:
        print(json.dumps(result), flush=True)
    model.close()
    pool.close()
    close_dist(world)


def run_prefix(args):
    """Prefix reuse on the 8M model: request 0 prefills the shared prefix and
    publishes its full blocks; the other requests attach them through the
    block table and prefill only their own suffix over the attached cache (in
    batches of at most 1024 rows, the exact-order projections' limit); then
    every request decodes PREFIX_DECODE_STEPS greedy tokens in batched steps,
    each step's tokens staying on the device. Each GPU serves its own 64
    requests (weak scaling). Reports the prefill tokens the reuse saved and
    the decode throughput; the e2e run copies the prompts in from pinned host
    memory and every step's chosen tokens out. At one GPU the oracle
    generates two requests alone, from their whole prompts (the reference has
    no prefix cache): every greedy token must agree."""
    import numpy as np
    import torch

    import slmkv
    from slmkv.shard import max_over_ranks

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    init_dist(world, dev, args.pg_timeout)
    prefix_len, suffix_len = LEN_LO, LEN_HI
    rng = np.random.default_rng(args.seed + 77)
    prefix_ids = [int(x) for x in rng.integers(0, MODEL_VOCAB, size=prefix_len)]
    suffix_ids = [[int(x) for x in rng.integers(0, MODEL_VOCAB, size=suffix_len)] for _ in range(B)]
    total_len = prefix_len + suffix_len + PREFIX_DECODE_STEPS
    pool = slmkv.KvPool(num_layers=LAYERS, num_query_heads=HQ, num_key_value_heads=HKV,
                        head_dimension=D, context_length=CTX,
                        num_blocks=B * ((total_len + BLOCK - 1) // BLOCK) + 160, max_sequences=B,
                        device=local)
    pool.shuffle(args.seed + 1)
    tensors = model_tensors(args.seed)
    model = slmkv.Model(pool, vocab_size=MODEL_VOCAB, intermediate_size=MODEL_INTER,
                        tensors=tensors)
    exact_rows = 1024 if args.exact_rows is None else args.exact_rows
    model.set_exact_rows(exact_rows)
    # the other requests' suffixes, in prefill batches of at most 1024 rows
    per_batch = max(1, 1024 // suffix_len)
    groups = [list(range(i, min(B, i + per_batch))) for i in range(1, B, per_batch)]
    stream = torch.cuda.current_stream()
    # all prompt tokens on the host (pinned): prefix, then every suffix
    h_ids = torch.tensor(prefix_ids + [t for sfx in suffix_ids for t in sfx],
                         dtype=torch.int32).pin_memory()
    d_ids = torch.zeros_like(h_ids, device=dev)
    tok = [torch.zeros(B, dtype=torch.int32, device=dev) for _ in range(2)]
    gen = torch.zeros((PREFIX_DECODE_STEPS + 1, B), dtype=torch.int32, device=dev)
    h_gen = torch.zeros(B, dtype=torch.int32).pin_memory()

    def suffix(i):  # request i's suffix tokens in d_ids
        return d_ids[prefix_len + i * suffix_len:prefix_len + (i + 1) * suffix_len]

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def run_once(e2e):
        caches = [pool.allocate_kv_cache(total_len) for _ in range(B)]
        e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        barrier()
        torch.cuda.synchronize()
        e[0].record(stream)
        if e2e:
            d_ids.copy_(h_ids, non_blocking=True)
        # request 0: the prefix, published, then its own suffix
        with pool.begin([caches[0]], [prefix_len]) as b:
            model.prefill(b, d_ids[:prefix_len])
        indexed = caches[0].publish_prefix(prefix_ids)
        with pool.begin([caches[0]], [suffix_len]) as b:
            model.prefill(b, suffix(0), None, tok[0][:1])
        # the others: attach the prefix blocks, prefill only the suffix
        reused = [c.attach_prefix(prefix_ids + suffix_ids[i]) for i, c in enumerate(caches[1:], 1)]
        for g in groups:
            lo, hi = g[0], g[-1] + 1
            with pool.begin(caches[lo:hi], [suffix_len] * len(g)) as b:
                model.prefill(b, d_ids[prefix_len + lo * suffix_len:prefix_len + hi * suffix_len],
                              None, tok[0][lo:hi])
        e[1].record(stream)
        gen[0].copy_(tok[0])
        # batched greedy decode of every request
        plan = pool.step_plan(caches, 1)
        inflight = []
        e[2].record(stream)
        for i in range(PREFIX_DECODE_STEPS):
            b = plan.begin()
            model.decode(b, tok[i % 2], None, tok[(i + 1) % 2])
            if e2e:
                h_gen.copy_(tok[(i + 1) % 2], non_blocking=True)
                if any(b.end(raise_on_error=False)):
                    raise RuntimeError("decode step failed")
                stream.synchronize()
            else:
                gen[i + 1].copy_(tok[(i + 1) % 2])
                inflight.append(b.submit())
                while len(inflight) > 1:
                    if any(inflight.pop(0).wait(raise_on_error=False)):
                        raise RuntimeError("decode step failed")
        e[3].record(stream)
        for b in inflight:
            if any(b.wait(raise_on_error=False)):
                raise RuntimeError("decode step failed")
        torch.cuda.synchronize()
        lengths = [c.sequence_length() for c in caches]
        if lengths != [total_len] * B or any(r != prefix_len for r in reused):
            raise RuntimeError(f"unexpected lengths {set(lengths)} or reuse {set(reused)}")
        for c in caches:  # the prefix index keeps its blocks; a later run attaches to them
            c.free()
        return e[0].elapsed_time(e[1]), e[2].elapsed_time(e[3]), e[0].elapsed_time(e[3]), indexed

    d_ids.copy_(h_ids)
    run_once(False)  # warm-up with the timed shapes
    l0 = pool.launch_count()
    prefill_ms, decode_ms, _, indexed = run_once(False)
    launches = pool.launch_count() - l0
    gen_h = gen.cpu().numpy().T.copy()  # [B, steps + 1]
    _, e2e_decode_ms, _, _ = run_once(True)
    prefill_ms, decode_ms, e2e_decode_ms = max_over_ranks([prefill_ms, decode_ms, e2e_decode_ms],
                                                          device=dev)
    computed = prefix_len + B * suffix_len
    without = B * (prefix_len + suffix_len)
    tokens = world * B * PREFIX_DECODE_STEPS
    result = {
        "metric": METRIC, "value": tokens / (decode_ms / 1e3), "unit": "tok/s", "n_gpus": world,
        "steps": PREFIX_DECODE_STEPS, "warmup": 1, "ms_per_step": decode_ms / PREFIX_DECODE_STEPS,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": (f"prefix reuse on the 8M model: {B} requests per GPU share a "
                                f"{prefix_len}-token random prefix and add {suffix_len} own "
                                f"tokens, then {PREFIX_DECODE_STEPS} greedy decode steps each; "
                                f"{LAYERS} layers, hidden {HQ * D}, Hq={HQ}, Hkv={HKV}, d={D}, "
                                "f32 KV, random N(0, 0.02^2) weights"), "name": "prefix",
                   "exact_rows": exact_rows, "seed": args.seed},
        "prefill_tokens_computed": computed, "prefill_tokens_without_reuse": without,
        "prefill_tokens_saved": without - computed, "prefix_blocks_indexed": indexed,
        "prefill_ms": prefill_ms,
        "e2e": {"value": tokens / (e2e_decode_ms / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B,
                "loop": "decode steps with every step's chosen tokens copied to pinned host memory "
                        "and synchronized (the prompts copied in from pinned host memory before "
                        "the prefill)"},
        "gpu_launches": launches,
        "projections": "this library's fused exact-order projection kernels for every step"
                       if exact_rows >= 1024 else
                       f"exact order up to {exact_rows} rows, tensor-core GEMMs beyond",
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ok, secs = True, 0.0
        for i in (0, 1):  # request 0 prefilled the prefix; request 1 attached it
            good, t = oracle_generate_check(tensors, prefix_ids + suffix_ids[i],
                                            [int(x) for x in gen_h[i]], host_threads())
            ok, secs = ok and good, secs + t
        result["parity"] = {"greedy_tokens_match_cpu": ok, "requests_checked": 2,
                            "tokens_checked": 2 * (PREFIX_DECODE_STEPS + 1),
                            "oracle": "oracle model generating each request alone from its "
                                      "whole prompt"}
        result["cpu_baseline"] = {
            "value": 2 * PREFIX_DECODE_STEPS / secs, "unit": "tok/s", "cores": host_threads(),
            "kind": "port",
            "sample": (f"2 requests one at a time: oracle prefill of all {prefix_len + suffix_len} "
                       f"prompt tokens (no prefix cache in the reference), then "
                       f"{PREFIX_DECODE_STEPS} greedy steps; decode tokens / total seconds")}
    if rank == 0:
        print(json.dumps(result), flush=True)
    model.close()
    pool.close()
    close_dist(world)


def model_tensors(seed: int, intermediate_size: int = MODEL_INTER):
    """Random-init weights of the workload's model in the reference layout and
    order: matrices and the embedding N(0, 0.02^2) (seeded), norms 1."""
    import numpy as np

    import slmkv

    rng = np.random.default_rng(seed)
    out = []
    for _, shape in slmkv.model_tensor_shapes(vocab_size=MODEL_VOCAB, hidden_size=HQ * D,
                                              intermediate_size=intermediate_size,
                                              num_layers=LAYERS, kv_width=HKV * D):
        out.append(np.ones(shape, np.float32) if len(shape) == 1
                   else (0.02 * rng.standard_normal(shape)).astype(np.float32))
    return out


def model_cpu_baseline(tensors, prompt, threads: int, budget_s: float = 10.0):
    """The oracle's model decode on the host cores: prefill the prompt, then
    time greedy decode steps until about budget_s."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O

    cfg = dict(vocab_size=MODEL_VOCAB, hidden_size=HQ * D, intermediate_size=MODEL_INTER,
               num_layers=LAYERS, num_query_heads=HQ, num_key_value_heads=HKV, head_dimension=D,
               rms_norm_epsilon=1e-5, rope_theta=10000.0, situ_beta_gate=4.0, situ_beta_up=25.0)
    m = O.Model(cfg, tensors)
    cache = m.new_cache(CTX)
    tok = O.argmax_finite(m.prefill(cache, prompt, threads)[-1])
    toks = []
    n, t0 = 0, time.perf_counter()
    while n < LEN_HI and (time.perf_counter() - t0) < budget_s:
        toks.append(tok)
        tok = O.argmax_finite(m.decode(cache, tok, threads))
        n += 1
    dt = time.perf_counter() - t0
    toks.append(tok)  # n steps choose n tokens after the prompt's own
    return n / dt, n, toks


def run_model(args):
    """The 8M model end to end: prefill a 64-token random prompt, then greedy
    decode (one token per step, batch 1) through slm_model_decode; each step's
    next token stays on the device and feeds the next step's embedding.
    `value` is the decode steps per second with two steps in flight, summed
    over the GPUs (each runs its own replica of the request: weak scaling);
    `e2e` copies each step's token from pinned host memory and reads the
    chosen token back before the next step (a streaming server's loop). At one
    GPU the oracle generates from the same prompt on the host cores: every
    greedy token must agree (the CPU baseline)."""
    import numpy as np
    import torch

    import slmkv
    from slmkv.shard import max_over_ranks

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    init_dist(world, dev, args.pg_timeout)
    rng = np.random.default_rng(args.seed)
    prompt = [int(x) for x in rng.integers(0, MODEL_VOCAB, size=LEN_LO)]
    steps = min(max(args.steps, 1), LEN_HI)
    tensors = model_tensors(args.seed)
    pool = slmkv.KvPool(num_layers=LAYERS, num_query_heads=HQ, num_key_value_heads=HKV,
                        head_dimension=D, context_length=CTX, num_blocks=4 * (CTX // BLOCK) + 8,
                        max_sequences=2, device=local)
    model = slmkv.Model(pool, vocab_size=MODEL_VOCAB, intermediate_size=MODEL_INTER,
                        tensors=tensors)
    if args.exact_rows is not None:
        model.set_exact_rows(args.exact_rows)
    stream = torch.cuda.current_stream()
    ids = torch.tensor(prompt, dtype=torch.int32, device=dev)
    tok = [torch.zeros(1, dtype=torch.int32, device=dev) for _ in range(2)]
    gen = torch.zeros(LEN_HI + 1, dtype=torch.int32, device=dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def generate(n_steps, e2e=False, record=False):
        cache = pool.allocate_kv_cache(CTX)
        e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        e[0].record(stream)
        with pool.begin([cache], [LEN_LO]) as b:
            model.prefill(b, ids, None, tok[0])
        e[1].record(stream)
        if record:
            gen[0:1].copy_(tok[0])
        plan = pool.step_plan([cache], 1)
        h_tok = torch.zeros(1, dtype=torch.int32).pin_memory()
        out = []
        if e2e:  # the prompt's own next token, streamed before the first step
            h_tok.copy_(tok[0], non_blocking=True)
            stream.synchronize()
            out.append(int(h_tok[0]))
        inflight = []
        t_host = time.perf_counter()
        for i in range(n_steps):
            cur, nxt = tok[i % 2], tok[(i + 1) % 2]
            if e2e:
                cur.copy_(h_tok, non_blocking=True)
            b = plan.begin()
            model.decode(b, cur, None, nxt)
            if record:
                gen[i + 1:i + 2].copy_(nxt)
            if e2e:
                if b.end(raise_on_error=False) != [0]:
                    raise RuntimeError("decode step failed")
                h_tok.copy_(nxt, non_blocking=True)
                stream.synchronize()
                out.append(int(h_tok[0]))
            else:
                inflight.append(b.submit())
                while len(inflight) > 1:
                    if any(inflight.pop(0).wait(raise_on_error=False)):
                        raise RuntimeError("decode step failed")
        for b in inflight:
            if any(b.wait(raise_on_error=False)):
                raise RuntimeError("decode step failed")
        e[2].record(stream)
        torch.cuda.synchronize()
        host_s = time.perf_counter() - t_host
        if cache.sequence_length() != LEN_LO + n_steps:
            raise RuntimeError(f"unexpected length {cache.sequence_length()}")
        cache.free()
        return e[0].elapsed_time(e[1]), e[1].elapsed_time(e[2]), host_s, out

    for _ in range(max(args.warmup, 3)):
        generate(min(steps, 16))
    barrier()
    l0 = pool.launch_count()
    prefill_ms, decode_ms, _, _ = generate(steps)
    launches = pool.launch_count() - l0
    barrier()
    _, _, e2e_s, toks = generate(steps, e2e=True)
    _, _, _, _ = generate(steps, record=True)  # the generated tokens, for the parity check
    decode_ms, e2e_ms, prefill_ms = max_over_ranks([decode_ms, e2e_s * 1e3, prefill_ms], device=dev)
    gen_h = gen[:steps + 1].cpu().tolist()
    if gen_h != toks:
        raise RuntimeError("the e2e run chose other tokens than the device-resident run")
    value = world * steps / (decode_ms / 1e3)
    result = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
        "warmup": max(args.warmup, 3), "ms_per_step": decode_ms / steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": (f"8M model end to end: batch 1 per GPU, {LEN_LO}-token random "
                                f"prompt, {steps} greedy decode steps; {LAYERS} layers, hidden "
                                f"{HQ * D}, FFN {MODEL_INTER} SiTU-GLU, Hq={HQ}, Hkv={HKV}, d={D}, "
                                f"vocab {MODEL_VOCAB}, f32 KV, random N(0, 0.02^2) weights "
                                f"(seed {args.seed})"), "name": "model", "seed": args.seed,
                   "exact_rows": 1024 if args.exact_rows is None else args.exact_rows},
        "prefill_ms": prefill_ms,
        "e2e": {"value": world * steps / (e2e_ms / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                "loop": "pinned H2D of the step's token, decode, D2H of the chosen token, "
                        "host synchronizes every step"},
        "gpu_launches": launches,
        "projections": "this library's fused exact-order projection kernels (bf16 operands, "
                       "the reference's fp32 fold order); cuBLAS fp32 SGEMV for the tied head "
                       "of one row",
        "generated_head": toks[:8],
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        tps, n, cpu_toks = model_cpu_baseline(tensors, prompt, threads, budget_s=1e9)
        # every greedy token of the run, the prompt's own next token first
        match = cpu_toks == toks[:len(cpu_toks)]
        result["parity"] = {"greedy_tokens_match_cpu": match, "tokens_checked": len(cpu_toks),
                            "oracle": "oracle model (model.rs:342-397 restated), same weights "
                                      "and prompt"}
        result["greedy_tokens_match_cpu"] = match
        result["cpu_baseline"] = {"value": tps, "unit": "tok/s", "cores": threads, "kind": "port",
                                  "sample": f"{n} greedy decode steps of the same model and "
                                            f"prompt (oracle, OpenMP projections, serial "
                                            f"attention as the reference)"}
    if rank == 0:
        print(json.dumps(result), flush=True)
    model.close()
    pool.close()
    close_dist(world)


def gqa_model_step_bytes(lengths) -> int:
    """Algorithmic HBM bytes of one decode step of the scaled model for a
    batch whose caches hold `lengths` entries: every bf16 projection matrix
    once, the fp32 tied embedding once (the vocabulary projection), and the
    KV path's bytes for every layer. Activations (a few MB) are left out."""
    H, KV, I = HQ * D, HKV * D, GQA_MODEL_INTER
    weights = LAYERS * 2 * (H * (H + 2 * KV) + H * H + 2 * H * I + I * H)
    head = 4 * MODEL_VOCAB * H
    return weights + head + LAYERS * algorithmic_bytes(lengths)


def gqa_model_cpu_baseline(tensors, length: int, seed: int, threads: int, budget_s: float = 20.0):
    """The oracle's model decode of ONE sequence at the scaled shape (the
    reference engine serves one request at a time): its cache is filled with
    `length` random bf16-rounded K/V entries per layer, then greedy decode
    steps are timed (projections on all threads, attention serial)."""
    import numpy as np

    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O

    cfg = dict(vocab_size=MODEL_VOCAB, hidden_size=HQ * D, intermediate_size=GQA_MODEL_INTER,
               num_layers=LAYERS, num_query_heads=HQ, num_key_value_heads=HKV, head_dimension=D,
               rms_norm_epsilon=1e-5, rope_theta=10000.0, situ_beta_gate=4.0, situ_beta_up=25.0)
    m = O.Model(cfg, tensors)
    cache = m.new_cache(CTX, quantize_bf16=True)
    rng = np.random.default_rng(seed + 5)
    for layer in range(LAYERS):
        kv = rng.standard_normal((2, length, HKV, D)).astype(np.float32)
        cache.append_layer(layer, kv[0], kv[1], length)
    tok, n = 1, 0
    t0 = time.perf_counter()
    while n < 2 or (n < 8 and time.perf_counter() - t0 < budget_s):
        tok = O.argmax_finite(m.decode(cache, tok, threads))
        n += 1
    return n / (time.perf_counter() - t0), n


def run_gqa_model(args):
    """The scaled GQA model end to end on every GPU (weak scaling, no
    collective on the data path): B sequences a GPU with random prompts,
    prefilled in one batch, then greedy decode steps for all of them in one
    batch per step, two steps in flight, the chosen tokens staying on the
    device. Projections run as tensor-core GEMMs (cuBLAS bf16, fp32
    accumulate). value = decode tokens of all ranks / the slowest rank's
    device time; e2e copies each step's tokens from pinned host memory and
    reads the chosen tokens back before the next step. Parity of this shape
    (bf16 KV, 2e-2) is checked by the GPU tests on two of its layers; the
    oracle's CPU prefill of 16 prompts of thousands of tokens would take
    hours."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import slmkv
    from slmkv.shard import max_over_ranks

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    init_dist(world, dev, args.pg_timeout)
    steps = min(max(args.steps, 1), GQA_MODEL_STEPS)
    warm = max(args.warmup, 3)
    # B lengths per rank from one seeded draw, so rank r's share is the same
    # at every world size
    all_lens = np.random.default_rng(args.seed).integers(LEN_LO, LEN_HI + 1, size=B * max(world, 8))
    lens = [int(x) for x in all_lens[rank * B:(rank + 1) * B]]
    prng = np.random.default_rng(args.seed + 1 + rank)
    prompts = [prng.integers(0, MODEL_VOCAB, size=L).astype(np.int32) for L in lens]
    tensors = model_tensors(args.seed, GQA_MODEL_INTER)
    blocks = sum(-(-(L + GQA_MODEL_STEPS) // BLOCK) for L in lens) + 8
    pool = slmkv.KvPool(num_layers=LAYERS, num_query_heads=HQ, num_key_value_heads=HKV,
                        head_dimension=D, context_length=CTX, num_blocks=blocks, max_sequences=B,
                        kv_dtype=slmkv.KV_BF16, device=local)
    pool.shuffle(args.seed + 1)
    model = slmkv.Model(pool, vocab_size=MODEL_VOCAB, intermediate_size=GQA_MODEL_INTER,
                        tensors=tensors)
    model.set_exact_rows(0 if args.exact_rows is None else args.exact_rows)
    caches = [pool.allocate_kv_cache(CTX) for _ in lens]
    stream = torch.cuda.current_stream()
    ids = torch.from_numpy(np.concatenate(prompts)).to(dev)
    tok = [torch.zeros(B, dtype=torch.int32, device=dev) for _ in range(2)]
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    ev[0].record(stream)
    with pool.begin(caches, lens) as b:
        model.prefill(b, ids, None, tok[0])
    ev[1].record(stream)
    torch.cuda.synchronize()
    prefill_ms = ev[0].elapsed_time(ev[1])
    first = tok[0].clone()
    h_tok = torch.zeros(B, dtype=torch.int32).pin_memory()
    plan = pool.step_plan(caches, 1)
    lens_arr = plan.lengths(lens)

    def decode(n, e2e=False):
        tok[0].copy_(first)
        if e2e:
            h_tok.copy_(first)
        inflight = []
        for i in range(n):
            cur, nxt = tok[i % 2], tok[(i + 1) % 2]
            if e2e:
                cur.copy_(h_tok, non_blocking=True)
            b = plan.begin()
            model.decode(b, cur, None, nxt)
            if e2e:
                if any(b.end(raise_on_error=False)):
                    raise RuntimeError("decode step failed")
                h_tok.copy_(nxt, non_blocking=True)
                stream.synchronize()
            else:
                inflight.append(b.submit())
                while len(inflight) > 1:
                    if any(inflight.pop(0).wait(raise_on_error=False)):
                        raise RuntimeError("decode step failed")
        for b in inflight:
            if any(b.wait(raise_on_error=False)):
                raise RuntimeError("decode step failed")

    def rewind():
        torch.cuda.synchronize()
        if [c.sequence_length() for c in caches] != [L + done[0] for L in lens]:
            raise RuntimeError("unexpected cache lengths")
        plan.truncate_all(lens_arr)

    done = [warm]
    decode(warm)
    rewind()
    clocks = ClockSampler(local)
    clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    l0 = pool.launch_count()
    ev[2].record(stream)
    decode(steps)
    ev[3].record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    launches = pool.launch_count() - l0
    (ms,) = max_over_ranks([ev[2].elapsed_time(ev[3])], device=dev)
    done[0] = steps
    rewind()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev[4].record(stream)
    decode(steps, e2e=True)
    ev[5].record(stream)
    torch.cuda.synchronize()
    (e2e_ms,) = max_over_ranks([ev[4].elapsed_time(ev[5])], device=dev)
    rewind()
    (prefill_ms,) = max_over_ranks([prefill_ms], device=dev)
    step_bytes = sum(gqa_model_step_bytes([L + i for L in lens]) for i in range(steps))
    peaks, kind = measured_peaks()
    achieved = step_bytes / (ms / 1e3) / 1e9
    tokens = world * B * steps
    result = {
        "metric": METRIC, "value": tokens / (ms / 1e3), "unit": "tok/s", "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": ms / steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": (f"scaled GQA model end to end: {B} sequences per GPU, random "
                                f"prompts of U[{LEN_LO},{LEN_HI}] tokens prefilled in one batch, "
                                f"then {steps} greedy decode steps of all {B} per step; "
                                f"{LAYERS} layers, hidden {HQ * D}, FFN {GQA_MODEL_INTER} "
                                f"SiTU-GLU, Hq={HQ}, Hkv={HKV}, d={D}, vocab {MODEL_VOCAB}, "
                                f"context {CTX}, bf16 KV, {BLOCK}-token shuffled blocks, random "
                                f"N(0, 0.02^2) weights (seed {args.seed})"),
                   "name": "gqa-model", "seed": args.seed,
                   "exact_rows": 0 if args.exact_rows is None else args.exact_rows,
                   "l2": "no flush: a step reads ~2 GB (weights and K/V), far above the 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": None,
                     "peak_kind": kind,
                     "kernel": "the whole decode step: algorithmic bytes (bf16 projection "
                               "matrices, fp32 tied embedding, the KV path per layer) / step "
                               "time"},
        "prefill_ms": prefill_ms,
        "prefill_tok_s": world * sum(lens) / (prefill_ms / 1e3),
        "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": 4 * B,
                "d2h_bytes_per_step": 4 * B,
                "loop": "pinned H2D of the step's tokens, decode, D2H of the chosen tokens, host "
                        "synchronizes every step"},
        "gpu_launches": launches,
        "clocks": clk,
        "projections": "this library's tcgen05 row GEMMs (bf16 operands, fp32 accumulate; "
                       "cuBLAS beyond 512 rows: the prefill); cuBLAS fp32 SGEMM for the tied "
                       "head; embedding, RMSNorm, rounding, argmax and the KV step are this "
                       "library's kernels",
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle as O

        threads = host_threads()
        at = int(np.mean(lens)) + steps // 2
        tps, n = gqa_model_cpu_baseline(tensors, at, args.seed, threads)
        result["cpu_baseline"] = {
            "value": tps, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": (f"{n} greedy decode steps of one sequence of the same model whose cache "
                       f"holds {at} entries (this GPU's mean prompt + half the steps); oracle, "
                       "OpenMP projections, serial attention as the reference, which serves one "
                       "request at a time")}
    if rank == 0:
        print(json.dumps(result), flush=True)
    model.close()
    pool.close()
    close_dist(world)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif WORKLOAD_NAME == "model":
        run_model(args)
    elif WORKLOAD_NAME == "gqa-model":
        run_gqa_model(args)
    elif WORKLOAD_NAME == "serve":
        run_serve(args)
    elif WORKLOAD_NAME == "prefix":
        run_prefix(args)
    else:
        result = run_ours(args)
        if WORKLOAD_NAME == "microbench" and not args.no_configs and args.batch is None:
            configs = run_configs(args, dist_env()[1])
            if result is not None:
                result["configs"] = configs
        if result is not None:
            print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()

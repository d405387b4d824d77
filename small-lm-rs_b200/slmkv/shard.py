"""Request sharding across the GPUs of one node (one process per GPU).

Sequences of the KV-cache path are independent, so requests are partitioned
across GPUs with no collective on the data path: each GPU owns its own pool
and its own requests. The only cross-rank steps are host-side: assigning
requests to ranks, and agreeing on timings (max over ranks) in benchmarks.
"""

from __future__ import annotations

import heapq
from typing import Sequence


def assign_requests(costs: Sequence[int], world: int) -> list[int]:
    """Rank of every request, balancing total cost (e.g. prompt + output
    tokens) with a longest-first greedy onto the least-loaded rank. Ties go
    to the lower rank, so every process computes the same assignment."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-int(costs[i]), i))
    heap = [(0, r) for r in range(world)]
    owner = [0] * len(costs)
    for i in order:
        load, r = heapq.heappop(heap)
        owner[i] = r
        heapq.heappush(heap, (load + int(costs[i]), r))
    return owner


def rank_share(costs: Sequence[int], world: int, rank: int) -> list[int]:
    """Indices of the requests rank `rank` serves, in request order."""
    owner = assign_requests(costs, world)
    return [i for i, r in enumerate(owner) if r == rank]


def max_over_ranks(values: Sequence[float], device=None) -> list[float]:
    """Element-wise max of `values` over all ranks of the default process
    group (identity without one). Used for timings: a multi-GPU step takes as
    long as its slowest rank."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]

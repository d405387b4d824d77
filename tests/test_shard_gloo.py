"""Multi-rank host logic on CPU: two gloo ranks agree on the request
assignment (disjoint, complete, balanced) and on max-over-ranks timings —
the only cross-rank steps of the multi-GPU path (no data-path collective)."""

import os
import socket

import pytest
import torch.multiprocessing as mp

from slmkv.shard import assign_requests, max_over_ranks, rank_share


def test_assignment_is_deterministic_balanced_and_complete():
    costs = [(i * 37) % 251 + 8 for i in range(4096)]
    for world in (1, 2, 4, 8):
        owner = assign_requests(costs, world)
        assert owner == assign_requests(costs, world)
        loads = [0] * world
        for c, r in zip(costs, owner):
            loads[r] += c
        assert max(loads) - min(loads) <= max(costs)
        shares = [rank_share(costs, world, r) for r in range(world)]
        assert sorted(i for s in shares for i in s) == list(range(len(costs)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, costs, out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = rank_share(costs, world, rank)
        timing = max_over_ranks([1.0 + rank, 10.0 - rank])
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        out[rank] = (timing, gathered)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_share_requests_and_max_timings():
    costs = [(i * 13) % 97 + 16 for i in range(300)]
    world = 2
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(world, _free_port(), costs, out), nprocs=world, join=True)
        results = dict(out)
    for rank in range(world):
        timing, gathered = results[rank]
        assert timing == [2.0, 10.0]  # element-wise max over the two ranks
        flat = sorted(i for share in gathered for i in share)
        assert flat == list(range(len(costs)))
        assert not set(gathered[0]) & set(gathered[1])

"""The N>1 host logic on CPU: two gloo ranks agree on a whole-request assignment without
communicating, and the timing reductions (max over ranks, sum over ranks) are right."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vflorence_b200.sharding import assign_requests, max_over_ranks, sum_over_ranks


def test_assignment_is_a_partition_and_balanced():
    costs = [577 + 3 * 256] * 10 + [300 + 3 * 142] * 30 + [1024 + 64] * 7
    shards = assign_requests(costs, 4)
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(len(costs)))
    loads = [sum(costs[i] for i in s) for s in shards]
    assert max(loads) - min(loads) <= max(costs)
    assert assign_requests(costs, 4) == shards            # deterministic
    assert assign_requests([5, 1], 1) == [[0, 1]]
    assert assign_requests([], 3) == [[], [], []]
    with pytest.raises(ValueError):
        assign_requests([1], 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, costs, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = assign_requests(costs, world)[rank]
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        elapsed = 10.0 + rank * 5.0
        out[rank] = (gathered, max_over_ranks(elapsed), sum_over_ranks(len(mine)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree():
    costs = [int(c) for c in torch.randint(200, 1200, (23,), generator=torch.Generator().manual_seed(1))]
    world = 2
    with mp.Manager() as m:
        out = m.dict()
        mp.start_processes(_rank_main, args=(world, _free_port(), costs, out), nprocs=world,
                           start_method="spawn", join=True)
        res = dict(out)
    g0, mx0, sm0 = res[0]
    g1, mx1, sm1 = res[1]
    assert g0 == g1                                        # same view on both ranks
    assert sorted(g0[0] + g0[1]) == list(range(len(costs)))
    assert not set(g0[0]) & set(g0[1])
    assert mx0 == mx1 == 15.0
    assert sm0 == sm1 == len(costs)

"""Whole-request sharding across GPUs (one process per GPU) and the two reductions timing needs.

The paged path has no cross-GPU exchange: a request - with all its beams, its encoder pages and
its self-attention blocks - lives on one GPU. Requests are dealt to ranks greedily by estimated
cost (longest first onto the least-loaded rank), deterministically, so every rank computes the
same assignment without communicating. The only collectives are the timing reductions below
(max of elapsed time, sum of work), never on the data path.
"""

from __future__ import annotations

import heapq

import torch


def assign_requests(costs, world_size: int) -> list[list[int]]:
    """Indices of the requests each rank serves (each rank's list in ascending order).

    ``costs[i]`` estimates request i's work (e.g. encoder length + beams x max tokens). Longest
    first onto the least-loaded rank (ties: lower rank); deterministic for equal inputs.
    """
    if world_size < 1:
        raise ValueError("world_size must be >= 1")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0, r) for r in range(world_size)]
    shards = [[] for _ in range(world_size)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    return [sorted(s) for s in shards]


def _reduce(value: float, op) -> float:
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=op)
    return float(t.item())


def max_over_ranks(value: float) -> float:
    """The largest ``value`` of any rank (elapsed times: the job ends with its slowest rank)."""
    import torch.distributed as dist

    return _reduce(value, dist.ReduceOp.MAX)


def sum_over_ranks(value: float) -> float:
    """The sum of ``value`` over ranks (work done by the whole job)."""
    import torch.distributed as dist

    return _reduce(value, dist.ReduceOp.SUM)


def gather_to_rank0(obj):
    """Every rank's ``obj`` as a list on rank 0 (None on the other ranks); ``[obj]`` without a
    process group. Host-side reporting only, after the timed regions."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [obj]
    out = [None] * dist.get_world_size() if dist.get_rank() == 0 else None
    dist.gather_object(obj, out, dst=0)
    return out

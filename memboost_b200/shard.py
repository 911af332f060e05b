"""Multi-GPU host logic: quantizing many independent matrices over ranks.

Quantization of one matrix needs nothing from any other, so a model's
matrices shard over one process per GPU with no collective on the data path:
``lpt_partition`` balances them by size (longest processing time first), each
rank quantizes its own share, and results or timings are combined only at
the end (``gather_to_all``, ``max_over_ranks``).  Works with any
torch.distributed backend (NCCL for the GPU runs, gloo for the CPU tests).
"""
from __future__ import annotations

import heapq
from typing import Callable, Sequence


def lpt_partition(costs: Sequence[float], world: int) -> list[list[int]]:
    """Indices of ``costs`` per rank: the costliest first, each to the rank
    with the least total so far (ties to the lowest rank); every index
    appears exactly once and each rank's list is ascending."""
    if world < 1:
        raise ValueError("world must be >= 1")
    heap = [(0.0, r) for r in range(world)]
    heapq.heapify(heap)
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + float(costs[i]), r))
    return [sorted(p) for p in parts]


def quantize_shard(items: Sequence, rank: int, world: int, cost: Callable, fn: Callable) -> dict:
    """Apply ``fn`` to this rank's share of ``items`` (partitioned by
    ``cost(item)``); returns {index: result}."""
    part = lpt_partition([cost(it) for it in items], world)[rank]
    return {i: fn(items[i]) for i in part}


def _dist():
    import torch.distributed as dist
    return dist if dist.is_available() and dist.is_initialized() else None


def max_over_ranks(x: float) -> float:
    """The maximum of ``x`` over the ranks of the default process group (x
    itself without one); every rank must call it."""
    dist = _dist()
    if dist is None or dist.get_world_size() == 1:
        return x
    import torch
    dev = torch.device("cuda", torch.cuda.current_device()) \
        if dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_to_all(local: dict) -> dict:
    """Union of every rank's ``local`` dict (picklable values, disjoint
    keys), on every rank."""
    dist = _dist()
    if dist is None or dist.get_world_size() == 1:
        return dict(local)
    parts = [None] * dist.get_world_size()
    dist.all_gather_object(parts, local)
    out: dict = {}
    for p in parts:
        out.update(p)
    return out

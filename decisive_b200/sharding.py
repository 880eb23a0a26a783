"""Request-level data parallelism across the GPUs of one node.

Independent requests (sequences) are partitioned across ranks -- one process and one full model
replica per GPU -- with no collective on the hot path; each rank runs its share on its own device
and the results are gathered on the host afterwards (one host-side gather per batch).

- C2 (independent fixed-length sequences): round-robin.
- C3 (ragged batch): longest-processing-time-first by the cost len + c * len^2 (the linear
  projections plus the quadratic attention of one sequence), each sequence to the least loaded
  rank; ties go to the lowest rank, so every rank computes the same assignment locally.
"""
from __future__ import annotations

from typing import Any, Sequence


def assign_round_robin(n_items: int, world: int) -> list[list[int]]:
    """Indices of the items each rank owns: item i -> rank i % world."""
    if world <= 0 or n_items < 0:
        raise ValueError("world must be positive and n_items non-negative")
    return [list(range(r, n_items, world)) for r in range(world)]


def sequence_cost(length: int, quadratic: float) -> float:
    """Relative cost of one sequence: projections grow with len, attention with len^2."""
    return float(length) + quadratic * float(length) * float(length)


def assign_lpt(lengths: Sequence[int], world: int, quadratic: float = 1.0 / 1024) -> list[list[int]]:
    """Longest-processing-time-first partition of sequences across ranks.  Deterministic: items
    are taken by decreasing cost (ties by index) and placed on the least loaded rank (ties by
    rank).  Each rank's list is returned in ascending index order."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(lengths)), key=lambda i: (-sequence_cost(lengths[i], quadratic), i))
    load = [0.0] * world
    owned: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        owned[r].append(i)
        load[r] += sequence_cost(lengths[i], quadratic)
    return [sorted(o) for o in owned]


def rank_loads(assignment: list[list[int]], lengths: Sequence[int], quadratic: float = 1.0 / 1024) -> list[float]:
    return [sum(sequence_cost(lengths[i], quadratic) for i in items) for items in assignment]


def gather_ordered(local: dict[int, Any], n_items: int, group=None, dst: int = 0) -> list[Any] | None:
    """Gathers every rank's {item index: result} on rank dst and returns the results in item
    order there (None on the other ranks).  Uses torch.distributed object collectives (works with
    the gloo and nccl backends); raises if an item is missing or produced twice."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    parts = [None] * world if rank == dst else None
    dist.gather_object(local, parts, dst=dst, group=group)
    if rank != dst:
        return None
    merged: dict[int, Any] = {}
    for p in parts:
        for k, v in p.items():
            if k in merged:
                raise RuntimeError(f"item {k} produced by two ranks")
            merged[k] = v
    missing = [i for i in range(n_items) if i not in merged]
    if missing:
        raise RuntimeError(f"items never produced: {missing[:8]}")
    return [merged[i] for i in range(n_items)]

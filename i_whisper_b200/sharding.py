"""Utterance sharding across GPUs (one process per GPU).

Utterances are independent through the whole encoder + greedy decoder, so
a job over G GPUs gives rank r a contiguous block of utterances and runs
the full model on it with no data exchange. The only collectives are for
bookkeeping outside the data path: the slowest rank's time (max over ranks)
and gathering the token matrices back in global utterance order.
"""
from __future__ import annotations

from typing import List, Tuple


def shard_bounds(n_total: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, stop) of rank's utterances: contiguous blocks of
    ceil(n_total / world), the last ones possibly shorter or empty."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"rank {rank} outside world of {world}")
    if n_total < 0:
        raise ValueError("n_total must be non-negative")
    per = -(-n_total // world)
    start = min(rank * per, n_total)
    return start, min(start + per, n_total)


def window_seeds(start: int, stop: int, n_distinct: int = 32) -> List[int]:
    """Audio seeds of utterances [start, stop): the global utterance index
    modulo the number of distinct synthetic windows."""
    return [g % n_distinct for g in range(start, stop)]


def _dist():
    import torch.distributed as dist
    return dist if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1 else None


def max_over_ranks(value: float, device=None) -> float:
    """The largest value over all ranks (the job's time is its slowest
    rank's); the value itself in a single-process run."""
    import torch
    dist = _dist()
    if dist is None:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_rows(t):
    """Concatenate every rank's rows of ``t`` in rank order (equal row
    counts per rank), on every rank."""
    import torch
    dist = _dist()
    if dist is None:
        return t
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t.contiguous())
    return torch.cat(parts, dim=0)

"""Utterance sharding across GPUs (one process per GPU).

Utterances are independent through the whole encoder + greedy decoder, so
a job over G GPUs gives rank r a contiguous block of utterances and runs
the full model on it with no data exchange. The only collectives are for
bookkeeping outside the data path: the slowest rank's time (max over ranks)
and gathering the token matrices back in global utterance order.
"""
from __future__ import annotations

import time
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


class PeerFailure(RuntimeError):
    """A peer rank stopped posting steps (it raised, exited or hangs on the host)."""


class PeerMonitor:
    """Host-side liveness check between steps of the sharded run.

    Each rank posts the number of the step it has finished in a key-value
    store shared by the job (the process group's store, or any
    ``torch.distributed.Store``). Before launching step ``s`` a rank calls
    ``wait_peers(s)``: it returns once every peer has posted step ``s - 1``
    and raises :class:`PeerFailure`, naming the silent ranks, when that takes
    longer than ``timeout_s``. A rank therefore learns that a peer has gone
    between steps, before it launches work that would wait on that peer, and
    no GPU-side wait is involved. Ranks post only between steps, with none of
    their kernels or collectives in flight.
    """

    def __init__(self, store, rank: int, world: int, timeout_s: float = 30.0, prefix: str = "iw/step",
                 poll_s: float = 0.01):
        if world <= 0 or not (0 <= rank < world):
            raise ValueError(f"rank {rank} outside world of {world}")
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix, self.poll_s = float(timeout_s), prefix, float(poll_s)

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def post(self, step: int) -> None:
        """Record that this rank has finished ``step``."""
        self.store.set(self._key(self.rank), str(int(step)))

    def _posted(self, r: int) -> int:
        if self.store.check([self._key(r)]):
            return int(self.store.get(self._key(r)).decode())
        return -1

    def wait_peers(self, step: int) -> None:
        """Return once every other rank has finished ``step - 1``."""
        need = int(step) - 1
        if need < 0 or self.world == 1:
            return
        deadline = time.monotonic() + self.timeout_s
        missing: List[int] = []
        while True:
            missing = [r for r in range(self.world) if r != self.rank and self._posted(r) < need]
            if not missing:
                return
            if time.monotonic() >= deadline:
                raise PeerFailure(f"rank {self.rank}: rank(s) {missing} did not finish step {need} "
                                  f"within {self.timeout_s:.1f} s")
            time.sleep(self.poll_s)


def default_store():
    """The store of the default process group (None without one)."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return None
    return dist.distributed_c10d._get_default_store()

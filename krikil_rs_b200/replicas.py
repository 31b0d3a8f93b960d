"""Multi-GPU decode as independent replicas.

A 25M-parameter model does not shard: every rank (one process per GPU) holds a
full copy of the weights and decodes its own contiguous slice of the
sequences, so the data path has no collective.  torch.distributed is used only
around the timed region -- a barrier before it and, after it, the max over
ranks of the device times and the sum of the generated-token counts.  Every
rank takes the same collective steps in the same order.

Failures: the driver's work runs in phases (`Phase`), each ended on every rank
by one status exchange that also serves as the phase's barrier.  A rank whose
phase raised still takes that exchange, so it never leaves the others waiting
in a collective it will not reach; once any rank reports a failure, every rank
raises `ReplicaFailure` naming the failed ranks and their errors, and skips the
remaining collectives together.  A rank that dies outright (never reaches the
exchange) is caught by the process group's timeout: the others' exchange ends
with an error instead of waiting for good.
"""
from __future__ import annotations

from typing import Dict, Optional, Sequence, Tuple


def shard(items: Sequence, world: int, rank: int) -> Sequence:
    """Rank `rank`'s slice of `items` split into `world` equal contiguous parts
    (len(items) must be a multiple of world)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if len(items) % world:
        raise ValueError(f"{len(items)} items do not split evenly over {world} ranks")
    per = len(items) // world
    return items[rank * per:(rank + 1) * per]


def reduce_timings(dist, device, times_ms: Sequence[float], tokens: int) -> Tuple[list, int]:
    """Max over ranks of each time, sum over ranks of the token count.  With a
    single process (dist not initialised) the inputs come back unchanged."""
    import torch
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(times_ms), int(tokens)
    t = torch.tensor(list(times_ms), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    g = torch.tensor([int(tokens)], dtype=torch.int64, device=device)
    dist.all_reduce(g)
    return [float(x) for x in t.tolist()], int(g.item())


class ReplicaFailure(RuntimeError):
    """Raised on every rank when some rank's phase failed; `failed` maps each
    failed rank to its error message."""

    def __init__(self, failed: Dict[int, str]):
        self.failed = dict(failed)
        super().__init__("replica failure on rank(s) " +
                         "; ".join(f"{r}: {m}" for r, m in sorted(self.failed.items())))


def exchange_status(dist, error: Optional[str]) -> None:
    """Every rank reports its phase's outcome (None = fine); all ranks raise
    ReplicaFailure together if any rank failed.  Without an initialised
    multi-rank process group the local outcome alone decides."""
    if not (dist is not None and dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        if error is not None:
            raise ReplicaFailure({0: error})
        return
    msgs = [None] * dist.get_world_size()
    dist.all_gather_object(msgs, error)
    failed = {r: m for r, m in enumerate(msgs) if m is not None}
    if failed:
        raise ReplicaFailure(failed)


class Phase:
    """A phase of the replicated driver: `with Phase(dist): ...` runs the body
    on this rank, then exchanges the outcome with the other ranks (the
    exchange is the phase's barrier).  An exception from the body is reported,
    not propagated alone: every rank then raises ReplicaFailure together.
    Exceptions that are not Exceptions (KeyboardInterrupt, SystemExit) pass
    through untouched."""

    def __init__(self, dist):
        self.dist = dist

    def __enter__(self):
        return self

    def __exit__(self, et, ev, tb):
        if et is not None and not issubclass(et, Exception):
            return False
        exchange_status(self.dist, None if ev is None else f"{et.__name__}: {ev}")
        return False

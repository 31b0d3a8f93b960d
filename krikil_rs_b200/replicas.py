"""Multi-GPU decode as independent replicas.

A 25M-parameter model does not shard: every rank (one process per GPU) holds a
full copy of the weights and decodes its own contiguous slice of the
sequences, so the data path has no collective.  torch.distributed is used only
around the timed region -- a barrier before it and, after it, the max over
ranks of the device times and the sum of the generated-token counts.  Every
rank takes the same collective steps in the same order.
"""
from __future__ import annotations

from typing import Sequence, Tuple


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

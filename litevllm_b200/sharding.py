"""Request sharding across GPUs (one process per GPU, no data-path collective).

shard(): sequence i of a global batch belongs to rank i // per_rank.
balanced_shard(): the same number of sequences per rank, chosen so that the
ranks' total context lengths (their decode bytes) are nearly equal: the
step's time is the slowest rank's, and contiguous index blocks of random
lengths leave one rank with noticeably more tokens than the mean.
Every input of a sequence is keyed by its global index
(litevllm_b200.workloads), so any world size reproduces the same union of
work. torch.distributed is used only to agree on timing: a barrier and the
max over ranks.
"""

from __future__ import annotations

import torch


def shard(global_batch: int, world: int, rank: int) -> range:
    """Contiguous block of global sequence indices owned by `rank`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    per, rem = divmod(global_batch, world)
    start = rank * per + min(rank, rem)
    return range(start, start + per + (1 if rank < rem else 0))


def balanced_shard(lengths, world: int, rank: int) -> list:
    """Global indices owned by `rank` when sequences of the given lengths are
    dealt to `world` ranks, longest first, in serpentine order (0 .. W-1,
    W-1 .. 0, ...): every rank gets the same count (+-1) and one sequence of
    each length band, so the totals differ by less than one band's spread.
    Deterministic: ties keep index order. Returned in increasing index order."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    mine = []
    for pos, i in enumerate(order):
        band, k = divmod(pos, world)
        owner = k if band % 2 == 0 else world - 1 - k
        if owner == rank:
            mine.append(i)
    return sorted(mine)


def max_over_ranks(values, device=None):
    """Element-wise max of a list of floats over all ranks (identity when not distributed)."""
    if not (torch.distributed.is_available() and torch.distributed.is_initialized()):
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]

"""Request sharding across GPUs (one process per GPU, no data-path collective).

Sequence i of a global batch belongs to rank i // per_rank. Every input of a
sequence is keyed by its global index (litevllm_b200.workloads), so any world
size reproduces the same union of work. torch.distributed is used only to
agree on timing: a barrier and the max over ranks.
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


def max_over_ranks(values, device=None):
    """Element-wise max of a list of floats over all ranks (identity when not distributed)."""
    if not (torch.distributed.is_available() and torch.distributed.is_initialized()):
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]

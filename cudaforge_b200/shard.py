"""Batch sharding across GPUs (one process per GPU, no data-path collective).

Sequences are independent units: rank r owns its own `batch_per_rank`
sequences, weights replica, KV pools and page tables.  The only collective
is the bench's timing reduction: max over ranks of the device times (the
job is as slow as its slowest rank) and the sum of the emitted tokens."""
from __future__ import annotations

from typing import Sequence, Tuple

import torch


def rank_sequence_ids(rank: int, batch_per_rank: int) -> list:
    """Global sequence ids owned by `rank` (contiguous blocks)."""
    return list(range(rank * batch_per_rank, (rank + 1) * batch_per_rank))


def reduce_step_metrics(times_ms: Sequence[float], tokens: Sequence[float], device=None,
                        group=None) -> Tuple[list, list]:
    """All-reduce MAX over `times_ms` and SUM over `tokens` (no-op when
    torch.distributed is not initialised)."""
    import torch.distributed as dist
    t = torch.tensor(list(times_ms), dtype=torch.float64, device=device)
    n = torch.tensor(list(tokens), dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        dist.all_reduce(n, op=dist.ReduceOp.SUM, group=group)
    return t.tolist(), n.tolist()


def split_global_batch(global_batch: int, world: int) -> int:
    """Sequences per rank when a fixed global batch is split across `world`
    ranks (strong scaling); the batch must divide evenly."""
    if global_batch % world:
        raise ValueError(f"global batch {global_batch} does not split evenly over {world} ranks")
    return global_batch // world


def gather_emitted(seq_ids: Sequence[int], emitted: Sequence[Sequence[int]], group=None, dst: int = 0):
    """Collect every rank's emitted tokens on rank `dst` (host side, outside
    the timed region): returns {global sequence id: tokens} on `dst`, None
    elsewhere; without torch.distributed the local dict."""
    import torch.distributed as dist
    local = {int(s): list(map(int, e)) for s, e in zip(seq_ids, emitted)}
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return local
    rank = dist.get_rank(group)
    parts = [None] * dist.get_world_size(group) if rank == dst else None
    dist.gather_object(local, parts, dst=dst, group=group)
    if rank != dst:
        return None
    out = {}
    for p in parts:
        if set(p) & set(out):
            raise ValueError("two ranks own the same sequence id")
        out.update(p)
    return out

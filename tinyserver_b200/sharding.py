"""Token sharding across the GPUs of one box.

Every op of the path works per token (row) and every rank stores into its own
KV-cache shard, so a batch splits by contiguous token ranges with no exchange
on the compute path: rank r of P owns tokens ``[r*T//P, (r+1)*T//P)``.  The one
collective is :func:`gather_rows`, an all-gather that assembles the ranks'
outputs (e.g. on rank 0) for validation; it is never on the timed path.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = ["shard_range", "shard_rows", "gather_rows"]


def shard_range(num_tokens: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of rank's contiguous token range (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world or num_tokens < 0:
        raise ValueError(f"bad shard request: {num_tokens} tokens, rank {rank} of {world}")
    return rank * num_tokens // world, (rank + 1) * num_tokens // world


def shard_rows(x: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's rows of a token-major tensor (a view)."""
    s, e = shard_range(x.shape[0], world, rank)
    return x[s:e]


def gather_rows(rows: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather token-major shards of unequal length into the full tensor
    (rank order), on every rank.  Rows must share trailing shape and dtype."""
    world = dist.get_world_size(group)
    n = torch.tensor([rows.shape[0]], dtype=torch.int64, device=rows.device)
    counts = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(counts, n, group=group)
    counts = [int(c) for c in counts]
    cap = max(counts)
    padded = rows.new_zeros((cap, *rows.shape[1:]))
    padded[: rows.shape[0]] = rows
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    return torch.cat([p[:c] for p, c in zip(parts, counts)])

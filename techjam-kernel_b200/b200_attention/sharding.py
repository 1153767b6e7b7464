"""(batch x head) sharding of attention over the GPUs of one node.

Every (batch, head) pair is an independent attention problem, so work is split
without any exchange on the data path: each rank (one process per GPU) runs the
kernel on its own shard.  The only collective is an optional gather of outputs
for validation, outside any timed region.

* ``head_ranges``: contiguous, near-equal head ranges (32 heads over 8 GPUs =
  4 heads per GPU for the long-sequence configuration).
* ``balance_batches``: longest-processing-time assignment of batch entries to
  ranks by cost (for key-padded batches the cost of entry b is L_b^2).
* ``gather_heads``: all-gather of head-sharded [B, h, S, D] outputs into the
  full [B, H, S, D] tensor (NCCL on GPUs, gloo on CPU).
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.distributed as dist


def head_ranges(num_heads: int, world_size: int) -> list[tuple[int, int]]:
    """[lo, hi) head range of every rank; sizes differ by at most one."""
    if num_heads < 1 or world_size < 1:
        raise ValueError("num_heads and world_size must be positive")
    return [((num_heads * r) // world_size, (num_heads * (r + 1)) // world_size)
            for r in range(world_size)]


def balance_batches(costs: Sequence[float], world_size: int) -> list[list[int]]:
    """Assign batch entries to ranks, heaviest first onto the least-loaded rank."""
    if world_size < 1:
        raise ValueError("world_size must be positive")
    loads = [0.0] * world_size
    owners: list[list[int]] = [[] for _ in range(world_size)]
    for b in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        r = min(range(world_size), key=lambda j: (loads[j], j))
        owners[r].append(b)
        loads[r] += costs[b]
    return [sorted(o) for o in owners]


def head_shard(t: torch.Tensor, rank: int, world_size: int) -> torch.Tensor:
    """This rank's heads of a [B, H, S, D] tensor (a view, no copy)."""
    lo, hi = head_ranges(t.shape[1], world_size)[rank]
    return t[:, lo:hi]


def gather_heads(local: torch.Tensor, num_heads: int, world_size: int,
                 group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """All-gather head shards [B, h_r, S, D] into [B, H, S, D] on every rank.

    Shards may differ in size by one head; each is padded to the largest
    shard for the collective and trimmed afterwards."""
    ranges = head_ranges(num_heads, world_size)
    width = max(hi - lo for lo, hi in ranges)
    B, h, S, D = local.shape
    padded = local.new_zeros((B, width, S, D))
    padded[:, :h] = local
    parts = [torch.empty_like(padded) for _ in range(world_size)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    return torch.cat([p[:, :hi - lo] for p, (lo, hi) in zip(parts, ranges)], dim=1)

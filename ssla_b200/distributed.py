"""Multi-GPU use of the hot path: independent samples / sequences are sharded across ranks (one
process per GPU, torch.distributed over NCCL) and only the per-sample detections are exchanged.

The reference trains with Lightning DDP (train.py:86-100) and has no collective on the hot path;
sequences never cross ranks here either (weak scaling for the operators, a batch split for the
model), so the only collective is one all_gather of the head outputs.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


def shard_range(n: int, rank: int, world: int):
    """Contiguous [start, stop) share of `n` items for `rank` (sizes differ by at most one)."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_outputs(x: torch.Tensor, group: Optional["dist.ProcessGroup"] = None) -> torch.Tensor:
    """Concatenate every rank's [b_r, ...] tensor along dim 0 on all ranks (ranks may hold
    different b_r)."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return x
    world = dist.get_world_size(group)
    n = torch.tensor([x.shape[0]], device=x.device, dtype=torch.int64)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(s) for s in sizes]
    m = max(sizes)
    pad = torch.zeros((m,) + tuple(x.shape[1:]), device=x.device, dtype=x.dtype)
    pad[: x.shape[0]] = x
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[:s] for p, s in zip(parts, sizes)], 0)

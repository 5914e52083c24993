"""Data-parallel plumbing: batch sharding across ranks and the output gather.

The path shards by image: rank r of W processes images
[r*B/W, (r+1)*B/W) of a global batch B (weak scaling gives every rank a full
per-GPU batch instead), weights are replicated, and the only collective is one
all-gather of the per-rank outputs per step, in rank order, over the process
group's backend (NCCL over NVLink on GPUs, gloo in the CPU tests).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def shard_range(global_batch: int, rank: int, world: int) -> Tuple[int, int]:
    """[begin, end) of the images rank `rank` owns; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(global_batch, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def gather_outputs(local: torch.Tensor, out: Optional[torch.Tensor] = None,
                   group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """All-gather equal-shaped per-rank outputs along dim 0, in rank order."""
    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out

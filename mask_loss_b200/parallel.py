"""Batch-by-image data parallelism (one process per GPU).

Every cost, assignment and gradient depends on one image only, so ranks own
disjoint image shards and exchange nothing on the data path.  The only
collectives are:

* ``global_num_masks``: all-reduce (SUM) of the per-rank GT count, divided by
  the world size and clamped to >= 1 (the Mask2Former convention, so that
  DDP's gradient averaging reproduces the single-process loss normalised by
  the total GT count);
* ``average_losses``: all-reduce of the (3, L) loss means for reporting.

Both work on any device/backend (NCCL on GPUs, gloo on CPU for tests) and
keep num_masks on the device, so the loss kernels read it without a host
synchronisation.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_images(B_global: int, rank: int, world: int) -> range:
    """Contiguous image shard of this rank: [rank*B/W, (rank+1)*B/W)."""
    lo = (B_global * rank) // world
    hi = (B_global * (rank + 1)) // world
    return range(lo, hi)


def global_num_masks(local_count: torch.Tensor, group=None) -> torch.Tensor:
    """Device scalar: sum over ranks / world, clamped >= 1."""
    nm = local_count.detach().to(torch.float32).reshape(()).clone()
    world = 1
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(nm, group=group)
        world = dist.get_world_size(group)
    return (nm / world).clamp(min=1.0)


def average_losses(losses: torch.Tensor, group=None, async_op: bool = False):
    """All-reduce (mean over ranks) of a loss tensor, in place."""
    if not (dist.is_available() and dist.is_initialized()):
        return None
    world = dist.get_world_size(group)
    losses.div_(world)
    return dist.all_reduce(losses, group=group, async_op=async_op)

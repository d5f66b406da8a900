"""Sample sharding across GPUs (one process per GPU).

Aircraft are independent, so a batch is split into contiguous slices, one
per rank, with no exchange during extraction.  The only cross-rank step is
the final gather of the [n,142] feature slices into host memory of one rank.
"""
from __future__ import annotations

from typing import Tuple

import numpy as np


def shard_range(total: int, rank: int, world: int) -> Tuple[int, int]:
    """(first, count) of rank's contiguous slice; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    first = total * rank // world
    return first, total * (rank + 1) // world - first


def gather_features(local: np.ndarray, total: int, group=None, dst: int = 0):
    """Gather every rank's [count,142] slice into a [total,142] array on `dst`
    (None elsewhere).  Uses torch.distributed on CPU tensors (gloo) or, with an
    NCCL group, on the current CUDA device."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    backend = dist.get_backend(group)
    device = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    counts = [shard_range(total, r, world)[1] for r in range(world)]
    width = local.shape[1]
    biggest = max(counts)
    buf = torch.zeros((biggest, width), dtype=torch.float32, device=device)
    buf[: local.shape[0]] = torch.from_numpy(np.ascontiguousarray(local)).to(device)
    parts = [torch.empty_like(buf) for _ in range(world)] if rank == dst else None
    if backend == "nccl":
        # NCCL has no gather; all_gather keeps every rank on the same collective.
        parts = [torch.empty_like(buf) for _ in range(world)]
        dist.all_gather(parts, buf, group=group)
    else:
        dist.gather(buf, parts, dst=dst, group=group)
    if rank != dst:
        return None
    return np.concatenate([p[:c].cpu().numpy() for p, c in zip(parts, counts)], axis=0)


def max_over_ranks(value: float, group=None) -> float:
    """The largest of every rank's `value` (used for timed regions: a job is as
    slow as its slowest GPU).  Single-process runs return `value`."""
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return value
    device = (torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl"
              else torch.device("cpu"))
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())

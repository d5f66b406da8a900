"""Sample sharding across GPUs (one process per GPU).

Aircraft are independent, so a batch is split into contiguous slices, one
per rank, with no exchange during extraction.  The only cross-rank step is
the final gather of the [n,142] feature slices into host memory, which
SharedHostGather does without any GPU collective: every rank copies its own
slice over its own PCIe link, at the same time as the others, into its offset
of one page-locked buffer that all ranks of the node map.
"""
from __future__ import annotations

import mmap
import os
import uuid
from typing import Tuple

import numpy as np

PAGE = 4096


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


def _multi_rank(group=None) -> bool:
    import torch.distributed as dist

    return dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1


def _reduce_device(group=None):
    import torch
    import torch.distributed as dist

    return (torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl"
            else torch.device("cpu"))


def max_over_ranks_list(values, group=None) -> list:
    """Element-wise max over ranks of a list of floats (per-repetition times)."""
    import torch
    import torch.distributed as dist

    if not _multi_rank(group):
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=_reduce_device(group))
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t.cpu().tolist()


def sum_over_ranks(values, group=None) -> list:
    """Element-wise sum over ranks of a list of integers (checked / mismatch counts)."""
    import torch
    import torch.distributed as dist

    if not _multi_rank(group):
        return [int(v) for v in values]
    t = torch.tensor([int(v) for v in values], dtype=torch.int64, device=_reduce_device(group))
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return [int(v) for v in t.cpu().tolist()]


def all_ranks(value, group=None) -> list:
    """Every rank's (picklable) value, in rank order; [value] on one rank."""
    import torch.distributed as dist

    if not _multi_rank(group):
        return [value]
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, value, group=group)
    return out


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


def _shared_dir(nbytes: int) -> str:
    """/dev/shm when it has room for the buffer (with 10 % to spare), else the
    temporary directory: a mapped file anywhere is shared by the processes
    that map it, and writing past a full tmpfs would kill them (SIGBUS)."""
    import tempfile

    try:
        st = os.statvfs("/dev/shm")
        if st.f_bavail * st.f_frsize >= 1.1 * nbytes:
            return "/dev/shm"
    except OSError:
        pass
    return tempfile.gettempdir()


class SharedHostGather:
    """One host buffer of [total, width] float32 rows shared by all ranks of
    a node (a /dev/shm file, or a temporary-directory file when /dev/shm is
    too small, that every rank maps), with each rank's own rows
    page-locked in its process so that a device-to-host copy lands there
    directly.  gather(slice) copies this rank's [count, width] device rows to
    its offset, asynchronously on `stream`; after a barrier every rank (rank 0
    in particular) reads the whole batch from .array.  No GPU collective and
    no extra copy: each feature byte crosses one PCIe link once.

    Replaces the reference's host-mediated exchange between devices
    (src/gpu/trainer.cu:398-441) for the sample-sharded feature path."""

    def __init__(self, total: int, width: int, group=None, prefix: str = "tb_gather", pin: bool = True):
        import torch
        import torch.distributed as dist

        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.total, self.width = total, width
        self.nbytes = total * width * 4
        name = [os.path.join(_shared_dir(self.nbytes), f"{prefix}_{os.getpid()}_{uuid.uuid4().hex[:12]}")
                if self.rank == 0 else None]
        if self.world > 1:
            dist.broadcast_object_list(name, src=0, group=group)
        self.path = name[0]
        if self.rank == 0:
            fd = os.open(self.path, os.O_CREAT | os.O_EXCL | os.O_RDWR, 0o600)
            os.ftruncate(fd, max(self.nbytes, PAGE))
            os.close(fd)
        if self.world > 1:
            dist.barrier(group=group)
        fd = os.open(self.path, os.O_RDWR)
        try:
            self.map = mmap.mmap(fd, max(self.nbytes, PAGE))
        finally:
            os.close(fd)
        self.array = np.frombuffer(self.map, dtype=np.float32, count=total * width).reshape(total, width)
        self.first, self.count = shard_range(total, self.rank, self.world)
        # page-lock the pages that hold this rank's rows (in this process)
        lo = (self.first * width * 4) // PAGE * PAGE
        hi = min(-(-((self.first + self.count) * width * 4) // PAGE) * PAGE, len(self.map))
        self._base = np.frombuffer(self.map, dtype=np.uint8).ctypes.data
        self._reg = (self._base + lo, hi - lo)
        self.registered = False
        if pin and hi > lo:
            # a refusal (e.g. file pages that the kernel will not pin) leaves the
            # rows pageable: the copy still lands, through the driver's staging
            self.registered = int(torch.cuda.cudart().cudaHostRegister(self._reg[0], self._reg[1], 0)) == 0
        self.mine = torch.from_numpy(self.array[self.first:self.first + self.count])

    def gather(self, device_rows, stream=None) -> None:
        """Enqueue the copy of this rank's device rows into the shared buffer
        (asynchronous on `stream`; synchronise it before reading)."""
        import torch

        if self.count == 0:
            return
        if not isinstance(device_rows, torch.Tensor):
            device_rows = torch.from_numpy(np.ascontiguousarray(device_rows))
        if stream is None:
            self.mine.copy_(device_rows, non_blocking=True)
        else:
            with torch.cuda.stream(stream):
                self.mine.copy_(device_rows, non_blocking=True)

    def close(self, group=None) -> None:
        import torch
        import torch.distributed as dist

        if self.registered:
            torch.cuda.cudart().cudaHostUnregister(self._reg[0])
            self.registered = False
        self.mine = None
        self.array = None
        try:
            self.map.close()
        except BufferError:  # a view of the buffer is still alive somewhere
            pass
        if self.world > 1:
            dist.barrier(group=group)  # every rank has unmapped before the file goes
        if self.rank == 0:
            try:
                os.unlink(self.path)
            except FileNotFoundError:
                pass

"""Multi-rank host logic on CPU (gloo, world size 2): each rank generates and
reduces its own contiguous slice, the slices gather into the full batch, and
the timing reduction takes the slowest rank.  The per-rank reduction here is
the CPU oracle, standing in for the GPU so the test runs without one."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from turbinator_c_b200.shard import shard_range


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, total, seed, stress, result_path):
    import datetime

    import torch.distributed as dist

    import oracle
    import turbinator_c_b200 as tb
    from turbinator_c_b200.shard import gather_features, max_over_ranks

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        first, count = shard_range(total, rank, world)
        obs, mission, cams, _ = tb.generate(seed, first, count, total=total, stress=stress, threads=2)
        local = oracle.features(obs, mission, cams, threads=2)
        full = gather_features(local, total)
        slowest = max_over_ranks(float(rank + 1))
        if rank == 0:
            np.save(result_path, full)
            with open(result_path + ".max", "w") as f:
                f.write(repr(slowest))
    finally:
        dist.destroy_process_group()


def test_shard_range_partitions():
    for total in (0, 1, 7, 8, 1000, 524288):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(total, r, world) for r in range(world)]
            assert sum(c for _, c in spans) == total
            assert all(spans[i][0] + spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


@pytest.mark.parametrize("total,stress", [(37, False), (64, True)])
def test_two_rank_gather_matches_single_process(tmp_path, total, stress):
    import oracle
    import turbinator_c_b200 as tb

    path = str(tmp_path / "gathered.npy")
    mp.spawn(_worker, args=(2, _free_port(), total, 9, stress, path), nprocs=2, join=True)
    gathered = np.load(path)
    obs, mission, cams, _ = tb.generate(9, 0, total, stress=stress)
    expected = oracle.features(obs, mission, cams)
    assert np.array_equal(gathered.view(np.uint32), expected.view(np.uint32))
    assert float(open(path + ".max").read()) == 2.0


def _gather_worker(rank, world, port, total, result_path):
    import datetime

    import torch
    import torch.distributed as dist

    from turbinator_c_b200.shard import SharedHostGather, all_ranks, max_over_ranks_list, sum_over_ranks

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        g = SharedHostGather(total, 142, pin=False)   # no GPU here: plain host copies into the shared file
        first, count = shard_range(total, rank, world)
        rows = np.arange(first * 142, (first + count) * 142, dtype=np.float32).reshape(count, 142)
        g.gather(torch.from_numpy(rows))
        dist.barrier()
        ok = rank != 0 or np.array_equal(g.array, np.arange(total * 142, dtype=np.float32).reshape(total, 142))
        maxes = max_over_ranks_list([rank, -rank])
        sums = sum_over_ranks([1, rank])
        everyone = all_ranks({"rank": rank})
        g.close()
        if rank == 0:
            with open(result_path, "w") as f:
                f.write(repr((bool(ok), maxes, sums, [e["rank"] for e in everyone], os.path.exists(g.path))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,total", [(2, 37), (3, 1000)])
def test_shared_host_gather_assembles_every_slice(tmp_path, world, total):
    """Each rank writes its own slice into the shared host buffer at its
    offset; rank 0 then reads the whole batch.  The reductions used by the
    benchmark's timing and parity counts work over the same ranks, and the
    shared file is removed on close."""
    path = str(tmp_path / "gather.txt")
    mp.spawn(_gather_worker, args=(world, _free_port(), total, path), nprocs=world, join=True)
    ok, maxes, sums, ranks, left = eval(open(path).read())
    assert ok
    assert maxes == [world - 1.0, 0.0]
    assert sums == [world, sum(range(world))]
    assert ranks == list(range(world))
    assert not left

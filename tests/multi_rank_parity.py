"""Config-3 and config-4 parity across ranks (run by tests/test_multi_rank_gpu.py
under torchrun, one process per GPU, NCCL):

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P tests/multi_rank_parity.py [total [config3|config4]]

Config 4 (seed 4, 131,072 aircraft in four stress quarters) is checked in
full: every rank compares its whole shard with the CPU oracle.

BASELINE config 3 is seed 3 and 524,288 aircraft split into contiguous
slices of B/N.  Each rank generates only its own slice, extracts it on its
GPU through tb_cuda_extract_features_device, and copies its device slice into
one page-locked host buffer shared by all ranks (shard.SharedHostGather, the
library's gather: no GPU collective).  Rank 0 checks the strided subsample -- every
97th aircraft plus the first and last aircraft of every shard -- against the
CPU oracle on inputs regenerated for just those indices (the generator is
keyed by (seed, aircraft index), so any index can be rebuilt alone).  Every
rank exits 0 on success, 1 on a mismatch.
"""
from __future__ import annotations

import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import oracle  # noqa: E402
import turbinator_c_b200 as tb  # noqa: E402
from tests.parity import check_features  # noqa: E402
from turbinator_c_b200.shard import SharedHostGather, shard_range  # noqa: E402

SEEDS = {"config3": 3, "config4": 4}


def main() -> int:
    total = int(sys.argv[1]) if len(sys.argv) > 1 else 524288
    mode = sys.argv[2] if len(sys.argv) > 2 else "config3"
    seed, stress = SEEDS[mode], mode == "config4"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    ok = True
    try:
        first, count = shard_range(total, rank, world)
        obs, mission, cams, _ = tb.generate(seed, first, count, total=total, stress=stress)
        d = [torch.from_numpy(x).cuda() for x in (obs, mission, cams)]
        out = torch.empty((count, 142), device="cuda")
        assert tb.tb_cuda_extract_features_device(*d, out, count, None) == 1
        assert tb.tb_cuda_synchronize(None) == 1
        mine = out.cpu().numpy()
        if stress:
            try:
                check_features(mine, oracle.features(obs, mission, cams), f"config 4 rank {rank} of {world}")
                print(f"config 4: rank {rank} of {world}, all {count} aircraft match the oracle")
            except AssertionError as e:
                print(f"config 4 mismatch on rank {rank}: {e}")
                ok = False
        gatherer = SharedHostGather(total, 142)
        gatherer.gather(out)
        torch.cuda.synchronize()
        dist.barrier()
        full = gatherer.array
        if not np.array_equal(full[first:first + count].view(np.uint32), mine.view(np.uint32)):
            print(f"gather mismatch on rank {rank}")
            ok = False
        if rank == 0 and not stress:
            idx = set(range(0, total, 97))
            for r in range(world):
                f, c = shard_range(total, r, world)
                idx.update((f, f + c - 1))
            idx = np.array(sorted(idx))
            rows = [tb.generate(seed, int(i), 1, total=total) for i in idx]
            o = np.concatenate([r[0] for r in rows])
            m = np.concatenate([r[1] for r in rows])
            cam = np.concatenate([r[2] for r in rows])
            try:
                check_features(full[idx], oracle.features(o, m, cam), f"config 3 over {world} GPUs")
                print(f"config 3: {total} aircraft over {world} GPUs, {len(idx)} sampled aircraft match the oracle")
            except AssertionError as e:
                print(f"config 3 mismatch: {e}")
                ok = False
        full = None
        gatherer.close()
        flag = torch.tensor([1 if ok else 0], device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = bool(flag.item())
    finally:
        dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())

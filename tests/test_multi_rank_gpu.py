"""BASELINE config 3 across every visible GPU, one process per GPU (torchrun,
NCCL): contiguous shards extracted on their own GPUs, gathered to rank 0 and
checked on the strided subsample (every 97th aircraft plus each shard's first
and last) against the CPU oracle.  The ranks run tests/multi_rank_parity.py;
the process group has a 120 s timeout and the whole run a 600 s limit."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(total: int, mode: str, port_offset: int):
    n = min(torch.cuda.device_count(), 8)
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1",
           "--master-port", str(29600 + port_offset + os.getpid() % 100),
           os.path.join(ROOT, "tests", "multi_rank_parity.py"), str(total), mode]
    run = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
    print(run.stdout[-2000:])
    assert run.returncode == 0, run.stdout[-4000:] + run.stderr[-4000:]
    assert "match the oracle" in run.stdout
    return run.stdout


def test_config3_parity_across_ranks():
    _run(524288, "config3", 0)


def test_config4_full_parity_across_ranks():
    out = _run(131072, "config4", 100)
    assert out.count("all ") >= 1

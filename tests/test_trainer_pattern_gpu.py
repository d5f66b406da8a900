"""The reference trainer's feature call pattern (src/trainer/main.c:511-699)
on real simulator observations, through this library's host ABI.

oracle/_ref/trainer_pattern (built by oracle/Makefile from
oracle/trainer_pattern.c and the reference's simulator and training.c) steps
the simulator with its reference controller and checks every extracted batch
against the reference CPU path.  Its dumped batches -- real LiDAR with
dropouts, ray-traced cameras, arena missions -- also drive the onboard kernel
against the reference onboard header."""
from __future__ import annotations

import os
import re
import subprocess

import numpy as np
import pytest

import oracle
import turbinator_c_b200 as tb

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DRIVER = os.path.join(ROOT, "oracle", "_ref", "trainer_pattern")
needs_driver = pytest.mark.skipif(not os.path.exists(DRIVER), reason="trainer-pattern driver not built")


def run_driver(batch, steps, seed, *extra, batched=False, pinned=False, timing=False):
    env = dict(os.environ, TB_PATTERN_BATCHED="1" if batched else "0", TB_PATTERN_PINNED="1" if pinned else "0")
    r = subprocess.run([DRIVER, "0", str(batch), str(steps), str(seed), *map(str, extra)],
                       capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    m = re.search(r"calls=(\d+) samples=(\d+) failures=(\d+) exact_mismatches=(\d+) lidar_over_tol=(\d+)",
                  r.stdout)
    assert m, r.stdout
    calls, samples, failures, exact, over = map(int, m.groups())
    assert failures == 0 and exact == 0 and over == 0
    if timing:
        return calls, samples, float(re.search(r"extract_ms=([0-9.]+)", r.stdout).group(1))
    return calls, samples


@needs_driver
def test_trainer_default_scale():
    calls, samples = run_driver(32, 64, 7)
    assert calls >= 65 and samples >= 65 * 32


@needs_driver
@pytest.mark.parametrize("batch", [8, 256])
def test_batched_trainer_calls(batch):
    """The same episode with next, post-reset and next-step opponent
    observations written into one buffer and extracted in one call per step
    (pageable, then page-locked): the same rows, all matching the reference CPU
    path, in fewer calls.  Prints the three extraction times."""
    calls, samples, ms = run_driver(batch, 96, 5, timing=True)
    b_calls, b_samples, b_ms = run_driver(batch, 96, 5, batched=True, timing=True)
    p_calls, p_samples, p_ms = run_driver(batch, 96, 5, batched=True, pinned=True, timing=True)
    print(f"\ntrainer pattern, batch {batch}, 96 steps: {calls} calls {ms:.1f} ms; batched {b_calls} calls "
          f"{b_ms:.1f} ms; batched into page-locked rows {p_calls} calls {p_ms:.1f} ms")
    assert b_samples == samples == p_samples
    assert b_calls < calls and p_calls == b_calls
    assert p_ms < ms  # measured 1.9x (batch 8) and 4.0x (batch 256) less time in extraction


def read_dump(path):
    batches = []
    with open(path, "rb") as f:
        while True:
            head = f.read(4)
            if not head:
                break
            n = int(np.frombuffer(head, np.int32)[0])
            obs = np.frombuffer(f.read(n * 4148 * 4), np.float32).reshape(n, 4148).copy()
            mission = np.frombuffer(f.read(n * 10 * 4), np.float32).reshape(n, 10).copy()
            cams = np.frombuffer(f.read(n * 16384), np.uint8).reshape(n, 16384).copy()
            batches.append((obs, mission, cams))
    return batches


@needs_driver
def test_reference_max_batch_and_onboard_on_simulated_observations(tmp_path):
    dump = tmp_path / "batches.bin"
    run_driver(1024, 4, 11, dump, 3)
    batches = read_dump(dump)
    assert len(batches) == 3
    for obs, mission, _ in batches:
        n = obs.shape[0]
        d_obs = torch.from_numpy(obs).cuda()
        d_mis = torch.from_numpy(mission).cuda()
        tac = torch.empty((n, 24), device="cuda")
        pri = torch.empty((n, 15), device="cuda")
        assert tb.tb_cuda_extract_onboard_device(d_obs, d_mis, tac, pri, n) == 1
        torch.cuda.synchronize()
        gpu = np.concatenate([tac.cpu().numpy(), pri.cpu().numpy()], axis=1)
        cr = oracle.onboard_reference_cr(obs, mission)
        ref = oracle.onboard_reference(obs, mission)
        assert np.array_equal(gpu, cr)
        assert np.max(np.abs(gpu.astype(np.float64) - ref)) <= 5e-5
        for c in (11, 22, 38):
            assert np.array_equal(gpu[:, c], ref[:, c])

"""The allocation-free host entry point, checked against the handle-based one.

tb_cuda_extract_features_host_noalloc serves callers that cannot allocate
device memory (an onboard control loop that forbids allocation once running,
or a process whose GPU memory a learner's pool already holds).  It stages rows
through a fixed array the library reserves on each GPU, so the array is shared
by consecutive calls: two calls in a row, with different batches, must each
match tb_cuda_extract_features_host.  The first call in a fresh process also
performs the one-time address look-up.  This file is collected last so a
failure here does not stop the other GPU tests from running first.
"""
from __future__ import annotations

import numpy as np
import pytest

import turbinator_c_b200 as tb
from tests.parity import check_features

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _batch(seed, n):
    obs, mission, cams, _ = tb.generate(seed, 0, n)
    return obs, mission, cams


def test_noalloc_entry_matches_host_entry_on_two_calls_in_a_row():
    torch.cuda.set_device(0)
    first = _batch(31, 48)
    second = _batch(32, tb.NOALLOC_MAX_BATCH)

    out1 = np.full((48, 142), np.nan, np.float32)
    out2 = np.full((tb.NOALLOC_MAX_BATCH, 142), np.nan, np.float32)
    assert tb.tb_cuda_extract_features_host_noalloc(*first, 48, out1) == 1
    free_before, _ = torch.cuda.mem_get_info()
    assert tb.tb_cuda_extract_features_host_noalloc(*second, tb.NOALLOC_MAX_BATCH, out2) == 1
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before, "the second call changed free device memory"

    with tb.FeatureBatch(0, tb.NOALLOC_MAX_BATCH) as fb:
        exp1 = np.zeros((48, 142), np.float32)
        exp2 = np.zeros((tb.NOALLOC_MAX_BATCH, 142), np.float32)
        assert fb.extract(*first, 48, exp1) == 1, fb.error()
        assert fb.extract(*second, tb.NOALLOC_MAX_BATCH, exp2) == 1, fb.error()
    check_features(out1, exp1, "no-alloc call 1")
    check_features(out2, exp2, "no-alloc call 2")


def test_noalloc_entry_rejects_sizes_beyond_its_maximum():
    obs, mission, cams = _batch(33, tb.NOALLOC_MAX_BATCH + 1)
    out = np.zeros((tb.NOALLOC_MAX_BATCH + 1, 142), np.float32)
    assert tb.tb_cuda_extract_features_host_noalloc(obs, mission, cams, tb.NOALLOC_MAX_BATCH + 1, out) == -1
    assert tb.tb_cuda_extract_features_host_noalloc(obs, mission, cams, 0, out) == -1
    assert not out.any()
    assert tb.tb_cuda_extract_features_host_noalloc(obs, mission, None, 4, out) == 0


_FIRST_CALL = r"""
import sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
import turbinator_c_b200 as tb
torch.cuda.set_device(0)
torch.cuda.init()
obs, mission, cams, _ = tb.generate(34, 0, 8)
out = np.zeros((8, 142), np.float32)
torch.cuda.synchronize()
before, _ = torch.cuda.mem_get_info()
assert tb.tb_cuda_extract_features_host_noalloc(obs, mission, cams, 8, out) == 1
after_first, _ = torch.cuda.mem_get_info()
assert tb.tb_cuda_extract_features_host_noalloc(obs, mission, cams, 8, out) == 1
after_second, _ = torch.cuda.mem_get_info()
print(before - after_first, after_first - after_second)
"""


def test_first_call_in_a_fresh_process_reserves_the_array():
    """Modules load lazily: in a fresh process the first call on a device is
    what reserves the fixed array (and the kernels' code) there, which is why
    callers make it at start-up; the next call reserves nothing."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    run = subprocess.run([sys.executable, "-c", _FIRST_CALL, root], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stderr[-2000:]
    first, second = (int(v) for v in run.stdout.split()[-2:])
    print(f"first no-alloc call reserved {first} bytes of device memory; the second {second}")
    assert first >= 2_149_376, first   # at least the staging array
    assert second == 0, second

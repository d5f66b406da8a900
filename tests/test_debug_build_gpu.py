"""The feature kernels built with TB_FEATURES_DEBUG (every global load and
store index checked against its buffer, violations reported in the stream's
status word instead of trapping): the stand-in for compute-sanitizer's
memcheck together with tests/test_guard_bands_gpu.py.  The debug library is
loaded in its own process (tests/debug_build_cases.py)."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

import turbinator_c_b200 as tb

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_debug_build_reports_no_out_of_bounds_index():
    assert os.path.exists(tb.DEBUG_LIB_PATH), "build the library first (make -C turbinator_c_b200/csrc)"
    env = dict(os.environ, TB_CUDA_LIBRARY=tb.DEBUG_LIB_PATH)
    run = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "debug_build_cases.py")], env=env,
                         capture_output=True, text=True, timeout=600)
    print(run.stdout[-1000:])
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-3000:]
    assert "no index outside its buffer" in run.stdout

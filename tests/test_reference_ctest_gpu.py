"""The reference's own CUDA parity test (tests/test_cuda_features.c), compiled
unchanged against this repository's include/turbinator/training/cuda_features.h
and libturbinator_cuda.so by oracle/Makefile, must pass: that is the drop-in
contract at the C level."""
from __future__ import annotations

import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BINARY = os.path.join(ROOT, "oracle", "_ref", "test_cuda_features")


@pytest.mark.skipif(not os.path.exists(BINARY), reason="reference test binary not built (no reference tree)")
def test_reference_cuda_feature_test_passes_against_this_library():
    env = dict(os.environ, TB_CUDA_TEST_DEVICE="0")
    r = subprocess.run([BINARY], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "CUDA feature batch matches C11 extraction" in r.stdout

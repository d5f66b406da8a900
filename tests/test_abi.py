"""The C-ABI library loads, exports every symbol the public headers declare,
and rejects bad arguments before touching a device (runs without a GPU)."""
from __future__ import annotations

import ctypes
import glob
import os
import re

import turbinator_c_b200 as tb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = set()
    for header in glob.glob(os.path.join(ROOT, "include", "**", "*.h"), recursive=True):
        text = open(header).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(tb_\w+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(tb.LIB_PATH)
    names = _declared_functions()
    assert {"tb_cuda_extract_features_device", "tb_cuda_synchronize", "tb_cuda_feature_batch_create",
            "tb_cuda_feature_batch_destroy", "tb_cuda_feature_batch_error",
            "tb_cuda_extract_features_host"} <= names
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_argument_rejection_without_device():
    fake = 0x10000  # never dereferenced: every call below is rejected first
    assert tb.tb_cuda_extract_features_device(None, fake, fake, fake, 4) == 0
    assert tb.tb_cuda_extract_features_device(fake, None, fake, fake, 4) == 0
    assert tb.tb_cuda_extract_features_device(fake, fake, fake, None, 4) == 0
    assert tb.tb_cuda_extract_features_device(fake, fake, fake, fake, 0) == 0
    assert tb.tb_cuda_extract_features_device(fake, fake, fake, fake, 0x80000000) == 0
    assert tb.tb_cuda_extract_features_device(fake + 2, fake, fake, fake, 4) == 0  # misaligned float*
    assert tb.tb_cuda_feature_batch_error(None) == "CUDA feature batch unavailable"
    assert tb.tb_cuda_extract_features_host(None, fake, fake, fake, 1, fake) == 0
    assert tb.tb_cuda_feature_batch_create(0, 0) is None
    tb.tb_cuda_feature_batch_destroy(None)  # NULL-safe
    sharded = tb.tb_cuda_extract_features_device_sharded
    assert sharded([], [], [], None, [], []) == 0                       # no shards
    assert sharded([0] * 65, [fake] * 65, [fake] * 65, None, [fake] * 65, [1] * 65) == 0  # too many
    lib = tb.load_library()
    assert lib.tb_cuda_extract_features_device_sharded(1, None, None, None, None, None, None, None) == 0
    from turbinator_c_b200.sensors import tb_cuda_render_sensors_device as render
    assert render(None, 4, fake, 4096, fake, 2, fake) == 0
    assert render(fake, 0, fake, 4096, fake, 2, fake) == 0
    assert render(fake, 0x80000000, fake, 4096, fake, 2, fake) == 0
    assert render(fake + 4, 4, fake, 4096, fake, 2, fake) == 0        # scenes not 8-byte aligned
    assert render(fake, 4, fake, 4095, fake, 2, fake) == 0            # LiDAR stride below 4096
    assert render(fake, 4, fake, 4096, fake, 1, fake) == 0            # valid stride below 2
    assert render(fake, 4, fake + 2, 4096, fake, 2, fake) == 0        # misaligned LiDAR
    assert render(fake, 4, fake, 4096, fake, 2, fake + 1) == 0        # misaligned cameras
    assert render(fake, 4, fake, 4096, fake, 2, fake, fake + 2) == 0  # misaligned raw capture


def test_library_is_sm100a_only_build():
    """The build recipe targets sm_100a alone (no PTX for JIT, no other arch)."""
    mk = open(os.path.join(ROOT, "turbinator_c_b200", "csrc", "Makefile")).read()
    assert "arch=compute_100a,code=sm_100a" in mk
    assert not re.search(r"sm_(?!100a)\d+", mk)

"""Runs the feature kernels of the bounds-checked debug library
(libturbinator_cuda_debug.so, TB_FEATURES_DEBUG) over every launch shape the
product uses and checks, after each launch, that no index fell outside its
buffer (no TB_FEATURE_STATUS_BOUNDS bit in the stream's status word) and that
the features match the CPU oracle.  Started by tests/test_debug_build_gpu.py
in its own process with TB_CUDA_LIBRARY pointing at the debug library."""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

import oracle  # noqa: E402
import turbinator_c_b200 as tb  # noqa: E402
from tests.parity import check_features  # noqa: E402

BOUNDS = 2  # TB_FEATURE_STATUS_BOUNDS


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run(what, obs, mission, cams, launch, expected):
    n = obs.shape[0]
    out = torch.full((n, 142), float("nan"), device="cuda")
    torch.cuda.synchronize()
    assert launch(out) == 1, what
    torch.cuda.synchronize()
    status = tb.take_status()
    assert status & BOUNDS == 0, f"{what}: an index fell outside its buffer"
    assert status == 0, f"{what}: status {status}"
    check_features(out.cpu().numpy(), expected, what)


def main() -> int:
    assert tb.LIB_PATH.endswith("libturbinator_cuda_debug.so"), tb.LIB_PATH
    tb.load_library()
    with open("/proc/self/maps") as f:
        assert "libturbinator_cuda_debug.so" in f.read(), "debug library not loaded"
    torch.cuda.set_device(0)
    cases = 0
    for n in (1, 3, 297, 2369, 9001):
        obs, mission, cams, camf = tb.generate(51, 0, n, f32_cameras=True)
        exp = oracle.features(obs, mission, cams)
        d_obs, d_mis, d_cam, d_camf = dev(obs), dev(mission), dev(cams), dev(camf)
        for name, kw in (("flat", {}), ("staged", {"flat": -1}), ("direct", {"force_direct": True})):
            run(f"{name} B={n}", obs, mission, cams,
                lambda out, kw=kw: tb.launch(d_obs, d_mis, d_cam, out, n, None, **kw), exp)
            cases += 1
        run(f"flat no cameras B={n}", obs, mission, None,
            lambda out: tb.launch(d_obs, d_mis, None, out, n, None), oracle.features(obs, mission, None))
        for direct in (False, True):
            run(f"f32cam direct={direct} B={n}", obs, mission, cams,
                lambda out, direct=direct: tb.launch_f32cam(d_obs, d_mis, d_camf, out, n, force_direct=direct), exp)
        cases += 3
        if n in (297, 2369):
            for g in (1, 5):
                run(f"staged grid={g} B={n}", obs, mission, cams,
                    lambda out, g=g: tb.launch(d_obs, d_mis, d_cam, out, n, None, grid_limit=g), exp)
                cases += 1
            # input rows 4 bytes past a 16-byte boundary (the plain-load kernel)
            flat_obs = torch.zeros(n * 4148 + 1, device="cuda")
            flat_obs[1:] = d_obs.reshape(-1)
            run(f"unaligned B={n}", obs, mission, cams,
                lambda out: tb.tb_cuda_extract_features_device(flat_obs.data_ptr() + 4, d_mis, d_cam, out, n), exp)
            host = np.zeros((n, 142), np.float32)
            with tb.FeatureBatch(0, n) as fb:
                assert fb.extract(obs, mission, cams, n, host) == 1, fb.error()
            assert tb.take_status() == 0
            check_features(host, exp, f"host ABI B={n}")
            cases += 2
    print(f"debug build: {cases} launches, no index outside its buffer, all features match the oracle")
    return 0


if __name__ == "__main__":
    sys.exit(main())

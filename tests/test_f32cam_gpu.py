"""GPU parity of the FP32-camera entry point
(tb_cuda_extract_features_device_f32cam): features must equal the reference
CPU path fed the bytes that the simulator's quantisation rule
(src/sim/sensors.c:67) makes of the same float cameras -- bit-exact for the
camera, scalar and mission features, 1e-6 + 1e-5*|ref| for LiDAR means."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import turbinator_c_b200 as tb
from tests.parity import check_features

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def run_f32(obs, mission, camf, **opts):
    n = obs.shape[0]
    d = [torch.from_numpy(np.ascontiguousarray(x)).cuda() if x is not None else None for x in (obs, mission, camf)]
    out = torch.full((n, 142), float("nan"), device="cuda")
    torch.cuda.synchronize()
    if opts:
        assert tb.launch_f32cam(d[0], d[1], d[2], out, n, None, **opts) == 1
    else:
        assert tb.tb_cuda_extract_features_device_f32cam(d[0], d[1], d[2], out, n) == 1
    assert tb.tb_cuda_synchronize() == 1
    return out.cpu().numpy()


def expected(obs, mission, camf):
    cams = oracle.quantize_cameras(camf) if camf is not None else None
    return oracle.features(obs, mission, cams)


@pytest.mark.parametrize("config", [0, 1, 2])
def test_configs(config):
    seed, batch, _ = tb.CONFIGS[config]
    obs, mission, cams, camf = tb.generate(seed, 0, batch, f32_cameras=True)
    assert np.array_equal(oracle.quantize_cameras(camf), cams)
    out = run_f32(obs, mission, camf)
    check_features(out, expected(obs, mission, camf), f"f32 config{config}")


def test_config4_stress():
    seed, batch, _ = tb.CONFIGS[4]
    obs, mission, _, camf = tb.generate(seed, 0, batch, stress=True, f32_cameras=True)
    check_features(run_f32(obs, mission, camf), expected(obs, mission, camf), "f32 config4")


def _boundary_values():
    """Floats within a few ulps of every rounding boundary (k + 0.5)/255, the
    extremes and the non-finite values."""
    vals = []
    for k in range(256):
        c = np.float32((k + 0.5) / 255.0)
        v = c
        for _ in range(4):
            v = np.nextafter(v, np.float32(-1))
        for _ in range(9):
            vals.append(v)
            v = np.nextafter(v, np.float32(2))
        vals.append(np.float32(k / 255.0))
    vals += [np.nan, -np.nan, np.inf, -np.inf, -0.0, 0.0, 1e-45, -1e-45, 1.0, np.nextafter(np.float32(1), np.float32(2)),
             2.0, 1e30, -1e30, -0.5, 0.99999994]
    return np.array(vals, np.float32)


def test_quantisation_boundaries():
    vals = _boundary_values()
    rng = np.random.default_rng(3)
    n = 8
    obs, mission, _, _ = tb.generate(5, 0, n)
    camf = rng.choice(vals, size=(n, 16384)).astype(np.float32)
    camf[0, : vals.size] = vals                      # every value at least once
    out = run_f32(obs, mission, camf)
    check_features(out, expected(obs, mission, camf), "f32 boundaries")
    check_features(run_f32(obs, mission, camf, force_direct=True), expected(obs, mission, camf),
                   "f32 boundaries/direct")


def test_null_cameras_and_ragged_and_few_ctas():
    obs, mission, _, camf = tb.generate(6, 0, 301, f32_cameras=True)
    check_features(run_f32(obs, mission, None), expected(obs, mission, None), "f32 no camera")
    check_features(run_f32(obs, mission, camf, grid_limit=3), expected(obs, mission, camf), "f32 grid=3")
    check_features(run_f32(obs[:1], mission[:1], camf[:1]), expected(obs[:1], mission[:1], camf[:1]), "f32 B=1")


def test_unaligned_rows_take_the_direct_kernel():
    obs, mission, _, camf = tb.generate(7, 0, 64, f32_cameras=True)
    n = 64
    flat = torch.zeros(n * 16384 + 1, device="cuda")
    flat[1:] = torch.from_numpy(camf).cuda().reshape(-1)
    out = torch.zeros((n, 142), device="cuda")
    d_obs, d_mis = torch.from_numpy(obs).cuda(), torch.from_numpy(mission).cuda()
    assert tb.tb_cuda_extract_features_device_f32cam(d_obs, d_mis, flat.data_ptr() + 4, out, n) == 1
    assert tb.tb_cuda_synchronize() == 1
    check_features(out.cpu().numpy(), expected(obs, mission, camf), "f32 unaligned")

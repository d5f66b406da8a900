"""GPU sensor rendering (tb_cuda_render_sensors_device) against the reference
simulator's own renderers, through the C ABI.

Bar: LiDAR ranges and valid fractions bit for bit, camera and raw-capture
bytes equal.  Expected values come from the committed golden renders (made by
the reference's tb_sim_render_lidar / tb_sim_render_camera) and, when the
reference simulator build travels with the tree (oracle/_ref), from the
reference renderers run live on the same scenes: synthetic flight and
heaviest-case scenes, hand-built edge cases, and scenes packed from simulated
episodes.  Also covered: writing straight into observation rows (strides),
the per-scene sensor mask and NULL outputs (nothing else written), a
non-default stream, and a 65,536-scene batch (sampled against the reference,
and rendered twice with identical bytes).
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle
from tests.sensor_cases import bits_equal, edge_scenes, random_scenes
from turbinator_c_b200.sensors import SCENE_DTYPE, synthetic_scenes, tb_cuda_render_sensors_device

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sensors_reference.npz")
needs_reference = pytest.mark.skipif(not oracle.have_reference_sensors(),
                                     reason="reference simulator build (oracle/_ref) not available")
DEV = "cuda:0"


def _scenes_to_device(scenes):
    raw = np.ascontiguousarray(scenes).view(np.uint8).reshape(-1)
    return torch.from_numpy(raw.copy()).to(DEV)


def render_gpu(scenes, raw=False, stream=None):
    n = len(scenes)
    d_scenes = _scenes_to_device(scenes)
    lidar = torch.full((n, 4096), float("nan"), device=DEV)
    valid = torch.full((n, 2), float("nan"), device=DEV)
    cams = torch.zeros((n, 16384), dtype=torch.uint8, device=DEV)
    raws = torch.zeros((n, 147456), dtype=torch.uint8, device=DEV) if raw else None
    ok = tb_cuda_render_sensors_device(d_scenes, n, lidar, 4096, valid, 2, cams, raws, stream)
    assert ok == 1
    torch.cuda.synchronize()
    return (lidar.cpu().numpy(), valid.cpu().numpy(), cams.cpu().numpy(),
            raws.cpu().numpy() if raw else None)


def assert_same(got, want, what):
    lidar, valid, cams, raw = got
    rl, rv, rc, rr = want
    bad = ~bits_equal(lidar, rl)
    assert not bad.any(), (f"{what}: LiDAR differs in {bad.sum()} bins; first {np.argwhere(bad)[:4].tolist()} "
                           f"gpu {lidar[bad][:4]} ref {rl[bad][:4]}")
    assert bits_equal(valid, rv).all(), f"{what}: valid fractions differ"
    bad = cams != rc
    assert not bad.any(), (f"{what}: camera differs in {bad.sum()} pixels; first {np.argwhere(bad)[:4].tolist()} "
                           f"gpu {cams[bad][:4]} ref {rc[bad][:4]}")
    if raw is not None and rr is not None:
        assert np.array_equal(raw, rr), f"{what}: raw capture differs"


def test_golden_reference_renders():
    g = np.load(GOLDEN)
    scenes = g["scenes"].view(SCENE_DTYPE).reshape(-1)
    lidar, valid, cams, raw = render_gpu(scenes, raw=True)
    n_raw = g["raw"].shape[0]
    assert_same((lidar, valid, cams, raw[:n_raw]), (g["lidar"], g["valid"], g["cameras"], g["raw"]), "golden")


@needs_reference
@pytest.mark.parametrize("kind", ["flight", "max"])
def test_synthetic_scenes_match_reference(kind):
    scenes = synthetic_scenes(7 + len(kind), 512, balls=kind)
    assert_same(render_gpu(scenes, raw=True), oracle.render_sensors_reference(scenes, raw=True), kind)


@needs_reference
def test_edge_cases_match_reference():
    scenes = edge_scenes()
    assert_same(render_gpu(scenes, raw=True), oracle.render_sensors_reference(scenes, raw=True), "edge")


@needs_reference
@pytest.mark.parametrize("unit", [True, False])
def test_adversarial_random_scenes_match_reference(unit):
    """Spheres at random directions and distances around the sensors (some
    enclosing them, some grazing the units' cones), random attitudes, any
    scenario, sky distance and dome: the cases the exact culling must get
    right.  Non-unit attitudes turn culling off and exercise the full path."""
    scenes = random_scenes(1234 + unit, 2048, unit_attitude=unit)
    want = oracle.render_sensors_reference(scenes)
    assert_same(render_gpu(scenes), (want[0], want[1], want[2], None), f"random unit={unit}")


@needs_reference
def test_simulated_episodes_match_environment_renders():
    n = 224
    idx = np.arange(n)
    scenes, lidar, valid, cams = oracle.simulate_sensor_scenes(idx % 28, idx * 7 + 3, (idx * 97) % 900, idx % 2,
                                                               SCENE_DTYPE)
    assert scenes["ball_count"].max() > 0
    assert_same(render_gpu(scenes), (lidar, valid, cams, None), "simulated")


def test_writes_into_observation_rows():
    """lidar = obs + 48 (stride 4148), valid = obs + 4146: the observation
    layout of tb_sim_observe (sensors.c:117-119); nothing else changes."""
    g = np.load(GOLDEN)
    scenes = g["scenes"].view(SCENE_DTYPE).reshape(-1)
    scenes = scenes[scenes["sensors"] & 1 == 1]
    n = len(scenes)
    obs = torch.full((n, 4148), 123.5, device=DEV)
    cams = torch.zeros((n, 16384), dtype=torch.uint8, device=DEV)
    d = _scenes_to_device(scenes)
    lidar_view, valid_view = obs[:, 48:], obs[:, 4146:]
    assert tb_cuda_render_sensors_device(d, n, lidar_view, 4148, valid_view, 4148, cams) == 1
    torch.cuda.synchronize()
    o = obs.cpu().numpy()
    keep = np.r_[0:48, 4144:4146]
    assert (o[:, keep] == 123.5).all()
    want = oracle.render_sensors_port(scenes)
    assert bits_equal(o[:, 48:4144], want[0]).all()
    assert bits_equal(o[:, 4146:4148], want[1]).all()
    assert np.array_equal(cams.cpu().numpy(), want[2])


def test_sensor_mask_and_null_outputs():
    base = synthetic_scenes(3, 8)
    base["sensors"] = [0, 1, 2, 3, 3, 2, 1, 0]
    want = oracle.render_sensors_port(base)
    n = len(base)
    d = _scenes_to_device(base)
    lidar = torch.full((n, 4096), -7.0, device=DEV)
    valid = torch.full((n, 2), -7.0, device=DEV)
    cams = torch.full((n, 16384), 7, dtype=torch.uint8, device=DEV)
    assert tb_cuda_render_sensors_device(d, n, lidar, 4096, valid, 2, cams) == 1
    torch.cuda.synchronize()
    l, v, c = lidar.cpu().numpy(), valid.cpu().numpy(), cams.cpu().numpy()
    for i, bits in enumerate(base["sensors"]):
        if bits & 1:
            assert bits_equal(l[i], want[0][i]).all() and bits_equal(v[i], want[1][i]).all()
        else:
            assert (l[i] == -7).all() and (v[i] == -7).all()
        if bits & 2:
            assert np.array_equal(c[i], want[2][i])
        else:
            assert (c[i] == 7).all()
    # NULL outputs: cameras only, then LiDAR only without valid fractions
    lidar.fill_(-7.0)
    cams.fill_(7)
    assert tb_cuda_render_sensors_device(d, n, None, 4096, None, 2, cams) == 1
    assert tb_cuda_render_sensors_device(d, n, lidar, 4096, None, 2, None) == 1
    torch.cuda.synchronize()
    l, c = lidar.cpu().numpy(), cams.cpu().numpy()
    for i, bits in enumerate(base["sensors"]):
        assert bits_equal(l[i], want[0][i]).all() if bits & 1 else (l[i] == -7).all()
        assert np.array_equal(c[i], want[2][i]) if bits & 2 else (c[i] == 7).all()


@pytest.mark.parametrize("count", [1, 3, 17])
def test_ragged_counts_write_only_their_rows(count):
    """Small and odd counts render exactly their scenes; rows past count stay
    untouched."""
    g = np.load(GOLDEN)
    scenes = g["scenes"].view(SCENE_DTYPE).reshape(-1)[-count:].copy()
    scenes["sensors"] = 3
    n = count + 2
    d = _scenes_to_device(scenes)
    lidar = torch.full((n, 4096), -3.0, device=DEV)
    valid = torch.full((n, 2), -3.0, device=DEV)
    cams = torch.full((n, 16384), 9, dtype=torch.uint8, device=DEV)
    assert tb_cuda_render_sensors_device(d, count, lidar, 4096, valid, 2, cams) == 1
    torch.cuda.synchronize()
    l, v, c = lidar.cpu().numpy(), valid.cpu().numpy(), cams.cpu().numpy()
    want = oracle.render_sensors_port(scenes)
    assert_same((l[:count], v[:count], c[:count], None), (want[0], want[1], want[2], None), f"count {count}")
    assert (l[count:] == -3).all() and (v[count:] == -3).all() and (c[count:] == 9).all()


def test_non_default_stream():
    scenes = synthetic_scenes(11, 64)
    s = torch.cuda.Stream(device=DEV)
    with torch.cuda.stream(s):
        got = render_gpu(scenes, stream=s)
    want = oracle.render_sensors_port(scenes)
    assert_same(got, (want[0], want[1], want[2], None), "stream")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_every_visible_gpu_renders_the_same():
    """The ray tables are uploaded per device on first use; every GPU renders
    the golden scenes exactly."""
    g = np.load(GOLDEN)
    scenes = g["scenes"].view(SCENE_DTYPE).reshape(-1)
    n = len(scenes)
    for dev in range(torch.cuda.device_count()):
        with torch.cuda.device(dev):
            d = torch.from_numpy(scenes.view(np.uint8).reshape(-1).copy()).to(f"cuda:{dev}")
            lidar = torch.full((n, 4096), float("nan"), device=f"cuda:{dev}")
            valid = torch.full((n, 2), float("nan"), device=f"cuda:{dev}")
            cams = torch.zeros((n, 16384), dtype=torch.uint8, device=f"cuda:{dev}")
            assert tb_cuda_render_sensors_device(d, n, lidar, 4096, valid, 2, cams) == 1
            torch.cuda.synchronize(dev)
            assert_same((lidar.cpu().numpy(), valid.cpu().numpy(), cams.cpu().numpy(), None),
                        (g["lidar"], g["valid"], g["cameras"], None), f"cuda:{dev}")


@needs_reference
def test_full_batch_sampled_and_deterministic():
    n = 65536
    scenes = synthetic_scenes(2026, n)
    d = _scenes_to_device(scenes)
    outs = []
    for _ in range(2):
        lidar = torch.empty((n, 4096), device=DEV)
        valid = torch.empty((n, 2), device=DEV)
        cams = torch.empty((n, 16384), dtype=torch.uint8, device=DEV)
        assert tb_cuda_render_sensors_device(d, n, lidar, 4096, valid, 2, cams) == 1
        torch.cuda.synchronize()
        outs.append((lidar, valid, cams))
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a.view(torch.uint8) if a.dtype != torch.uint8 else a,
                           b.view(torch.uint8) if b.dtype != torch.uint8 else b)
    pick = np.sort(np.random.default_rng(5).choice(n, 256, replace=False))
    sel = torch.from_numpy(pick).to(DEV)
    got = tuple(t.index_select(0, sel).cpu().numpy() for t in outs[0]) + (None,)
    assert_same(got, oracle.render_sensors_reference(scenes[pick]), "65536 sample")


def test_expf_error_bound_used_by_the_float_fog(tmp_path):
    """The sensor kernel's float fog (sensors_kernel.cu: shade) relies on
    CUDA's __expf being within 3e-7 (absolute) of exp for every argument
    a <= 0.  Checked on every float in [-88, 0] against CUDA's double exp
    (below -88 both are under 1e-38)."""
    import subprocess

    src = os.path.join(os.path.dirname(os.path.abspath(__file__)), "expf_bound.cu")
    exe = str(tmp_path / "expf_bound")
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-o", exe, src], check=True,
                   timeout=300)
    run = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stderr
    worst, where, count = run.stdout.split()
    print(f"\n__expf: largest |error| {float(worst):.3e} at a = {float(where):.9g} over {int(count)} arguments")
    assert int(count) > 1_000_000_000
    assert float(worst) <= 3e-7

"""Sensor-rendering checker, pinned on the CPU (no GPU needed).

* The restated renderers (oracle/sensors_oracle.c) reproduce the committed
  golden renders -- made by the reference simulator's own
  tb_sim_render_lidar / tb_sim_render_camera (tests/golden/make_sensor_golden.py)
  -- bit for bit.
* When the reference build is present (oracle/_ref/libtb_ref_sensors.so), the
  restatement equals the reference renderers live on synthetic, heaviest-case,
  edge-case and simulated-episode scenes, and a scene packed from a simulated
  environment renders exactly as that environment does.
* The product kernel's square-root skip (sphere_hit in sensors_kernel.cu),
  built into a test copy of the restatement, changes no output bit.
* The product's host-built body-frame ray tables (sensor_rays.c, compiled into
  libturbinator_cuda.so) equal the oracle's directions bit for bit, and
  tb_sensor_scene's numpy mirror matches the C layout.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest

import oracle
import turbinator_c_b200 as tb
from tests.sensor_cases import bits_equal, edge_scenes, random_scenes
from turbinator_c_b200.sensors import SCENE_DTYPE, synthetic_scenes

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sensors_reference.npz")
needs_reference = pytest.mark.skipif(not oracle.have_reference_sensors(),
                                     reason="reference simulator build (oracle/_ref) not available")


def _assert_same(got, want, what):
    lidar, valid, cams, raw = got
    rl, rv, rc, rr = want
    bad = ~bits_equal(lidar, rl)
    assert not bad.any(), f"{what}: LiDAR differs in {bad.sum()} bins, first {np.argwhere(bad)[:4].tolist()}"
    assert bits_equal(valid, rv).all(), f"{what}: valid fractions differ"
    bad = cams != rc
    assert not bad.any(), f"{what}: camera differs in {bad.sum()} pixels, first {np.argwhere(bad)[:4].tolist()}"
    if raw is not None and rr is not None:
        assert np.array_equal(raw, rr), f"{what}: raw capture differs"


def test_scene_layout_matches_c():
    layout = oracle.sensor_scene_layout()
    assert layout[0] == SCENE_DTYPE.itemsize == 2432
    assert [SCENE_DTYPE.fields[n][1] for n in SCENE_DTYPE.names] == list(layout[1:])


def test_port_reproduces_reference_golden():
    g = np.load(GOLDEN)
    scenes = g["scenes"].view(SCENE_DTYPE).reshape(-1)
    got = oracle.render_sensors_port(scenes, raw=True)
    n_raw = g["raw"].shape[0]
    _assert_same((got[0], got[1], got[2], got[3][:n_raw]), (g["lidar"], g["valid"], g["cameras"], g["raw"]),
                 "golden")
    # the fixture holds every branch the renderer takes
    assert set(np.unique(scenes["scenario"])) >= {0, 3, 10, 14, 18, 22, 27, 99}
    assert (scenes["ball_count"] >= 64).any() and (scenes["obstacle_count"] > 24).any()


def test_product_ray_tables_equal_oracle_directions():
    lib = ctypes.CDLL(tb.LIB_PATH)
    lib.tb_sensor_lidar_rays.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    lib.tb_sensor_camera_rays.argtypes = [ctypes.c_void_p]
    lidar = np.empty(3 * 4096)
    blocked = np.empty(4096, np.uint8)
    cams = np.empty(3 * 16384)
    lib.tb_sensor_lidar_rays(lidar.ctypes.data, blocked.ctypes.data)
    lib.tb_sensor_camera_rays(cams.ctypes.data)
    o_lidar, o_blocked, o_cams = np.empty_like(lidar), np.empty_like(blocked), np.empty_like(cams)
    ol = oracle.lib()
    ol.oracle_sensor_rays.argtypes = [ctypes.c_void_p] * 3
    ol.oracle_sensor_rays(o_lidar.ctypes.data, o_blocked.ctypes.data, o_cams.ctypes.data)
    assert np.array_equal(lidar.view(np.uint64), o_lidar.view(np.uint64))
    assert np.array_equal(blocked, o_blocked) and 0 < blocked.sum() < 4096
    assert np.array_equal(cams.view(np.uint64), o_cams.view(np.uint64))


@needs_reference
@pytest.mark.parametrize("kind", ["flight", "max", "none"])
def test_port_equals_reference_synthetic(kind):
    scenes = synthetic_scenes(100 + len(kind), 96, balls=kind)
    _assert_same(oracle.render_sensors_port(scenes, raw=kind == "max"),
                 oracle.render_sensors_reference(scenes, raw=kind == "max"), f"synthetic/{kind}")


@needs_reference
def test_port_equals_reference_edge_cases():
    scenes = edge_scenes()
    _assert_same(oracle.render_sensors_port(scenes, raw=True), oracle.render_sensors_reference(scenes, raw=True),
                 "edge")


@needs_reference
def test_packed_scene_renders_as_its_environment():
    n = 56
    idx = np.arange(n)
    scenes, lidar, valid, cams = oracle.simulate_sensor_scenes(idx % 28, idx + 1000, (idx * 53) % 800, idx % 2,
                                                               SCENE_DTYPE)
    assert scenes["ball_count"].max() > 0
    _assert_same(oracle.render_sensors_reference(scenes), (lidar, valid, cams, None), "packed vs environment")
    _assert_same(oracle.render_sensors_port(scenes), (lidar, valid, cams, None), "port vs environment")


@pytest.mark.parametrize("kind", ["flight", "max", "random", "edge"])
def test_sqrt_skip_never_changes_a_render(kind):
    """The product kernel drops a sphere without its square root when the
    sphere's near intersection is provably beyond the ray's nearest hit so
    far. The same condition, built into a copy of the restated renderer
    (oracle/liboracle_skip.so), must leave every output bit unchanged; the
    skip must also fire on the sphere-rich scenes, or the test proves nothing."""
    if kind in ("flight", "max"):
        scenes = synthetic_scenes(300 + len(kind), 64, balls=kind)
    elif kind == "random":
        scenes = np.concatenate([random_scenes(31, 48), random_scenes(32, 48, unit_attitude=False)])
    else:
        scenes = edge_scenes()
    before = oracle.sqrt_skips()
    _assert_same(oracle.render_sensors_port(scenes, raw=kind == "edge", sqrt_skip=True),
                 oracle.render_sensors_port(scenes, raw=kind == "edge"), f"square-root skip/{kind}")
    if kind in ("max", "random"):
        assert oracle.sqrt_skips() > before, "the skip never fired"


@pytest.mark.parametrize("kind", ["flight", "max", "random", "edge", "episodes"])
def test_float_camera_decision_never_changes_a_byte(kind):
    """The product kernel first offers each camera pixel to a float decision
    (turbinator_c_b200/csrc/tb_camera_float.h) and traces it in double only
    when that declines.  The same header, built into a copy of the restated
    renderer (oracle/liboracle_float.so, plain IEEE float arithmetic as on the
    GPU, glibc's expf in place of CUDA's __expf), must give every camera byte
    of the double renderer; on flight scenes it must decide most pixels, or
    the test proves little."""
    if kind in ("flight", "max"):
        scenes = synthetic_scenes(400 + len(kind), 256, balls=kind)
    elif kind == "random":
        scenes = np.concatenate([random_scenes(41, 128), random_scenes(42, 128, unit_attitude=False)])
    elif kind == "edge":
        scenes = edge_scenes()
    else:
        n = 112
        idx = np.arange(n)
        scenes, _, _, _ = oracle.simulate_sensor_scenes(idx % 28, idx + 3000, (idx * 37) % 800, idx % 2, SCENE_DTYPE)
    before = oracle.float_pixels()
    _assert_same(oracle.render_sensors_port(scenes, raw=kind == "edge", float_camera=True),
                 oracle.render_sensors_port(scenes, raw=kind == "edge"), f"float camera/{kind}")
    decided = oracle.float_pixels() - before
    if kind == "flight":
        assert decided > 0.5 * 16384 * len(scenes), decided
    print(f"\n{kind}: {decided} of {16384 * len(scenes)} camera pixels decided in float")

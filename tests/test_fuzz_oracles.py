"""Property-based checks of the CPU oracles against the reference's own code
(oracle/_ref, compiled from the reference sources), on adversarial inputs a
seeded generator rarely produces.  Runs on the CPU; skipped without the
reference build.

* 142 features: observations, missions and cameras drawn from special
  values (NaN, +-inf, -0.0, subnormals, the clamp boundaries, LiDAR ranges at
  0, 0.5, 120 and the float neighbours of 120) mixed with ordinary values;
  the restated oracle must equal tb_train_extract_features_cpu bit for bit.
* sensor rendering: scenes with random attitudes (unit and not), origins
  near or inside spheres, spheres grazing the sensor cones, the arena and
  shelf scenarios and random lidar_max / dome_radius; the restated renderers
  must equal the simulator's tb_sim_render_lidar / tb_sim_render_camera.
"""
from __future__ import annotations

import numpy as np
import pytest
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

import oracle
from tests.sensor_cases import bits_equal, random_scenes
from turbinator_c_b200.sensors import MAX_BALLS, MAX_OBSTACLES

pytestmark = pytest.mark.skipif(not (oracle.have_reference() and oracle.have_reference_sensors()),
                                reason="reference build (oracle/_ref) not available")

F32 = np.float32
SPECIAL = [np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-45, -1e-45, 1.17549435e-38, 0.5, -0.5, 1.0, -1.0,
           0.75, 0.7500001, 0.25, 120.0, float(np.nextafter(F32(120), F32(0))),
           float(np.nextafter(F32(120), F32(200))), 3.4e38, -3.4e38, 300.0, 30.0, 0.05]


def _mixed(rng, n, special_rate):
    v = rng.uniform(-2, 2, n).astype(F32)
    pick = rng.random(n) < special_rate
    v[pick] = np.array(SPECIAL, F32)[rng.integers(0, len(SPECIAL), pick.sum())]
    return v


@settings(max_examples=40, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(seed=st.integers(0, 2**32 - 1), special=st.floats(0.0, 1.0), lidar_log=st.booleans())
def test_feature_oracle_equals_reference_on_special_values(seed, special, lidar_log):
    rng = np.random.default_rng(seed)
    n = 16
    obs = _mixed(rng, n * 4148, special).reshape(n, 4148)
    if lidar_log:  # realistic ranges with the specials sprinkled in
        r = (0.5 * 600.0 ** rng.random((n, 4096))).astype(F32)
        pick = rng.random((n, 4096)) < special * 0.2
        r[pick] = np.array(SPECIAL, F32)[rng.integers(0, len(SPECIAL), pick.sum())]
        obs[:, 48:4144] = r
    mission = _mixed(rng, n * 10, special).reshape(n, 10)
    cams = rng.integers(0, 256, (n, 16384), dtype=np.uint8)
    if rng.random() < 0.3:
        cams[:] = rng.choice([0, 255])
    mine = oracle.features(obs, mission, cams)
    ref = oracle.features(obs, mission, cams, use_reference=True)
    assert np.array_equal(mine.view(np.uint32), ref.view(np.uint32))


@settings(max_examples=30, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(seed=st.integers(0, 2**32 - 1), scenario=st.integers(0, 27), unit=st.booleans(),
       crowd=st.integers(0, MAX_OBSTACLES), balls=st.integers(0, MAX_BALLS))
def test_sensor_oracle_equals_reference_on_random_scenes(seed, scenario, unit, crowd, balls):
    s = random_scenes(seed, 4, scenario=scenario, unit_attitude=unit, obstacles=crowd, balls=balls)
    got = oracle.render_sensors_port(s)
    want = oracle.render_sensors_reference(s, threads=1)
    assert bits_equal(got[0], want[0]).all()
    assert bits_equal(got[1], want[1]).all()
    assert np.array_equal(got[2], want[2])

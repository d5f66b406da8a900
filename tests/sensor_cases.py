"""Scene sets for the sensor-rendering parity tests (CPU and GPU).

edge_scenes(): hand-built scenes for the cases the renderer's branches turn
on -- origins inside spheres (far root), spheres touching rays and the ground,
an origin below the ground, scenario 10's raised shelf, the blended-wing arena
(300 m dome, 0.75 m opponent, 120 m minimum sky distance), a small dome,
full obstacle and ball tables, out-of-range counts (clamped), negative step
index, rng 0, player 1, unnormalised and zero quaternions, an inverted start,
far-off coordinates, non-finite inputs, an unknown scenario number, and each
value of the sensors bit mask.
"""
from __future__ import annotations

import numpy as np

from turbinator_c_b200.sensors import MAX_BALLS, MAX_OBSTACLES, SCENE_DTYPE


def _base(n: int) -> np.ndarray:
    s = np.zeros(n, SCENE_DTYPE)
    s["attitude"] = [1.0, 0.0, 0.0, 0.0]
    s["position"] = [0.0, 0.0, 8.0]
    s["lidar_max"] = 30.0
    s["dome_radius"] = 40.0
    s["rng"] = np.arange(n, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15) + np.uint64(12345)
    s["step_index"] = np.arange(n) * 9
    s["sensors"] = 3
    return s


def edge_scenes() -> np.ndarray:
    rng = np.random.default_rng(20260501)
    cases = []

    def case(**kw):
        cases.append(kw)

    case(obstacles=[[0.3, 0.2, 8.1, 2.0]])                                   # origin inside a sphere
    case(obstacles=[[6.0, 0.0, 8.0, 1.0], [0.0, 6.0, 8.0, 1.0], [4.0, 4.0, 1.0, 1.0],
                    [-5.0, 0.0, 0.5, 0.5], [10.0, 10.0, 8.0, 3.0]])           # touching the ground too
    case(position=[2.0, -1.0, -3.0])                                         # below the ground plane
    case(scenario=10, position=[15.0, 0.0, 12.0], attitude=[0.96, 0.0, 0.28, 0.0])  # shelf at x >= 20
    case(scenario=10, position=[25.0, 3.0, 9.5])                             # above the shelf edge
    case(scenario=22, position=[0.0, 0.0, 65.0], opponent=[0.5, 0.2, 65.1])  # blended-wing arena, r 0.75
    case(scenario=27, position=[250.0, 100.0, 70.0], opponent=[200.0, 90.0, 66.0], lidar_max=200.0)
    case(scenario=3, dome_radius=10.0, position=[8.5, 0.0, 3.0], opponent=[-2.0, 1.0, 4.0],
         balls=(np.array([8.5, 0.0, 3.0]) + rng.uniform(-3, 3, (MAX_BALLS, 3))).tolist())
    case(scenario=14, obstacle_count=99, ball_count=-5,
         obstacles=rng.uniform([-10, -10, 2, 0.5], [10, 10, 14, 2.5], (MAX_OBSTACLES, 4)).tolist(),
         opponent=[3.0, 0.0, 8.0])                                           # counts clamped to 24 and 0
    case(scenario=18, step_index=-7, rng=0, player=1, opponent=[1.0, 1.0, 8.0],
         ball_count=MAX_BALLS + 10, balls=rng.uniform([-6, -6, 4], [6, 6, 12], (MAX_BALLS, 3)).tolist())
    case(attitude=[2.0, 0.4, -0.2, 0.6])                                     # not normalised
    case(attitude=[0.0, 0.0, 0.0, 0.0])                                      # zero quaternion
    case(scenario=4, position=[0.0, 0.0, 14.0], attitude=[0.0, 1.0, 0.0, 0.0])  # inverted start
    case(position=[1.0e6, -2.0e6, 5.0e5], obstacles=[[1.0e6 + 5, -2.0e6, 5.0e5, 2.0]])
    case(position=[np.nan, 0.0, 8.0])                                        # non-finite position
    case(obstacles=[[np.nan, 0.0, 8.0, 1.0], [5.0, 0.0, 8.0, np.inf]])       # non-finite sphere
    case(lidar_max=np.inf)                                                   # sky at infinity
    case(lidar_max=2.0, obstacles=[[1.5, 0.0, 8.0, 1.0]])                   # short sky distance
    case(scenario=99)                                                        # unknown scenario: plain
    case(sensors=0, obstacles=[[3.0, 0.0, 8.0, 1.0]])
    case(sensors=1, obstacles=[[3.0, 0.0, 8.0, 1.0]])
    case(sensors=2, obstacles=[[3.0, 0.0, 8.0, 1.0]])

    s = _base(len(cases))
    for i, kw in enumerate(cases):
        obstacles = kw.pop("obstacles", None)
        balls = kw.pop("balls", None)
        if obstacles is not None:
            s["obstacles"][i, :len(obstacles)] = obstacles
            s["obstacle_count"][i] = len(obstacles)
        if balls is not None:
            s["balls"][i, :len(balls)] = balls
            s["ball_count"][i] = len(balls)
        for k, v in kw.items():
            s[k][i] = v
    return s


def bits_equal(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Elementwise: same float32 bit pattern, or both NaN."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))


def random_scenes(seed: int, n: int, scenario=None, unit_attitude=True, obstacles=None, balls=None):
    """Adversarial scenes for the culling and intersection code: random
    attitudes (unit or not), spheres at random directions and distances
    around the aircraft (some enclosing or grazing the sensors), random sky
    distance and dome, any scenario."""
    rng = np.random.default_rng(seed)
    s = np.zeros(n, SCENE_DTYPE)
    s["scenario"] = rng.integers(0, 28, n) if scenario is None else scenario
    s["position"] = rng.uniform([-30, -30, -2], [30, 30, 20], (n, 3))
    q = rng.normal(size=(n, 4))
    s["attitude"] = q / np.linalg.norm(q, axis=1, keepdims=True) if unit_attitude else q
    s["opponent"] = s["position"] + rng.normal(scale=3.0, size=(n, 3))
    s["lidar_max"] = rng.choice([5.0, 30.0, 150.0], n)
    s["dome_radius"] = rng.choice([10.0, 40.0, 400.0], n)
    s["rng"] = rng.integers(0, 2**63, n, dtype=np.int64).astype(np.uint64)
    s["step_index"] = rng.integers(-10, 100000, n)
    s["player"] = rng.integers(0, 2, n)
    s["sensors"] = 3
    centres = s["position"][:, None, :] + rng.normal(scale=4.0, size=(n, MAX_OBSTACLES, 3))
    radii = rng.uniform(0.0, 3.0, (n, MAX_OBSTACLES, 1))
    s["obstacles"] = np.concatenate([centres, radii], axis=2)
    s["obstacle_count"] = rng.integers(0, MAX_OBSTACLES + 1, n) if obstacles is None else obstacles
    s["balls"] = s["position"][:, None, :] + rng.normal(scale=6.0, size=(n, MAX_BALLS, 3))
    s["ball_count"] = rng.integers(0, MAX_BALLS + 1, n) if balls is None else balls
    return s

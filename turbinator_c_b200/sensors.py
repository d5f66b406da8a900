"""GPU sensor rendering -- Python view of ``include/turbinator/sim/cuda_sensors.h``.

``tb_cuda_render_sensors_device`` renders the simulator's LiDAR (2 heads x
2,048 rays) and four 64x64 cameras for a batch of ``tb_sensor_scene`` records
in one launch, replacing the reference simulator's CPU renderers
(src/sim/sensors.c:28-50 and :69-82).  ``SCENE_DTYPE`` is the record's numpy
layout; ``synthetic_scenes`` makes seeded scenes shaped like the simulator's
(its scenario layouts, src/sim/physics.c:122-170) for benchmarks and tests.
"""
from __future__ import annotations

import numpy as np

from . import _ptr, _stream_handle, load_library

MAX_OBSTACLES = 24
MAX_BALLS = 64
LIDAR_BINS = 4096
CAMERA_PIXELS = 16384
CAMERA_RAW_PIXELS = 147456
SENSOR_LIDAR = 1
SENSOR_CAMERA = 2

#: numpy mirror of tb_sensor_scene (2,432 bytes).
SCENE_DTYPE = np.dtype([
    ("position", "<f8", (3,)),
    ("attitude", "<f8", (4,)),
    ("opponent", "<f8", (3,)),
    ("lidar_max", "<f8"),
    ("dome_radius", "<f8"),
    ("rng", "<u8"),
    ("step_index", "<i4"),
    ("player", "<i4"),
    ("scenario", "<i4"),
    ("sensors", "<i4"),
    ("obstacle_count", "<i4"),
    ("ball_count", "<i4"),
    ("obstacles", "<f8", (MAX_OBSTACLES, 4)),
    ("balls", "<f8", (MAX_BALLS, 3)),
])
assert SCENE_DTYPE.itemsize == 2432

ARENA_SCENARIOS = (3, 14, 15, 16, 18, 22, 24, 27)


def is_arena(s: int) -> bool:
    return s in ARENA_SCENARIOS


def is_bwb(s: int) -> bool:
    return 22 <= s <= 27


def tb_cuda_render_sensors_device(scenes, count: int, lidar, lidar_stride: int, lidar_valid, valid_stride: int,
                                  cameras, raw_cameras=None, stream=None) -> int:
    """Render count scenes (device pointers / tensors; outputs may be None)."""
    return load_library().tb_cuda_render_sensors_device(
        _ptr(scenes), count, _ptr(lidar), lidar_stride, _ptr(lidar_valid), valid_stride, _ptr(cameras),
        _ptr(raw_cameras), _stream_handle(stream))


def _quaternions(rng: np.random.Generator, n: int, tilt: float) -> np.ndarray:
    """Unit quaternions (w, x, y, z): uniform yaw, roll and pitch within +-tilt."""
    yaw = rng.uniform(-np.pi, np.pi, n)
    pitch = rng.uniform(-tilt, tilt, n)
    roll = rng.uniform(-tilt, tilt, n)
    cy, sy = np.cos(yaw / 2), np.sin(yaw / 2)
    cp, sp = np.cos(pitch / 2), np.sin(pitch / 2)
    cr, sr = np.cos(roll / 2), np.sin(roll / 2)
    q = np.stack([cr * cp * cy + sr * sp * sy, sr * cp * cy - cr * sp * sy,
                  cr * sp * cy + sr * cp * sy, cr * cp * sy - sr * sp * cy], axis=1)
    return q / np.linalg.norm(q, axis=1, keepdims=True)


#: Obstacle layouts of the simulator's course scenarios (physics.c:162-166):
#: scenario -> (count, x0, dx, y alternating +-, z, radius).
_COURSES = {2: (5, 8, 7, 1.5, 8, 1.25), 8: (5, 8, 7, 1.5, 8, 1.25), 9: (5, 8, 6, 2.2, 8, 1.8),
            20: (5, 8, 6, 2.2, 8, 1.8), 11: (5, 8, 6, 0.0, 9.2, 2.6)}


def synthetic_scenes(seed: int, count: int, scenarios=None, *, balls: str = "flight",
                     sensors: int = SENSOR_LIDAR | SENSOR_CAMERA) -> np.ndarray:
    """Seeded scenes with the simulator's geometry.

    scenarios: None (uniform over 0..27) or a sequence repeated over count.
    balls: "flight" (arena scenes carry 0-12 cannon balls, as a match does),
    "max" (arena scenes carry all 64 and course scenes 24 obstacles: the
    heaviest scenes the record allows) or "none".
    """
    rng = np.random.default_rng(seed)
    s = np.zeros(count, SCENE_DTYPE)
    scen = (rng.integers(0, 28, count) if scenarios is None
            else np.resize(np.asarray(scenarios, np.int32), count))
    s["scenario"] = scen
    s["lidar_max"] = 30.0
    s["dome_radius"] = 40.0
    s["rng"] = rng.integers(1, 2**63 - 1, count, dtype=np.int64).astype(np.uint64) * np.uint64(2) + np.uint64(1)
    s["step_index"] = rng.integers(0, 1500, count)
    s["sensors"] = sensors
    s["attitude"] = _quaternions(rng, count, 0.45)
    bwb = (scen >= 22) & (scen <= 27)
    arena = np.isin(scen, ARENA_SCENARIOS)
    alt = np.where(bwb, 65.0, 8.0)
    # Course flight: along the course x in [-5, 45], a few metres either side.
    pos = np.stack([rng.uniform(-5, 45, count), rng.uniform(-5, 5, count),
                    alt + rng.uniform(-6, 6, count)], axis=1)
    pos[:, 2] = np.maximum(pos[:, 2], 0.7)
    # Blended-wing course: x from -140 along the 3 waypoints, altitude 40-90.
    wing = bwb & ~arena
    pos[wing] = np.stack([rng.uniform(-150, 150, wing.sum()), rng.uniform(-25, 25, wing.sum()),
                          rng.uniform(40, 90, wing.sum())], axis=1)
    # Arenas: both players inside the dome (300 m for the blended wing).
    dome = np.where(bwb, 300.0, 40.0)
    for who in ("position", "opponent"):
        r = dome * 0.8 * np.sqrt(rng.uniform(0, 1, count))
        a = rng.uniform(-np.pi, np.pi, count)
        xyz = np.stack([r * np.cos(a), r * np.sin(a), alt + rng.uniform(-5, 5, count)], axis=1)
        if who == "position":
            pos[arena] = xyz[arena]
        else:
            s["opponent"][arena] = xyz[arena]
    s["position"] = pos
    s["player"] = np.where(arena, rng.integers(0, 2, count), 0)
    # Scenario 4 starts inverted (physics.c:157).
    inv = scen == 4
    s["attitude"][inv] = np.array([0.0, 1.0, 0.0, 0.0])
    for sc, (n, x0, dx, y, z, radius) in _COURSES.items():
        m = scen == sc
        if not m.any():
            continue
        centres = np.array([[x0 + i * dx, (-y if i & 1 else y), z, radius] for i in range(n)])
        s["obstacles"][m, :n] = centres
        s["obstacle_count"][m] = n
    m = scen == 21
    s["obstacles"][m, :3] = np.array([[3.2, -1.2, 8, 1.05], [9.5, 1.2, 8, 1.05], [16, -1.2, 8, 1.05]])
    s["obstacle_count"][m] = 3
    if balls == "max":
        course = ~arena
        s["obstacle_count"][course] = MAX_OBSTACLES
        s["obstacles"][course] = np.concatenate([
            rng.uniform([-5, -8, 2], [50, 8, 14], (course.sum(), MAX_OBSTACLES, 3)),
            rng.uniform(0.8, 2.6, (course.sum(), MAX_OBSTACLES, 1))], axis=2)
    if balls != "none":
        nb = np.where(arena, MAX_BALLS if balls == "max" else rng.integers(0, 13, count), 0)
        s["ball_count"] = nb
        # Balls between the players, spread by flight.
        mid = 0.5 * (s["position"] + s["opponent"])
        spread = np.where(bwb, 60.0, 12.0)[:, None, None]
        s["balls"] = mid[:, None, :] + spread * rng.uniform(-1, 1, (count, MAX_BALLS, 3))
        s["balls"][~arena] = 0.0
    return s

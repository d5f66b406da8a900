"""Input recipes for the golden fixtures (shared by make_golden.py and the tests).

The expected outputs live in the .npz/.json files beside this module and were
produced by the reference's own CPU code (see make_golden.py).
"""
from __future__ import annotations

import numpy as np

OBS, MIS, CAM = 4148, 10, 16384

#: name -> (seed, batch total, samples generated from index 0, stress quarters?)
SEEDED_CASES = {
    "config0_seed0": (0, 8, 8, False),
    "config1_seed1_first256": (1, 1024, 256, False),
    "config4_seed4_b64": (4, 64, 64, True),
}


def reference_known_answer_inputs():
    """The three synthetic samples of the reference's CUDA parity test
    (tests/test_cuda_features.c:17-26), in float32 arithmetic as there."""
    count = 3
    obs = np.empty((count, OBS), np.float32)
    mission = np.empty((count, MIS), np.float32)
    cams = np.empty((count, CAM), np.uint8)
    i = np.arange(OBS)
    for b in range(count):
        lidar = np.float32(0.5) + ((i + 17 * b) % 119).astype(np.float32)
        other = (((i * 11 + b * 7) % 81) - 40).astype(np.float32) * np.float32(0.125)
        obs[b] = np.where((i >= 48) & (i < 4144), lidar, other)
        mission[b] = (np.arange(MIS) - 5 + b).astype(np.float32) * np.float32(0.2)
        cams[b] = ((np.arange(CAM) * 13 + b * 29) & 255).astype(np.uint8)
    return obs, mission, cams


def _f32(*vals):
    return np.array(vals, dtype=np.float32)


SPECIAL_RANGES = _f32(
    np.nan, np.inf, -np.inf, -1.0, -0.0, 0.0, 1e-45, 1.1754942e-38, 1e-7, 1e-3,
    0.35, 0.5, 1.0, 119.99999, 120.0, 120.00001, 299.99997, 300.0, 1e30, 3.4028235e38,
    -1e-45, -300.0, 11.5, 60.0)


def edge_inputs():
    """Eight hand-built samples that stress every branch of the 142 features."""
    rng = np.random.default_rng(20260601)
    n = 8
    obs = np.zeros((n, OBS), np.float32)
    mission = np.zeros((n, MIS), np.float32)
    cams = np.zeros((n, CAM), np.uint8)

    scalar_specials = _f32(np.nan, np.inf, -np.inf, -0.0, 0.0, 300.0, -300.0, 300.00003,
                           100.0, 50.0, 5.0, 30.0, 0.78539819, 1.5707964, -1.5707964, 1e-45,
                           1e38, -1e38, 2.0, -2.0, 0.99999994, -0.99999994, 1.0, -1.0)
    tail_specials = _f32(np.nan, -0.0, 2.0, 0.5, np.inf, -np.inf, 1e-45, 0.99999994)
    mission_specials = _f32(np.nan, np.inf, -np.inf, -0.0, 1.5, -1.5, 0.9, -0.99999994, 1.0, 0.0)

    for s in range(n):
        obs[s, :48] = np.roll(scalar_specials, s)[:24].repeat(2)[:48]
        obs[s, 4144:4148] = np.roll(tail_specials, s)[:4]
        mission[s] = np.roll(mission_specials, s)

    # LiDAR patterns
    obs[0, 48:4144] = np.resize(SPECIAL_RANGES, 4096)                    # cycling specials
    obs[1, 48:4144] = -1.0                                               # simulator dropouts
    obs[2, 48:4144] = 300.0                                              # all no-return
    obs[3, 48:4144] = np.nan                                             # all NaN
    obs[4, 48:4144] = 0.5                                                # identical terms
    obs[5, 48:4144] = rng.choice(SPECIAL_RANGES, 4096)                   # random specials
    obs[6, 48:4144] = np.concatenate([rng.uniform(0, 1e-3, 2048), rng.uniform(119.9, 120.1, 2048)]
                                     ).astype(np.float32)
    obs[7, 48:4144] = (0.5 * 600.0 ** rng.uniform(0, 1, 4096)).astype(np.float32)

    # Arena mask boundary: finite(m6) > 0.5 hides mission[7..9].
    mission[0, 6] = 0.5                    # not arena (not > 0.5)
    mission[1, 6] = np.nextafter(np.float32(0.5), np.float32(1))  # arena
    mission[2, 6] = np.nan                 # finite() -> 0: not arena
    mission[3, 6] = np.inf                 # finite() -> 0: not arena
    mission[4, 6] = 1.0                    # arena
    mission[5, 6] = -np.inf
    mission[6, 6] = 0.75
    mission[7, 6] = 0.25
    for s in (1, 4, 6):
        mission[s, 7:10] = _f32(0.9, np.nan, -np.inf)

    # Cameras: extremes, pattern, random
    cams[0] = 255
    cams[1] = 0
    cams[2] = (np.arange(CAM) * 7 & 255).astype(np.uint8)
    cams[3] = 128
    cams[4] = rng.integers(0, 256, CAM, dtype=np.uint8)
    cams[5] = 1
    cams[6] = 254
    cams[7] = rng.integers(0, 256, CAM, dtype=np.uint8)
    return obs, mission, cams


def onboard_fixture_inputs():
    """The four onboard fixtures of the reference's tests/test_onboard_features.cu:19-39
    (hover, slalom with two LiDAR hits, BWB cruise, arena)."""
    rows = 4
    obs = np.zeros((rows, OBS), np.float32)
    mission = np.zeros((rows, MIS), np.float32)
    for r in range(rows):
        o = obs[r]
        o[2] = 8.0; o[6] = 1.0; o[40] = 0.6; o[47] = 1.0
        o[16:20] = 0.5
        o[24:28] = 1.0
    obs[0, 3] = 1.0
    o, m = obs[1], mission[1]
    o[0] = 5.0; o[1] = 0.4; o[3] = 2.0; o[4] = -0.2
    o[48 + 2 * 128 + 3] = 5.0
    o[48 + 2 * 128 + 4] = 5.1
    m[4] = 1.0; m[7] = 0.3; m[8] = -0.2; m[9] = 0.1
    o, m = obs[2], mission[2]
    o[0] = 80.0; o[2] = 60.0; o[3] = 15.0; o[5] = -0.3
    o[6] = 0.98; o[7] = 0.10; o[8] = 0.10; o[9] = 0.05
    m[0] = 0.5; m[2] = 0.5; m[4] = 1.0
    m[7] = 0.2; m[8] = 0.05; m[9] = 0.1
    o, m = obs[3], mission[3]
    o[0] = 200.0; o[2] = 40.0; o[3] = 20.0; o[4] = 1.0
    o[6] = 0.9; o[7] = 0.1; o[8] = -0.2; o[9] = 0.3
    m[4] = -0.5; m[5] = 0.8; m[6] = 1.0
    m[7] = -0.3; m[8] = 0.1
    return obs, mission

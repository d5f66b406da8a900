"""Input builders shared by the onboard tests (standalone onboard entry point)
and the learner-input tests (whose kernel runs the same LiDAR scans from the
rows it has staged)."""
from __future__ import annotations

import numpy as np


def force_modes(mission, dodge_rows, slalom_rows):
    """Missions that read the LiDAR scans: dodge (nearest-return avoidance)
    and slalom (corridor cluster, with m[5] <= 0.25)."""
    mission[dodge_rows, 5] = 1.0
    mission[slalom_rows, 4] = 1.0
    mission[slalom_rows, 5] = -0.5


def cluster_cancellation(n: int, seed: int = 11):
    """Slalom aircraft whose corridor returns are mirror-symmetric about the
    lane centre line, so the cluster y sum cancels to rounding level and its
    sign must come from the reference's in-order float sum.  Returns
    (obs [n, 4148], mission [n, 10])."""
    rng = np.random.default_rng(seed)
    obs = np.zeros((n, 4148), np.float32)
    mission = np.zeros((n, 10), np.float32)
    obs[:, 6] = 1.0                                   # level attitude
    obs[:, 2] = 9.0
    obs[:, 1] = 0.0                                   # on the lane centre line
    obs[:, 40] = 0.5
    mission[:, 4] = 1.0                               # slalom
    mission[:, 7:10] = rng.uniform(-0.5, 0.5, (n, 3)).astype(np.float32)
    lidar = np.full((n, 2, 16, 128), 50.0, np.float32)  # out of the 0.35-11.5 m window
    for i in range(n):
        k = int(rng.integers(1, 16))                   # forward azimuth index and its mirror 96 - k
        r = np.float32(rng.uniform(1.0, 2.5))
        el = int(rng.integers(0, 3))
        lidar[i, 0, el, k] = r
        lidar[i, 0, el, 96 - k] = r
        if i % 3 == 0:                                 # a second symmetric pair
            k2 = int(rng.integers(1, 16))
            lidar[i, 1, el, k2] = r
            lidar[i, 1, el, 96 - k2] = r
        if i % 5 == 0:                                 # tiny attitude tilt: near, not exact, symmetry
            obs[i, 9] = np.float32(rng.uniform(-1e-6, 1e-6))
    obs[:, 48:4144] = lidar.reshape(n, 4096)
    return obs, mission

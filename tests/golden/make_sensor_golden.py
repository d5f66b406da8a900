"""Regenerates tests/golden/sensors_reference.npz from the reference itself.

Run in a checkout with the reference source tree next to the repository
after `make -C oracle` (which builds oracle/_ref/libtb_ref_sensors.so from the
reference simulator's own src/sim/{physics,sensors,c_api}.c):

    python tests/golden/make_sensor_golden.py

The scenes are the hand-built edge cases of tests/sensor_cases.py plus six
scenes packed from simulated episodes (reference controller; course, shelf,
quadrotor arena and blended-wing arena scenarios).  Every expected output is
rendered by the reference's tb_sim_render_lidar / tb_sim_render_camera.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from tests.sensor_cases import edge_scenes  # noqa: E402
from turbinator_c_b200.sensors import SCENE_DTYPE  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sensors_reference.npz")

SIMULATED = {  # scenario, seed, steps, player
    "scenarios": [2, 10, 3, 22, 18, 25],
    "seeds": [7, 8, 9, 10, 11, 12],
    "steps": [120, 300, 400, 350, 200, 90],
    "players": [0, 0, 1, 0, 0, 0],
}


def main() -> None:
    sim, _, _, _ = oracle.simulate_sensor_scenes(SIMULATED["scenarios"], SIMULATED["seeds"], SIMULATED["steps"],
                                                 SIMULATED["players"], SCENE_DTYPE)
    scenes = np.concatenate([edge_scenes(), sim])
    lidar, valid, cams, raw = oracle.render_sensors_reference(scenes, raw=True, threads=1)
    np.savez_compressed(OUT, scenes=scenes.view(np.uint8).reshape(len(scenes), -1), lidar=lidar, valid=valid,
                        cameras=cams, raw=raw[:4])
    print(f"wrote {OUT}: {len(scenes)} scenes, {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()

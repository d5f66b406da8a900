"""Regenerates the golden fixtures in tests/golden/ from the reference itself.

Run in a checkout that has the reference source tree next to the repository
(the default location oracle/Makefile looks in) after `make -C oracle`:

    python tests/golden/make_golden.py

Every expected output here comes from the reference's own code compiled in
oracle/_ref/ -- src/training/training.c (tb_train_extract_features_cpu) and
src/network/onboard_features.cuh built for the host -- never from this
repository's kernels.  The onboard golden values are read out of the
reference's tests/test_onboard_features.cu as text.  Inputs that come from the
seeded generator are recorded by SHA-256 so a test can confirm it regenerates
the same bytes before comparing outputs.
"""
from __future__ import annotations

import hashlib
import json
import os
import re
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
import turbinator_c_b200 as tb  # noqa: E402
from tests.golden import fixtures  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
REFERENCE = os.environ.get("TB_REFERENCE_DIR", os.path.join(os.path.dirname(ROOT), "reference"))


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def ref_features(obs, mission, cams):
    return oracle.features(obs, mission, cams, threads=1, use_reference=True)


def main() -> None:
    if not oracle.have_reference():
        raise SystemExit("oracle/_ref is not built; run `make -C oracle` with the reference present")

    # 1. The reference's CUDA parity test inputs (tests/test_cuda_features.c:17-26).
    obs, mission, cams = fixtures.reference_known_answer_inputs()
    np.savez_compressed(os.path.join(OUT, "ref_known_answer.npz"),
                        features=ref_features(obs, mission, cams))

    # 2. Seeded configurations at oracle-friendly sizes.
    seeded = {}
    for name, (seed, total, count, stress) in fixtures.SEEDED_CASES.items():
        obs, mission, cams, camf = tb.generate(seed, 0, count, total=total, stress=stress,
                                               f32_cameras=True)
        seeded[name] = dict(input_sha256=sha(obs, mission, cams), camf_sha256=sha(camf))
        np.savez_compressed(os.path.join(OUT, f"{name}.npz"),
                            features=ref_features(obs, mission, cams))
    with open(os.path.join(OUT, "seeded_inputs.json"), "w") as f:
        json.dump(seeded, f, indent=1, sort_keys=True)

    # 3. Hand-built edge values (non-finite, signed zeros, subnormals, mask
    #    boundary, camera extremes).
    obs, mission, cams = fixtures.edge_inputs()
    np.savez_compressed(os.path.join(OUT, "edge_cases.npz"), obs=obs, mission=mission, cameras=cams,
                        features=ref_features(obs, mission, cams),
                        features_no_camera=ref_features(obs, mission, None))

    # 4. Onboard tactical/prior: the reference test's four fixtures, the
    #    reference header's outputs for them, and the 40 golden values quoted
    #    in that test.
    obs, mission = fixtures.onboard_fixture_inputs()
    outputs = oracle.onboard_reference(obs, mission)
    text = open(os.path.join(REFERENCE, "tests", "test_onboard_features.cu")).read()
    goldens = [(int(r), int(i), float(v)) for r, i, v in
               re.findall(r"\{\s*(\d+)\s*,\s*(\d+)\s*,\s*([-+0-9.eE]+)f\s*\}", text)]
    if len(goldens) != 40:
        raise SystemExit(f"expected 40 onboard goldens, parsed {len(goldens)}")
    with open(os.path.join(OUT, "onboard_fixtures.json"), "w") as f:
        json.dump({"source": "tests/test_onboard_features.cu:55-73 (values), :19-39 (fixtures)",
                   "tolerance": 5e-5,
                   "goldens": goldens,
                   "reference_outputs": outputs.tolist(),
                   "reference_outputs_hex": [[int(x) for x in row.view(np.uint32)] for row in outputs]},
                  f, indent=1)
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()

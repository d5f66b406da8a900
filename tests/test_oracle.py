"""CPU oracle pinned against the reference: golden vectors produced by the
reference's own training.c / onboard header (tests/golden/make_golden.py),
the facts pinned by the reference's tests, and -- where the reference build in
oracle/_ref is present -- live bit-for-bit comparison."""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import pytest

import oracle
import turbinator_c_b200 as tb
from tests.golden import fixtures

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def _sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def test_reference_known_answer_samples():
    """tests/test_cuda_features.c:17-26 inputs; expected from the reference build."""
    obs, mission, cams = fixtures.reference_known_answer_inputs()
    assert _bits_equal(oracle.features(obs, mission, cams), _load("ref_known_answer.npz")["features"])


@pytest.mark.parametrize("name", sorted(fixtures.SEEDED_CASES))
def test_seeded_goldens(name):
    seed, total, count, stress = fixtures.SEEDED_CASES[name]
    meta = json.load(open(os.path.join(GOLDEN, "seeded_inputs.json")))[name]
    obs, mission, cams, camf = tb.generate(seed, 0, count, total=total, stress=stress, f32_cameras=True)
    assert _sha(obs, mission, cams) == meta["input_sha256"], "generator no longer reproduces the inputs"
    assert _sha(camf) == meta["camf_sha256"]
    assert _bits_equal(oracle.features(obs, mission, cams), _load(f"{name}.npz")["features"])


def test_edge_value_goldens():
    g = _load("edge_cases.npz")
    obs, mission, cams = fixtures.edge_inputs()
    assert np.array_equal(obs.view(np.uint32), g["obs"].view(np.uint32))
    assert _bits_equal(oracle.features(obs, mission, cams), g["features"])
    assert _bits_equal(oracle.features(obs, mission, None), g["features_no_camera"])


def test_reference_training_facts():
    """tests/test_training.c:25-35: f[2] > 0 and f[126] > 0 with cameras of 128;
    f[59] == 0 once mission[6] = 1 hides the goal error."""
    obs = np.zeros((1, 4148), np.float32)
    mission = np.zeros((1, 10), np.float32)
    cams = np.full((1, 16384), 128, np.uint8)
    mission[0, 0] = 1.0
    obs[0, 2] = 2.0
    f = oracle.features(obs, mission, cams)[0]
    assert f[2] > 0 and f[126] > 0
    mission[0, 6] = 1.0
    mission[0, 7] = 0.9
    assert oracle.features(obs, mission, cams)[0][59] == 0.0


def test_stress_quarter_properties():
    """Config-4 quarters at a small size: camera extremes give 0/1 exactly, an
    all-no-return scan gives sector means of exactly 1.0."""
    obs, mission, cams, _ = tb.generate(4, 0, 64, total=64, stress=True)
    f = oracle.features(obs, mission, cams)
    a, b = f[0:16], f[16:32]
    assert np.all(a[0::2, 126:142] == 0.0) and np.all(a[1::2, 126:142] == 1.0)
    assert np.all(b[:, 62:126] == 1.0)


@pytest.mark.skipif(not oracle.have_reference(), reason="reference build (oracle/_ref) not present")
def test_oracle_bitwise_equals_reference_live():
    obs, mission, cams, _ = tb.generate(11, 0, 1024)
    eobs, emission, ecams = fixtures.edge_inputs()
    for o, m, c in ((obs, mission, cams), (eobs, emission, ecams), (obs, mission, None)):
        assert _bits_equal(oracle.features(o, m, c), oracle.features(o, m, c, use_reference=True))


@pytest.mark.skipif(not os.path.exists(oracle.REF_ONBOARD_PATH), reason="reference onboard build absent")
def test_onboard_reference_reproduces_published_goldens():
    """tests/test_onboard_features.cu:55-85: 40 golden values within 5e-5 and
    every prior output in [-1, 1]."""
    g = json.load(open(os.path.join(GOLDEN, "onboard_fixtures.json")))
    obs, mission = fixtures.onboard_fixture_inputs()
    out = oracle.onboard_reference(obs, mission)
    for row, idx, expected in g["goldens"]:
        assert abs(out[row, idx] - expected) <= g["tolerance"], (row, idx)
    assert np.all(np.isfinite(out)) and np.all(np.abs(out[:, 24:]) <= 1.00001)
    assert np.array_equal(out.view(np.uint32), np.array(g["reference_outputs_hex"], np.uint32))


@pytest.mark.skipif(not os.path.exists(oracle.REF_ONBOARD_CR_PATH), reason="reference onboard build absent")
def test_onboard_reference_builds_differ_only_by_libm_rounding():
    """The correctly rounded build of the reference header stays within the
    reference test's 5e-5 of the glibc build and never flips a flag on the
    fixtures and a seeded batch."""
    obs, mission = fixtures.onboard_fixture_inputs()
    o2, m2, _, _ = tb.generate(2, 0, 4096)
    for o, m in ((obs, mission), (o2, m2)):
        a = oracle.onboard_reference(o, m)
        b = oracle.onboard_reference_cr(o, m)
        assert np.max(np.abs(a - b)) <= 5e-5
        for c in (11, 22, 38):
            assert np.array_equal(a[:, c], b[:, c])

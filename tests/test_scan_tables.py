"""The onboard scans' ray direction constants (turbinator_c_b200/csrc/
tb_scan_tables.h) are what their generator writes, and each is the float
nearest to cos / sin of its float angle (reference
src/network/onboard_features.cuh:188-196 forms the angles in float)."""
from __future__ import annotations

import importlib.util
import pathlib
import re

import numpy as np

CSRC = pathlib.Path(__file__).resolve().parents[1] / "turbinator_c_b200" / "csrc"


def _generator():
    spec = importlib.util.spec_from_file_location("gen_scan_tables", CSRC / "gen_scan_tables.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_header_is_the_generator_output():
    assert (CSRC / "tb_scan_tables.h").read_text() == _generator().header()


def test_constants_are_correctly_rounded():
    text = (CSRC / "tb_scan_tables.h").read_text()
    body = text[text.index("{") + 1:text.index("};")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    vals = [np.float32(float.fromhex(v.strip()[:-1]) if "0x" in v else float(v.strip()[:-1]))
            for v in body.split(",") if v.strip()]
    assert len(vals) == 280
    pi = np.float32(3.14159265358979323846)
    angles = [np.float32((1 if i < 6 else -1) * ((pi * np.float32(i % 6)) / np.float32(30))) for i in range(12)]
    angles += [np.float32(pi * (np.float32(0.25) + np.float32(a) / np.float32(64))) for a in range(128)]
    cos_el, sin_el, cos_az, sin_az = vals[:12], vals[12:24], vals[24:152], vals[152:]
    for got_c, got_s, x in zip(cos_el + cos_az, sin_el + sin_az, angles[:12] + angles[12:]):
        # numpy's double cos / sin are within an ulp of double; none of these
        # values lies that close to a float rounding boundary
        assert got_c == np.float32(np.cos(np.float64(x)))
        assert got_s == np.float32(np.sin(np.float64(x)))
        if x == 0:                                   # sin keeps the sign of a zero angle
            assert np.signbit(got_s) == np.signbit(x)

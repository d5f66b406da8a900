"""Parity rules shared by the tests (the bar set by the benchmark's north star).

 * Bit-exact: f[0..61] (scaled proprioception, LiDAR status, mission with the
   arena mask) and f[126..141] (camera quadrant means) -- the reference
   computes them with IEEE divisions, compare-based clamps and integer sums.
 * Tolerance: f[62..125] (LiDAR sector means) within
   |actual - expected| <= 1e-6 + 1e-5 * |expected|.
"""
from __future__ import annotations

import numpy as np

ABS_TOL = 1e-6
REL_TOL = 1e-5
EXACT = np.r_[0:62, 126:142]
LIDAR = np.r_[62:126]


def check_features(actual: np.ndarray, expected: np.ndarray, what: str = "") -> None:
    assert actual.shape == expected.shape, (actual.shape, expected.shape)
    a = np.ascontiguousarray(actual, np.float32)
    e = np.ascontiguousarray(expected, np.float32)
    ab, eb = a.view(np.uint32), e.view(np.uint32)
    bad = np.argwhere(ab[:, EXACT] != eb[:, EXACT])
    if bad.size:
        s, j = bad[0]
        f = EXACT[j]
        raise AssertionError(f"{what}: {len(bad)} exact-feature mismatches; first sample {s} feature {f}: "
                             f"got {a[s, f]!r} ({ab[s, f]:#010x}) expected {e[s, f]!r} ({eb[s, f]:#010x})")
    al, el = a[:, LIDAR], e[:, LIDAR]
    assert np.isfinite(al).all(), f"{what}: non-finite LiDAR feature"
    err = np.abs(al.astype(np.float64) - el.astype(np.float64))
    lim = ABS_TOL + REL_TOL * np.abs(el.astype(np.float64))
    over = np.argwhere(err > lim)
    if over.size:
        s, j = over[0]
        raise AssertionError(f"{what}: {len(over)} LiDAR features out of tolerance; first sample {s} "
                             f"feature {62 + j}: got {al[s, j]!r} expected {el[s, j]!r} (|d|={err[s, j]:.3g})")


def max_lidar_error(actual: np.ndarray, expected: np.ndarray) -> float:
    return float(np.max(np.abs(actual[:, LIDAR].astype(np.float64) - expected[:, LIDAR].astype(np.float64)),
                        initial=0.0))


def mismatch_counts(actual: np.ndarray, expected: np.ndarray) -> tuple:
    """(rows with an exact-class feature that differs in any bit, LiDAR
    values out of tolerance or non-finite) under the same rules as
    check_features; (0, 0) is a pass."""
    a = np.ascontiguousarray(actual, np.float32)
    e = np.ascontiguousarray(expected, np.float32)
    if a.shape != e.shape:
        raise ValueError(f"shape {a.shape} != {e.shape}")
    exact_rows = int(np.count_nonzero(np.any(a.view(np.uint32)[:, EXACT] != e.view(np.uint32)[:, EXACT], axis=1)))
    al = a[:, LIDAR].astype(np.float64)
    el = e[:, LIDAR].astype(np.float64)
    with np.errstate(invalid="ignore"):
        bad = ~(np.abs(al - el) <= ABS_TOL + REL_TOL * np.abs(el))
    return exact_rows, int(np.count_nonzero(bad))

"""The FP32-camera kernel's exact quantiser (luma_byte in
turbinator_c_b200/csrc/features_kernel.cu), restated step by step in numpy,
against the simulator's rule (reference src/sim/sensors.c:67 with the clamp of
src/sim/sim_internal.h:73): fmax(0, fmin(255, round(v * 255))) in double,
round half away from zero.

The kernel forms hi = RN(c * 255) and its exact FMA residual lo, rounds hi to
the nearest integer with ties to even by adding and subtracting 2^23, and
repairs exact half-integers from the sign of lo.  Checked here on every float
within 256 ulps of each rounding boundary (k + 1/2) / 255, a strided sample of
[0, 1], and values outside it; run with TB_EXHAUSTIVE=1 to check all
1,065,353,217 floats in [0, 1] (about a minute)."""
from __future__ import annotations

import os

import numpy as np

M = np.float32(2.0 ** 23)


def kernel_formula(v: np.ndarray) -> np.ndarray:
    v = v.astype(np.float32)
    with np.errstate(invalid="ignore"):
        c = np.maximum(np.minimum(v, np.float32(1)), np.float32(0))  # fminf then fmaxf: NaN -> 1
    hi = (c * np.float32(255)).astype(np.float32)
    # the FMA residual of a float product is a float: compute it exactly in double
    lo = (c.astype(np.float64) * 255.0 - hi.astype(np.float64)).astype(np.float32)
    r = ((hi + M).astype(np.float32) - M).astype(np.float32)
    half = np.where(np.signbit(lo), np.float32(-0.5), np.float32(0.5)).astype(np.float32)
    q = np.where(np.abs((r - hi).astype(np.float32)) == np.float32(0.5), (hi + half).astype(np.float32), r)
    return np.where(np.isnan(v), np.float32(255), q)


def simulator_rule(v: np.ndarray) -> np.ndarray:
    x = v.astype(np.float64) * 255.0
    with np.errstate(invalid="ignore"):
        r = np.where(x >= 0, np.floor(x + 0.5), np.ceil(x - 0.5))  # round half away from zero
        out = np.maximum(0.0, np.minimum(255.0, r))
    return np.where(np.isnan(x), 255.0, out)  # fmax/fmin in C pass NaN through only if both are NaN


def _check(v: np.ndarray) -> None:
    got, want = kernel_formula(v), simulator_rule(v)
    bad = np.flatnonzero(got.astype(np.float64) != want)
    assert bad.size == 0, f"{bad.size} mismatches, first v={v[bad[0]]!r}: {got[bad[0]]} != {want[bad[0]]}"


def test_near_every_rounding_boundary():
    bounds = ((np.arange(256, dtype=np.float64) + 0.5) / 255.0).astype(np.float32).view(np.int32)
    offsets = np.arange(-256, 257, dtype=np.int32)
    bits = (bounds[:, None] + offsets[None, :]).reshape(-1)
    _check(bits.view(np.float32))


def test_strided_sample_and_outside_values():
    one = int(np.float32(1).view(np.uint32))
    _check(np.arange(0, one + 1, 1021, dtype=np.uint32).view(np.float32))
    specials = np.array([np.nan, np.inf, -np.inf, -0.0, 0.0, -1e-30, 1e-45, 1.0, 1.0000001, 2.0, -2.0,
                         np.finfo(np.float32).max, -np.finfo(np.float32).max], dtype=np.float32)
    _check(specials)
    rng = np.random.default_rng(7)
    _check(rng.uniform(-3, 3, 1 << 16).astype(np.float32))


def test_exhaustive_when_asked():
    if os.environ.get("TB_EXHAUSTIVE") != "1":
        return
    one = int(np.float32(1).view(np.uint32))
    step = 1 << 24
    for start in range(0, one + 1, step):
        _check(np.arange(start, min(start + step, one + 1), dtype=np.uint32).view(np.float32))

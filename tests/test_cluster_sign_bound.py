"""The onboard scan kernel's shortcut for the sign of the corridor cluster's
y sum (scan_rays in turbinator_c_b200/csrc/onboard_kernel.cu).

The reference adds the cluster's y values in ray order in float and the
control law reads only the sign of that sum (onboard_features.cuh:213-239).
The kernel sums the same values in double, in whatever order its lanes
combine them, and takes the double sum's sign when |dsum| > 2 n 2^-24 sum|y| and
sum|y| < 2^127; otherwise it forms the in-order float sum exactly.  An in-order float sum of
n terms differs from the exact sum by at most (n - 1) 2^-24 sum|y| (to first
order), and the double sum's own error is below 2^-40 of that, so a settled
sign is the in-order float sum's sign.  Checked here on sums built to cancel:
mirror-symmetric clusters with small perturbations, values near the corridor
edge, long clusters with a wide dynamic range, and values near FLT_MAX whose
in-order float sum overflows (the 2^127 cap sends those to the exact path).
"""
from __future__ import annotations

import numpy as np

CORRIDOR_Y = 3.5  # |y| of a corridor centre (onboard_features.cuh:206)
MAX_RAYS = 1536


def in_order_float_sum(y: np.ndarray) -> np.float32:
    return np.cumsum(y.astype(np.float32), dtype=np.float32)[-1]


def kernel_sign(y: np.ndarray, rng: np.random.Generator):
    """The kernel's decision: +-1.0 when the bound settles the sign, None when
    it falls back to the exact in-order sum.  The double sum is taken in a
    shuffled order, as the kernel's lanes and shuffles take it in theirs."""
    d = rng.permutation(y.astype(np.float64))
    dsum = float(np.sum(d))
    dabs = float(np.sum(np.abs(d)))
    bound = 2.0 * len(y) * 2.0 ** -24 * dabs
    if dabs < 2.0 ** 127 and abs(dsum) > bound:
        return 1.0 if dsum > 0 else -1.0
    return None


def _cases(rng: np.random.Generator):
    for _ in range(4000):
        k = int(rng.integers(1, MAX_RAYS // 2 + 1))
        a = rng.uniform(-CORRIDOR_Y, CORRIDOR_Y, k).astype(np.float32)
        eps = np.float32(rng.choice([0.0, 1e-7, 1e-6, 1e-5, 1e-3]) * rng.choice([-1, 1]))
        y = np.concatenate([a, -a]).astype(np.float32)
        y[int(rng.integers(0, len(y)))] += eps
        yield rng.permutation(y)
    for _ in range(2000):
        n = int(rng.integers(1, MAX_RAYS + 1))
        scale = 10.0 ** rng.uniform(-6, 0.5, n)
        y = (rng.choice([-1.0, 1.0], n) * np.minimum(scale, CORRIDOR_Y)).astype(np.float32)
        y -= np.float32(np.mean(y.astype(np.float64)))  # pull the sum towards zero
        yield np.clip(y, -CORRIDOR_Y, CORRIDOR_Y).astype(np.float32)
    for _ in range(2000):
        n = int(rng.integers(2, 64))
        y = rng.uniform(3.4, CORRIDOR_Y, n).astype(np.float32) * rng.choice([-1, 1], n).astype(np.float32)
        yield y
    # magnitudes near FLT_MAX: the in-order float sum can overflow to +-inf
    # while the double sum stays finite with the other sign
    big = np.float32(3.4e38)
    yield np.array([big, big, -big, -big, -big], np.float32)
    yield np.array([-big, -big, big, big, big], np.float32)
    for _ in range(200):
        n = int(rng.integers(2, 16))
        yield (rng.uniform(1.0e38, 3.4e38, n) * rng.choice([-1.0, 1.0], n)).astype(np.float32)


def test_settled_sign_is_the_in_order_float_sums_sign():
    rng = np.random.default_rng(20261202)
    settled = fallback = 0
    for y in _cases(rng):
        sign = kernel_sign(y, rng)
        if sign is None:
            fallback += 1
            continue
        settled += 1
        with np.errstate(over="ignore"):
            s = in_order_float_sum(y)
        assert s != 0 and np.sign(s) == sign, f"n={len(y)}: settled {sign}, in-order float sum {s!r}"
    # both branches are exercised
    assert settled > 1000 and fallback > 100, (settled, fallback)


def test_overflowing_float_sum_takes_the_exact_path():
    big = np.float32(3.4e38)
    y = np.array([big, big, -big, -big, -big], np.float32)
    with np.errstate(over="ignore"):
        assert in_order_float_sum(y) == np.inf          # while the exact sum is negative
    assert kernel_sign(y, np.random.default_rng(0)) is None

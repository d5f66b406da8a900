"""The sensor kernel's float shortcuts restated with numpy float32 arithmetic
(certain_miss in turbinator_c_b200/csrc/sensors_kernel.cu; a float ground test
with relatively widened limits, the form the float camera decision in
tb_camera_float.h builds on -- that header's own bounds are checked bit for bit
by tests/test_sensors_oracle.py; and the float direction's error) and checked
against the double arithmetic they stand in for, on
cases built to sit at the decision boundaries: rays tangent to a sphere within
a relative 1e-12 .. 1e-3, spheres from 1 mm to 1e6 m away, and ground rays
grazing the 0.05 m and sky-distance limits.  A float decision may decline to
decide; it must never decide differently from the double arithmetic.

float32 FMA is emulated as one float64 operation rounded to float32 (the
product of two float32 values is exact in float64); the rare double rounding
this allows is far inside the margins under test.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def fma32(a, b, c):
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(F32)


def certain_miss(oc, rr, d):
    """The kernel's test: True where the float discriminant is below -margin."""
    occ = oc[:, 0] * oc[:, 0] + oc[:, 1] * oc[:, 1] + oc[:, 2] * oc[:, 2]
    f = oc.astype(F32)
    df = d.astype(F32)
    c = (rr - occ).astype(F32)
    margin = (2.0 ** -18 * (occ + rr)).astype(F32)
    b = fma32(f[:, 2], df[:, 2], fma32(f[:, 1], df[:, 1], f[:, 0] * df[:, 0]))
    return fma32(b, b, c) < -margin


def double_disc(oc, rr, d):
    """sphere_hit's discriminant, in the simulator's order."""
    occ = oc[:, 0] * oc[:, 0] + oc[:, 1] * oc[:, 1] + oc[:, 2] * oc[:, 2]
    b = oc[:, 0] * d[:, 0] + oc[:, 1] * d[:, 1] + oc[:, 2] * d[:, 2]
    return b * b - occ + rr


def unit(v):
    return v / np.linalg.norm(v, axis=1, keepdims=True)


def tangent_cases(rng, n):
    """Rays from the origin passing the sphere centre c at distance r (1 + eps)."""
    dist = 10.0 ** rng.uniform(-3, 6, n)
    r = dist * 10.0 ** rng.uniform(-4, -0.05, n)
    c = unit(rng.normal(size=(n, 3))) * dist[:, None]
    eps = rng.choice([-1, 1], n) * 10.0 ** rng.uniform(-12, -3, n)
    miss = r * (1 + eps)                              # closest approach
    ang = np.arcsin(np.clip(miss / dist, -1, 1))
    axis = unit(c)
    perp = unit(np.cross(axis, rng.normal(size=(n, 3))))
    d = unit(axis * np.cos(ang)[:, None] + perp * np.sin(ang)[:, None])
    return -c, r * r, d                               # oc = origin - centre


def test_float_miss_test_never_contradicts_the_double_discriminant():
    rng = np.random.default_rng(20261202)
    decided = 0
    for _ in range(20):
        oc, rr, d = tangent_cases(rng, 200_000)
        miss = certain_miss(oc, rr, d)
        disc = double_disc(oc, rr, d)
        bad = miss & (disc >= 0)
        assert not bad.any(), f"{bad.sum()} float misses with a double discriminant >= 0"
        decided += int(miss.sum())
    # wide random rays: almost every one is ruled out in float
    oc = rng.normal(size=(200_000, 3)) * 10.0 ** rng.uniform(-1, 4, (200_000, 1))
    rr = (np.linalg.norm(oc, axis=1) * 10.0 ** rng.uniform(-3, -1, 200_000)) ** 2
    d = unit(rng.normal(size=(200_000, 3)))
    miss = certain_miss(oc, rr, d)
    assert not (miss & (double_disc(oc, rr, d) >= 0)).any()
    assert miss.mean() > 0.95 and decided > 50_000   # both outcomes occur near tangency too


def ground_decision(oz, dz, best):
    """The kernel's float ground test: 1 certain hit, 0 certain miss, -1 undecided."""
    tf = (-(oz.astype(F32)) / dz.astype(F32)).astype(np.float64)
    hit = (tf > 0.05 * (1 + 1e-6)) & (tf < best * (1 - 1e-6))
    miss = (tf < 0.05 * (1 - 1e-6)) | (tf > best * (1 + 1e-6))
    return np.where(hit, 1, np.where(miss, 0, -1))


def test_float_ground_test_never_contradicts_the_double_division():
    rng = np.random.default_rng(7)
    n = 2_000_000
    dz = -(10.0 ** rng.uniform(-5, 0, n))
    best = rng.choice([30.0, 120.0, 300.0, 1e4], n)
    # heights that put t = -oz/dz near 0.05, near best, and anywhere
    target = np.where(rng.uniform(size=n) < 0.4, 0.05, np.where(rng.uniform(size=n) < 0.6, best, 0.0))
    t_want = np.where(target > 0, target * (1 + rng.choice([-1, 1], n) * 10.0 ** rng.uniform(-12, -4, n)),
                      10.0 ** rng.uniform(-3, 5, n))
    oz = -t_want * dz
    t = (0 - oz) / dz
    exact = (t > 0.05) & (t < best)
    dec = ground_decision(oz, dz, best)
    assert not ((dec == 1) & ~exact).any() and not ((dec == 0) & exact).any()
    assert (dec >= 0).mean() > 0.3                    # most cases sit at a limit on purpose


def float_rotate(q, v):
    """tb_camera_float.h's rotation: tb_rotate's formula in float, each
    multiply-add fused (one rounding) as the header writes it."""
    qw, qx, qy, qz = (q[:, i:i + 1].astype(F32) for i in range(4))
    vx, vy, vz = (v[None, :, i].astype(F32) for i in range(3))

    def fma(a, b, c):
        return (np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(c, np.float64)).astype(F32)

    cx, cy, cz = fma(qy, vz, -(qz * vy)), fma(qz, vx, -(qx * vz)), fma(qx, vy, -(qy * vx))
    tx, ty, tz = cx * F32(2), cy * F32(2), cz * F32(2)
    ax, ay, az = fma(tx, qw, vx), fma(ty, qw, vy), fma(tz, qw, vz)
    return ax + fma(qy, tz, -(qz * ty)), ay + fma(qz, tx, -(qx * tz)), az + fma(qx, ty, -(qy * tx))


def double_rotate(q, v):
    """tb_rotate (sim_internal.h:85) in double, the kernel's double path."""
    qw, qx, qy, qz = (q[:, i:i + 1] for i in range(4))
    vx, vy, vz = (v[None, :, i] for i in range(3))
    cx, cy, cz = qy * vz - qz * vy, qz * vx - qx * vz, qx * vy - qy * vx
    tx, ty, tz = cx * 2, cy * 2, cz * 2
    ax, ay, az = vx + tx * qw, vy + ty * qw, vz + tz * qw
    return ax + (qy * tz - qz * ty), ay + (qz * tx - qx * tz), az + (qx * ty - qy * tx)


def test_float_camera_direction_error_is_inside_the_assumed_bound():
    """tb_camera_float.h assumes the float direction is within TBF_ED = 8e-6
    of the double one per component (35 * 2^-24 = 2.1e-6 derived).  Measured
    here over every camera ray of the sensor tables and 256 random unit
    attitudes (with the 1e-9 slack in |q|^2 the kernel allows)."""
    import ctypes

    import oracle

    lib = oracle._sensor_port()
    lib.oracle_sensor_rays.restype = None
    lib.oracle_sensor_rays.argtypes = [ctypes.c_void_p] * 3
    lidar = np.zeros(3 * 4096)
    blocked = np.zeros(4096, np.uint8)
    cams = np.zeros(3 * 16384)
    lib.oracle_sensor_rays(lidar.ctypes.data, blocked.ctypes.data, cams.ctypes.data)
    v = cams.reshape(-1, 3)
    rng = np.random.default_rng(3)
    q = unit(rng.normal(size=(256, 4))) * (1 + rng.uniform(-4e-10, 4e-10, (256, 1)))
    worst = 0.0
    for chunk in np.array_split(np.arange(256), 16):
        fd = float_rotate(q[chunk], v)
        dd = double_rotate(q[chunk], v)
        worst = max(worst, max(float(np.max(np.abs(f.astype(np.float64) - d))) for f, d in zip(fd, dd)))
    print(f"\nfloat camera direction: largest component error {worst:.3e} (assumed bound 8e-6)")
    assert worst <= 2.1e-6

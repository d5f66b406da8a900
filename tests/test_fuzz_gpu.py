"""Special-value batches on the GPU, through the C ABI: observations and
missions mixed with NaN, +-inf, -0.0, subnormals, clamp boundaries and LiDAR
ranges at 0, 0.5, 120 and its float neighbours; cameras random, all 0 or all
255.  Each kernel is held to its usual bar: the 142 features against the
CPU oracle (exact, LiDAR means within 1e-6 + 1e-5|ref|), the onboard values
exactly against the correctly rounded reference build, the learner inputs
against the reference's own GPU kernels (and the numpy restatement)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import turbinator_c_b200 as tb
from tests.parity import check_features
from tests.test_actor_inputs_gpu import _outputs
from tests.test_onboard_gpu import run_onboard

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

F32 = np.float32
SPECIAL = [np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-45, -1e-45, 1.17549435e-38, 0.5, -0.5, 1.0, -1.0,
           0.75, 0.7500001, 0.25, 120.0, float(np.nextafter(F32(120), F32(0))),
           float(np.nextafter(F32(120), F32(200))), 3.4e38, -3.4e38, 300.0, 30.0, 0.05, 11.5, 0.35]


def special_batch(seed: int, n: int, rate: float, odd_attitudes: bool = True):
    rng = np.random.default_rng(seed)
    pool = np.array(SPECIAL, F32)

    def mixed(shape, lo, hi):
        v = rng.uniform(lo, hi, shape).astype(F32)
        pick = rng.random(shape) < rate
        v[pick] = pool[rng.integers(0, len(pool), pick.sum())]
        return v

    obs = mixed((n, 4148), -2.0, 2.0)
    obs[:, 48:4144] = (0.5 * 600.0 ** rng.random((n, 4096))).astype(F32)
    pick = rng.random((n, 4096)) < rate
    obs[:, 48:4144][pick] = pool[rng.integers(0, len(pool), pick.sum())]
    # unit attitude for most aircraft, specials for some
    q = rng.normal(size=(n, 4)).astype(F32)
    obs[:, 6:10] = q / np.linalg.norm(q, axis=1, keepdims=True)
    if odd_attitudes:
        odd = rng.random(n) < rate
        obs[odd, 6:10] = mixed((odd.sum(), 4), -1.0, 1.0)
    mission = mixed((n, 10), -1.0, 1.0)
    cams = rng.integers(0, 256, (n, 16384), dtype=np.uint8)
    cams[: n // 8] = 0
    cams[n // 8: n // 4] = 255
    return obs, mission, cams


@pytest.mark.parametrize("kernel", [-1, 1])   # staged, flat
@pytest.mark.parametrize("seed,rate", [(1, 0.02), (2, 0.2), (3, 0.6)])
def test_features_on_special_values(seed, rate, kernel):
    obs, mission, cams = special_batch(seed, 2048, rate)
    d = [torch.from_numpy(x).cuda() for x in (obs, mission, cams)]
    out = torch.full((2048, 142), float("nan"), device="cuda")
    assert tb.launch(*d, out, 2048, None, flat=kernel) == 1
    assert tb.tb_cuda_synchronize(None) == 1
    check_features(out.cpu().numpy(), oracle.features(obs, mission, cams), f"special rate {rate} flat={kernel}")


@pytest.mark.parametrize("seed,rate", [(4, 0.02), (5, 0.2), (6, 0.6)])
def test_onboard_on_special_values(seed, rate):
    obs, mission, _ = special_batch(seed, 2048, rate)
    # half the aircraft on scanning missions, so the LiDAR passes see the specials
    mission[0::4, 5] = 1.0
    mission[1::4, 4] = 1.0
    mission[1::4, 5] = -0.5
    gpu = run_onboard(obs, mission)
    cr = oracle.onboard_reference_cr(obs, mission)
    # pathological attitudes (a NaN or 120 in the quaternion) can make the
    # reference itself return NaN; NaN must then be NaN here too
    same = (gpu == cr) | (np.isnan(gpu) & np.isnan(cr))
    bad = np.argwhere(~same)
    assert not bad.size, (f"special rate {rate}: {len(bad)} values differ from the correctly rounded "
                          f"reference; first {bad[0].tolist()}: gpu {gpu[tuple(bad[0])]!r} ref {cr[tuple(bad[0])]!r}")
    # (No comparison with the glibc build here: on arguments such as 3.4e38
    # or near a pole of tan, two accurate float libraries can differ by far
    # more than rounding, so only the correctly rounded build is a bar.)


def _same_bits(a, b):
    """float32 arrays equal bit for bit, any NaN matching any NaN."""
    return (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))


@pytest.mark.skipif(not oracle.have_reference_actor_inputs(), reason="reference GPU build absent")
@pytest.mark.parametrize("seed,rate", [(7, 0.02), (8, 0.3)])
def test_actor_inputs_on_special_values(seed, rate):
    """Against the reference's own kernels on the same device buffers: LiDAR
    channels, luma, mission and symlog proprioception bit for bit.  The
    onboard slots equal the correctly rounded reference build (NaN where it
    gives NaN); the reference kernels evaluate them with CUDA's float
    functions, which on arguments like these can differ from correctly
    rounded values by far more than rounding."""
    n = 1024
    obs, mission, cams = special_batch(seed, n, rate, odd_attitudes=False)
    d = [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (obs, mission, cams)]
    mine, theirs = _outputs(n), _outputs(n)
    assert tb.tb_cuda_prepare_actor_inputs_device(*d, *mine, n) == 1
    assert tb.tb_cuda_synchronize(None) == 1
    oracle.actor_inputs_reference_gpu(*d, theirs, n)
    p, mv, tac, pri, lidar, luma = [t.cpu().numpy() for t in mine]
    rp, rmv, rtac, rpri, rlidar, rluma = [t.cpu().numpy() for t in theirs]
    assert _same_bits(lidar, rlidar).all() and _same_bits(luma, rluma).all()
    assert _same_bits(p[:, :52], rp[:, :52]).all() and _same_bits(mv[:, :10], rmv[:, :10]).all()
    onboard = np.concatenate([tac, pri], 1)
    assert _same_bits(onboard, oracle.onboard_reference_cr(obs, mission)).all()
    assert _same_bits(p[:, 52:], onboard).all() and _same_bits(mv[:, 10:], onboard).all()

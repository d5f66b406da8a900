"""Guard rows around every streaming output: the stand-in for
compute-sanitizer's out-of-bounds checks, which are closed on this pool.

Each output is allocated with G extra rows before and after the rows a call
may write (plus, for some cases, a 4-byte shift that leaves the rows
unaligned), all filled with a sentinel bit pattern.  The call writes the
inner n rows; afterwards every guard word must still hold the sentinel and the
inner rows must match the oracle.  This covers the index arithmetic of every
kernel that writes through computed row offsets: runs of aircraft per CTA and
their ragged last run, ring wraparound under a capped grid, shuffle-indexed
sector/quadrant stores, the flat one-CTA-per-aircraft kernel, the plain-load
kernel for unaligned rows, the onboard scan kernel's parked results in the
prior rows, the learner-input kernel's six tensors, and the host entry points'
copies back into caller memory.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import turbinator_c_b200 as tb
from tests.parity import check_features

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

G = 3                      # guard rows on each side
SENTINEL = 0x7FC0DEAD      # a quiet-NaN bit pattern no kernel produces
BATCHES = [1, 3, 297, 2369, 9001]


class Guarded:
    """A [n, width] float32 view inside a device (or host) buffer of
    (n + 2G) rows (+ shift words), every word set to SENTINEL."""

    def __init__(self, n, width, shift=0, device="cuda", pinned=False):
        self.n, self.width, self.shift = n, width, shift
        words = (n + 2 * G) * width + shift
        if device == "cuda":
            self.buf = torch.full((words,), SENTINEL, dtype=torch.int32, device="cuda")
        else:
            t = torch.full((words,), SENTINEL, dtype=torch.int32)
            self.buf = t.pin_memory() if pinned else t
        self.start = G * width + shift

    @property
    def ptr(self):
        return self.buf.data_ptr() + 4 * self.start

    @property
    def host(self):
        """The inner rows as a numpy float32 array (a view for host buffers)."""
        a = self.buf.numpy() if self.buf.device.type == "cpu" else self.buf.cpu().numpy()
        return a[self.start:self.start + self.n * self.width].view(np.float32).reshape(self.n, self.width)

    def check(self, what):
        a = self.buf.cpu().numpy() if self.buf.device.type == "cuda" else self.buf.numpy()
        head = a[:self.start]
        tail = a[self.start + self.n * self.width:]
        bad_head = np.flatnonzero(head != SENTINEL)
        bad_tail = np.flatnonzero(tail != SENTINEL)
        assert not bad_head.size and not bad_tail.size, (
            f"{what}: {len(bad_head)} words written before row 0 (first at word {bad_head[:1]} of "
            f"{len(head)}), {len(bad_tail)} after row n-1 (first at word {bad_tail[:1]} past the end)")


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


# ---------------------------------------------------------------- features

KERNELS = {
    "auto": {},
    "staged": {"flat": -1},
    "flat": {"flat": 1},
    "direct": {"force_direct": True},
}


@pytest.mark.parametrize("kernel", sorted(KERNELS))
@pytest.mark.parametrize("batch", BATCHES)
def test_feature_rows_stay_inside(kernel, batch):
    obs, mission, cams, _ = tb.generate(41, 0, batch)
    expected = oracle.features(obs, mission, cams)
    for shift in (0, 1):
        out = Guarded(batch, 142, shift)
        torch.cuda.synchronize()
        opts = KERNELS[kernel]
        if opts:
            assert tb.launch(_dev(obs), _dev(mission), _dev(cams), out.ptr, batch, None, **opts) == 1
        else:
            assert tb.tb_cuda_extract_features_device(_dev(obs), _dev(mission), _dev(cams), out.ptr, batch) == 1
        assert tb.tb_cuda_synchronize() == 1
        out.check(f"features {kernel} B={batch} shift={shift}")
        check_features(out.host, expected, f"features {kernel} B={batch} shift={shift}")


@pytest.mark.parametrize("grid_limit", [1, 5])
@pytest.mark.parametrize("batch", [297, 2369])
def test_feature_rows_stay_inside_under_a_capped_grid(grid_limit, batch):
    obs, mission, cams, _ = tb.generate(42, 0, batch)
    out = Guarded(batch, 142)
    torch.cuda.synchronize()
    assert tb.launch(_dev(obs), _dev(mission), _dev(cams), out.ptr, batch, None, grid_limit=grid_limit) == 1
    assert tb.tb_cuda_synchronize() == 1
    out.check(f"features grid={grid_limit} B={batch}")
    check_features(out.host, oracle.features(obs, mission, cams), f"features grid={grid_limit} B={batch}")


def test_feature_rows_stay_inside_with_unaligned_inputs():
    """Input rows 4 bytes past a 16-byte boundary take the plain-load kernel."""
    batch = 297
    obs, mission, cams, _ = tb.generate(43, 0, batch)
    flat = torch.zeros(batch * 4148 + 1, device="cuda")
    flat[1:] = _dev(obs).reshape(-1)
    out = Guarded(batch, 142, 1)
    torch.cuda.synchronize()
    assert tb.tb_cuda_extract_features_device(flat.data_ptr() + 4, _dev(mission), _dev(cams), out.ptr, batch) == 1
    assert tb.tb_cuda_synchronize() == 1
    out.check("features unaligned inputs")
    check_features(out.host, oracle.features(obs, mission, cams), "features unaligned inputs")


@pytest.mark.parametrize("direct", [False, True])
@pytest.mark.parametrize("batch", [1, 3, 297, 2369])
def test_f32_camera_feature_rows_stay_inside(direct, batch):
    obs, mission, cams, camf = tb.generate(44, 0, batch, f32_cameras=True)
    out = Guarded(batch, 142, 1)
    torch.cuda.synchronize()
    assert tb.launch_f32cam(_dev(obs), _dev(mission), _dev(camf), out.ptr, batch, force_direct=direct) == 1
    assert tb.tb_cuda_synchronize() == 1
    out.check(f"f32cam direct={direct} B={batch}")
    check_features(out.host, oracle.features(obs, mission, oracle.quantize_cameras(camf)),
                   f"f32cam direct={direct} B={batch}")


# ---------------------------------------------------------------- onboard

def _all_scanning(mission):
    m = np.array(mission, copy=True)
    m[0::2, 5] = 1.0       # dodge
    m[1::2, 4] = 1.0       # slalom
    m[1::2, 5] = -0.5
    return m


@pytest.mark.parametrize("scanning", [False, True])
@pytest.mark.parametrize("batch", BATCHES)
def test_onboard_rows_stay_inside(scanning, batch):
    obs, mission, _, _ = tb.generate(45, 0, batch)
    if scanning:
        mission = _all_scanning(mission)
    tac, pri = Guarded(batch, 24, 1), Guarded(batch, 15, 1)
    torch.cuda.synchronize()
    assert tb.tb_cuda_extract_onboard_device(_dev(obs), _dev(mission), tac.ptr, pri.ptr, batch) == 1
    assert tb.tb_cuda_synchronize() == 1
    tac.check(f"tactical B={batch} scanning={scanning}")
    pri.check(f"prior B={batch} scanning={scanning}")
    got = np.concatenate([tac.host, pri.host], axis=1)
    assert np.array_equal(got, oracle.onboard_reference_cr(obs, mission)), f"onboard B={batch}"


# ---------------------------------------------------------------- learner inputs

@pytest.mark.parametrize("batch", [1, 3, 297, 2369])
def test_learner_input_rows_stay_inside(batch):
    obs, mission, cams, _ = tb.generate(46, 0, batch)
    mission = _all_scanning(mission) if batch > 3 else mission
    widths = (91, 49, 24, 15, 6 * 2048, 16384)
    # LiDAR channels and luma need 16-byte aligned rows: shift only the others
    outs = [Guarded(batch, w, 1 if w < 1000 else 0) for w in widths]
    torch.cuda.synchronize()
    assert tb.tb_cuda_prepare_actor_inputs_device(_dev(obs), _dev(mission), _dev(cams),
                                                  *[o.ptr for o in outs], batch) == 1
    assert tb.tb_cuda_synchronize() == 1
    names = ("proprio", "mission", "tactical", "prior", "lidar", "luma")
    for o, name in zip(outs, names):
        o.check(f"learner {name} B={batch}")
    proprio, mvec, tac, pri, lidar, luma = (o.host for o in outs)
    assert np.array_equal(np.concatenate([tac, pri], 1), oracle.onboard_reference_cr(obs, mission))
    cpu = oracle.actor_inputs_cpu(obs, mission, cams, tac, pri)
    assert np.array_equal(lidar.view(np.uint32), cpu["lidar"].reshape(batch, -1).view(np.uint32))
    assert np.array_equal(luma.view(np.uint32), cpu["luma"].view(np.uint32))
    assert np.array_equal(mvec[:, :10].view(np.uint32), cpu["mission"][:, :10].view(np.uint32))
    assert np.array_equal(proprio[:, 52:76], tac) and np.array_equal(mvec[:, 34:], pri)
    err = np.abs(proprio[:, :52].astype(np.float64) - cpu["proprio"][:, :52])
    assert np.all(err <= 1e-6 + 1e-5 * np.abs(cpu["proprio"][:, :52]))


# ---------------------------------------------------------------- host entry points

@pytest.mark.parametrize("pinned", [False, True])
@pytest.mark.parametrize("batch", BATCHES)
def test_host_abi_rows_stay_inside(pinned, batch):
    obs, mission, cams, _ = tb.generate(47, 0, batch, pinned=pinned)
    out = Guarded(batch, 142, 0, device="cpu", pinned=pinned)
    with tb.FeatureBatch(0, batch) as fb:
        assert fb.extract(obs, mission, cams, batch, out.ptr) == 1, fb.error()
    out.check(f"host ABI pinned={pinned} B={batch}")
    check_features(out.host, oracle.features(np.asarray(obs), np.asarray(mission), np.asarray(cams)),
                   f"host ABI pinned={pinned} B={batch}")


@pytest.mark.parametrize("batch", [1, 3, 64])
def test_noalloc_host_rows_stay_inside(batch):
    obs, mission, cams, _ = tb.generate(48, 0, batch)
    out = Guarded(batch, 142, 1, device="cpu")
    assert tb.tb_cuda_extract_features_host_noalloc(obs, mission, cams, batch, out.ptr) == 1
    out.check(f"no-alloc B={batch}")
    check_features(out.host, oracle.features(obs, mission, cams), f"no-alloc B={batch}")

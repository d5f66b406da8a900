"""GPU parity: the sm_100a kernels, called through the C ABI, against the CPU
oracle (itself pinned to the reference in test_oracle.py).

Exactness classes and tolerances are in tests/parity.py: bit-exact for the
scalar/mission/camera features, |d| <= 1e-6 + 1e-5*|ref| for LiDAR means.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle
import turbinator_c_b200 as tb
from tests.golden import fixtures
from tests.parity import check_features

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_device(obs, mission, cams, *, stream=None, **opts):
    """Features via tb_cuda_extract_features_device (or the launch hook with opts)."""
    n = obs.shape[0]
    d_obs, d_mis = _dev(obs), _dev(mission)
    d_cam = _dev(cams) if cams is not None else None
    d_out = torch.full((n, 142), float("nan"), device="cuda")
    torch.cuda.synchronize()  # inputs and the NaN fill are complete before any stream reads them
    if opts:
        ok = tb.launch(d_obs, d_mis, d_cam, d_out, n, stream, **opts)
    else:
        ok = tb.tb_cuda_extract_features_device(d_obs, d_mis, d_cam, d_out, n, stream)
    assert ok == 1
    assert tb.tb_cuda_synchronize(stream) == 1
    return d_out.cpu().numpy()


def test_reference_known_answer_via_host_abi():
    """The reference's own CUDA parity test (tests/test_cuda_features.c:9-56)
    through the same host entry point, plus the stricter exactness classes."""
    obs, mission, cams = fixtures.reference_known_answer_inputs()
    out = np.empty((3, 142), np.float32)
    with tb.FeatureBatch(int(os.environ.get("TB_CUDA_TEST_DEVICE", "0")), 3) as fb:
        assert fb.extract(obs, mission, cams, 3, out) == 1, fb.error()
        assert fb.error() == ""
    expected = np.load(os.path.join(GOLDEN, "ref_known_answer.npz"))["features"]
    assert np.all(np.isfinite(out)) and np.max(np.abs(out - expected)) <= 2e-5
    check_features(out, expected, "known-answer")


@pytest.mark.parametrize("name", sorted(fixtures.SEEDED_CASES))
def test_seeded_goldens(name):
    seed, total, count, stress = fixtures.SEEDED_CASES[name]
    obs, mission, cams, _ = tb.generate(seed, 0, count, total=total, stress=stress)
    expected = np.load(os.path.join(GOLDEN, f"{name}.npz"))["features"]
    check_features(run_device(obs, mission, cams), expected, name)


@pytest.mark.parametrize("kernel", [-1, 1])
def test_edge_values_with_and_without_cameras(kernel):
    g = np.load(os.path.join(GOLDEN, "edge_cases.npz"))
    check_features(run_device(g["obs"], g["mission"], g["cameras"], flat=kernel), g["features"], "edge")
    check_features(run_device(g["obs"], g["mission"], None, flat=kernel), g["features_no_camera"],
                   "edge/no-camera")


def test_reference_training_facts_on_gpu():
    obs = np.zeros((2, 4148), np.float32)
    mission = np.zeros((2, 10), np.float32)
    cams = np.full((2, 16384), 128, np.uint8)
    mission[:, 0] = 1.0
    obs[:, 2] = 2.0
    mission[1, 6] = 1.0
    mission[1, 7] = 0.9
    f = run_device(obs, mission, cams)
    assert f[0, 2] > 0 and f[0, 126] > 0 and f[1, 59] == 0.0


@pytest.mark.parametrize("config", [1, 2])
def test_full_config_parity(config):
    seed, batch, _ = tb.CONFIGS[config]
    obs, mission, cams, _ = tb.generate(seed, 0, batch)
    check_features(run_device(obs, mission, cams), oracle.features(obs, mission, cams), f"config{config}")


def test_config4_stress_quarters_full_size():
    seed, batch, _ = tb.CONFIGS[4]
    obs, mission, cams, _ = tb.generate(seed, 0, batch, stress=True)
    out = run_device(obs, mission, cams)
    check_features(out, oracle.features(obs, mission, cams), "config4")
    q = batch // 4
    assert np.all(out[0:q:2, 126:] == 0.0) and np.all(out[1:q:2, 126:] == 1.0)  # (a)
    assert np.all(out[q:2 * q, 62:126] == 1.0)                                   # (b) exactly
    d = out[3 * q:, 62:126]
    assert np.all(d == d[0, 0])                                                   # (d) identical


# Staged kernel: 296 CTAs are resident at once, and batches past that go in runs of
# ceil(B / 296) aircraft per CTA (at most 8), so 297, 593, 2,367, 2,369 and 9,001 end in a
# shorter run.  Batches of up to 16 aircraft per SM (2,368) take the flat kernel by default;
# each size runs on the default choice and on both kernels forced.
@pytest.mark.parametrize("kernel", [0, -1, 1])
@pytest.mark.parametrize("batch", [1, 2, 3, 7, 147, 148, 149, 295, 296, 297, 592, 593, 1023, 1025,
                                   2367, 2368, 2369, 9001])
def test_ragged_batch_sizes(batch, kernel):
    obs, mission, cams, _ = tb.generate(21, 0, batch)
    opts = {"flat": kernel} if kernel else {}
    check_features(run_device(obs, mission, cams, **opts), oracle.features(obs, mission, cams),
                   f"B={batch} flat={kernel}")


@pytest.mark.parametrize("grid_limit", [1, 2, 5])
def test_many_samples_per_cta_ring_wraparound(grid_limit):
    """Few CTAs -> each walks the shared-memory ring many times (phase flips)."""
    obs, mission, cams, _ = tb.generate(22, 0, 301)
    out = run_device(obs, mission, cams, grid_limit=grid_limit)
    check_features(out, oracle.features(obs, mission, cams), f"grid={grid_limit}")


def test_direct_kernel_and_unaligned_rows():
    obs, mission, cams, _ = tb.generate(23, 0, 200)
    expected = oracle.features(obs, mission, cams)
    check_features(run_device(obs, mission, cams, force_direct=True), expected, "direct")
    # rows that start 4 bytes past a 16-byte boundary take the direct kernel
    n = obs.shape[0]
    flat = torch.zeros(n * 4148 + 1, device="cuda")
    flat[1:] = _dev(obs).reshape(-1)
    camflat = torch.zeros(n * 16384 + 3, dtype=torch.uint8, device="cuda")
    camflat[3:] = _dev(cams).reshape(-1)
    d_out = torch.zeros((n, 142), device="cuda")
    assert tb.tb_cuda_extract_features_device(flat.data_ptr() + 4, _dev(mission), camflat.data_ptr() + 3,
                                              d_out, n) == 1
    assert tb.tb_cuda_synchronize() == 1
    check_features(d_out.cpu().numpy(), expected, "unaligned")


def test_non_default_stream_and_null_stream():
    obs, mission, cams, _ = tb.generate(24, 0, 513)
    expected = oracle.features(obs, mission, cams)
    s = torch.cuda.Stream()
    check_features(run_device(obs, mission, cams, stream=s), expected, "stream")
    check_features(run_device(obs, mission, cams, stream=None), expected, "legacy stream")


def test_host_abi_contract():
    obs, mission, cams, _ = tb.generate(25, 0, 2500)
    expected = oracle.features(obs, mission, cams)
    with tb.FeatureBatch(0, 2500) as fb:  # above the reference's old 1024 cap
        out = np.zeros((2500, 142), np.float32)
        assert fb.extract(obs, mission, cams, 2500, out) == 1, fb.error()
        check_features(out, expected, "host")
        part = np.zeros((17, 142), np.float32)
        assert fb.extract(obs[100:117], mission[100:117], cams[100:117], 17, part) == 1
        check_features(part, expected[100:117], "host/part")
        assert fb.extract(obs, mission, cams, 2501, out) == 0          # count > max_batch
        assert fb.extract(obs, mission, None, 10, out) == 0           # cameras required
        assert fb.extract(obs, mission, cams, 0, out) == 0
    assert tb.tb_cuda_feature_batch_create(0, 0) is None
    assert tb.tb_cuda_feature_batch_create(10_000, 4) is None           # invalid device


def test_host_abi_pinned_and_chunked():
    """Page-locked buffers take the streamed, chunked path (> 1 chunk here)."""
    n = 20000
    obs, mission, cams, _ = tb.generate(26, 0, n, pinned=True)
    out = torch.zeros((n, 142), dtype=torch.float32, pin_memory=True).numpy()
    with tb.FeatureBatch(0, n) as fb:
        assert fb.extract(obs, mission, cams, n, out) == 1, fb.error()
    check_features(out, oracle.features(np.asarray(obs), np.asarray(mission), np.asarray(cams)), "pinned")


def test_bounded_pipeline_wait_reports_and_recovers():
    """A sample whose copies are withheld makes the consumers' bounded waits
    expire: the launch ends, tb_cuda_synchronize reports it once, and the
    device keeps working."""
    obs, mission, cams, _ = tb.generate(27, 0, 64)
    d_obs, d_mis, d_cam = _dev(obs), _dev(mission), _dev(cams)
    d_out = torch.zeros((64, 142), device="cuda")
    assert tb.take_status() == 0
    assert tb.launch(d_obs, d_mis, d_cam, d_out, 64, None, wait_ns=20_000_000, stall_sample=5) == 1
    assert tb.tb_cuda_synchronize() == 0
    assert tb.tb_cuda_synchronize() == 1          # reported once, then cleared
    check_features(run_device(obs, mission, cams), oracle.features(obs, mission, cams), "after-timeout")


@pytest.mark.parametrize("pin_in,pin_out", [(False, False), (True, False), (False, True)])
def test_host_abi_buffer_kinds_threaded(pin_in, pin_out):
    """Pageable inputs go through the handle's page-locked staging on several
    host threads; page-locked ones are streamed directly; either output kind."""
    n = 9000
    obs, mission, cams, _ = tb.generate(28, 0, n, pinned=pin_in)
    out = (torch.zeros((n, 142), dtype=torch.float32, pin_memory=True).numpy() if pin_out
           else np.zeros((n, 142), np.float32))
    with tb.FeatureBatch(0, n) as fb:
        assert fb.extract(obs, mission, cams, n, out) == 1, fb.error()
        expected = oracle.features(np.asarray(obs), np.asarray(mission), np.asarray(cams))
        check_features(out, expected, f"host pin_in={pin_in} pin_out={pin_out}")
        # a second, smaller call reuses the same staging
        part = np.zeros((777, 142), np.float32)
        assert fb.extract(obs[1000:1777], mission[1000:1777], cams[1000:1777], 777, part) == 1
        check_features(part, expected[1000:1777], "host second call")


def test_trainer_style_small_calls():
    """The trainer's pattern: a small persistent batch extracted again and
    again from pageable buffers (src/trainer/main.c:526-673)."""
    obs, mission, cams, _ = tb.generate(29, 0, 32)
    expected = oracle.features(obs, mission, cams)
    out = np.zeros((32, 142), np.float32)
    with tb.FeatureBatch(0, 32) as fb:
        for count in (32, 8, 1, 32):
            out[:] = 0
            assert fb.extract(obs, mission, cams, count, out) == 1, fb.error()
            check_features(out[:count], expected[:count], f"trainer count={count}")


@pytest.mark.parametrize("devices,n", [([0, 0], 5001), ([0, 0, 0], 3), ([0, 0, 0], 12000)])
def test_multi_device_handle_shards_and_gathers(devices, n):
    """A sample-sharded handle (the same GPU listed several times here; the
    slicing and gather are the same as over distinct GPUs)."""
    obs, mission, cams, _ = tb.generate(30, 0, n)
    out = np.zeros((n, 142), np.float32)
    with tb.FeatureBatch(devices, n) as fb:
        assert fb.extract(obs, mission, cams, n, out) == 1, fb.error()
    check_features(out, oracle.features(obs, mission, cams), f"multi {devices}")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_multi_device_handle_on_distinct_gpus():
    """The sample-sharded handle over every visible GPU: each device holds its
    own staging and runs its slice concurrently; rows come back in order."""
    devices = list(range(torch.cuda.device_count()))
    n = 9001
    obs, mission, cams, _ = tb.generate(33, 0, n)
    expected = oracle.features(obs, mission, cams)
    out = np.zeros((n, 142), np.float32)
    with tb.FeatureBatch(devices, n) as fb:
        for count in (n, 5, len(devices) - 1 or 1):
            out[:] = 0
            assert fb.extract(obs, mission, cams, count, out) == 1, fb.error()
            check_features(out[:count], expected[:count], f"distinct GPUs {devices} count={count}")


def test_sharded_device_entry_point():
    """tb_cuda_extract_features_device_sharded: contiguous slices of one batch
    as shards (here all on device 0, one of them empty), each with its own
    pointers and stream; the caller's current device is kept."""
    n = 3001
    obs, mission, cams, _ = tb.generate(34, 0, n)
    expected = oracle.features(obs, mission, cams)
    d_obs, d_mis, d_cam = _dev(obs), _dev(mission), _dev(cams)
    out = torch.full((n, 142), float("nan"), device="cuda")
    cuts = [0, 1000, 1000, 2999, n]
    sl = lambda t, i: t[cuts[i]:cuts[i + 1]]
    streams = [torch.cuda.Stream() for _ in range(4)]
    assert tb.tb_cuda_extract_features_device_sharded(
        [0] * 4, [sl(d_obs, i) for i in range(4)], [sl(d_mis, i) for i in range(4)],
        [sl(d_cam, i) for i in range(4)], [sl(out, i) for i in range(4)],
        [cuts[i + 1] - cuts[i] for i in range(4)], streams) == 1
    assert torch.cuda.current_device() == 0
    for s in streams:
        assert tb.tb_cuda_synchronize(s.cuda_stream) == 1
    check_features(out.cpu().numpy(), expected, "sharded")
    # rejected: unknown device, NULL pointer of a non-empty shard
    assert tb.tb_cuda_extract_features_device_sharded([10_000], [d_obs], [d_mis], None, [out], [n]) == 0
    assert tb.tb_cuda_extract_features_device_sharded([0], [None], [d_mis], None, [out], [n]) == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_sharded_device_entry_point_on_distinct_gpus():
    devices = list(range(torch.cuda.device_count()))
    n = 4099
    obs, mission, cams, _ = tb.generate(35, 0, n)
    expected = oracle.features(obs, mission, cams)
    from turbinator_c_b200.shard import shard_range
    ranges = [shard_range(n, r, len(devices)) for r in range(len(devices))]
    ins = [[torch.from_numpy(x[f:f + c]).to(f"cuda:{d}") for x in (obs, mission, cams)]
           for d, (f, c) in zip(devices, ranges)]
    outs = [torch.full((c, 142), float("nan"), device=f"cuda:{d}") for d, (f, c) in zip(devices, ranges)]
    assert tb.tb_cuda_extract_features_device_sharded(devices, [i[0] for i in ins], [i[1] for i in ins],
                                                      [i[2] for i in ins], outs, [c for _, c in ranges]) == 1
    for d in devices:
        with torch.cuda.device(d):
            assert tb.tb_cuda_synchronize(None) == 1
    got = np.concatenate([o.cpu().numpy() for o in outs])
    check_features(got, expected, f"sharded over {devices}")


def test_multi_device_handle_rejects_bad_devices():
    assert tb.tb_cuda_feature_batch_create_multi([0, 10_000], 16) is None
    assert tb.tb_cuda_feature_batch_create_multi([], 16) is None
    obs, mission, cams, _ = tb.generate(31, 0, 4)
    check_features(run_device(obs, mission, cams), oracle.features(obs, mission, cams), "after bad multi create")


def test_pipeline_timeout_is_reported_only_on_its_own_stream():
    """Each stream has its own status word: a launch whose bounded waits
    expire (one aircraft's copies withheld, 20 ms limit) on stream A is
    reported by tb_cuda_synchronize(A) alone, once.  A handle working on
    another host thread meanwhile and afterwards, and callers synchronising
    other streams, see no failure."""
    import threading

    obs, mission, cams, _ = tb.generate(32, 0, 16)
    d_obs, d_mis, d_cam = _dev(obs), _dev(mission), _dev(cams)
    d_out = torch.zeros((16, 142), device="cuda")
    expected = oracle.features(obs, mission, cams)
    stream_a, stream_b = torch.cuda.Stream(), torch.cuda.Stream()
    assert tb.take_status(stream_a) == 0 and tb.take_status(stream_b) == 0 and tb.take_status() == 0
    stalled = threading.Event()
    results = {}

    def caller_a():
        torch.cuda.set_device(0)
        ok = tb.launch(d_obs, d_mis, d_cam, d_out, 16, stream_a, wait_ns=20_000_000, stall_sample=3)
        stream_a.synchronize()  # the expiry is recorded in A's word by now
        results["a_launch"] = ok
        stalled.set()

    def caller_b():
        torch.cuda.set_device(0)
        out = np.zeros((16, 142), np.float32)
        calls = []
        with tb.FeatureBatch(0, 16) as fb:
            calls.append(fb.extract(obs, mission, cams, 16, out))   # while A's kernel waits
            stalled.wait(timeout=30)
            calls.append(fb.extract(obs, mission, cams, 16, out))   # after A's expiry
            results["b_error"] = fb.error()
        results["b_calls"] = calls
        results["b_out"] = out

    threads = [threading.Thread(target=caller_a), threading.Thread(target=caller_b)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=60)
    assert results["a_launch"] == 1
    assert results["b_calls"] == [1, 1], results.get("b_error")
    check_features(results["b_out"], expected, "handle beside a timed-out stream")
    assert tb.tb_cuda_synchronize(stream_b) == 1
    assert tb.tb_cuda_synchronize(None) == 1
    assert tb.tb_cuda_synchronize(stream_a) == 0      # reported to its own stream
    assert tb.tb_cuda_synchronize(stream_a) == 1      # once
    check_features(run_device(obs, mission, cams, stream=stream_a), expected, "stream A after its timeout")


def test_host_abi_buffer_page_locked_only_at_its_start():
    """Observation rows whose first pages are page-locked (cudaHostRegister of
    a prefix) but the rest pageable: the handle must see the buffer as
    pageable and still return every row correct."""
    n = 1200
    obs, mission, cams, _ = tb.generate(33, 0, n)
    prefix = 64 * 4148 * 4 // 4096 * 4096
    cudart = torch.cuda.cudart()
    assert int(cudart.cudaHostRegister(obs.ctypes.data, prefix, 0)) == 0
    try:
        out = np.zeros((n, 142), np.float32)
        with tb.FeatureBatch(0, n) as fb:
            assert fb.extract(obs, mission, cams, n, out) == 1, fb.error()
    finally:
        cudart.cudaHostUnregister(obs.ctypes.data)
    check_features(out, oracle.features(obs, mission, cams), "partly page-locked")

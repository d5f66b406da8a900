#!/usr/bin/env python
"""Benchmark of the batched 142-feature extraction on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1).  A step is one pass of the feature
path over one batch: 65,536 aircraft per GPU (at N = 8 the
whole job is config 3's 524,288), seeded synthetic inputs generated on the
host.  Rank 0 prints one JSON line:

  value      samples/s over all ranks, inputs resident in HBM, timed with CUDA
             events on the launching stream, max over ranks
  e2e        the same metric through the reference-facing host ABI
             tb_cuda_extract_features_host (page-locked host buffers; the
             host->device input copy and device->host feature copy are inside
             every step)
  roofline   achieved HBM GB/s of the kernel (algorithmic bytes / average
             launch time) against the measured copy bandwidth
  cpu_baseline  the reference's own CPU feature code (oracle/_ref) on this
             host's cores, a bounded sample of the same workload (rank 0, N=1)

--impl reference times that reference CPU code alone on all host cores (rank
0 only; other ranks exit at once).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import turbinator_c_b200 as tb  # noqa: E402
from turbinator_c_b200.shard import (SharedHostGather, all_ranks, max_over_ranks, max_over_ranks_list,  # noqa: E402
                                     shard_range, sum_over_ranks)

METRIC = "sensor-feature samples/sec"
UNIT = "samples/s"
BATCH_PER_GPU = 65536
SEED = 2
FALLBACK_HBM_GBS = 6650.0
PROFILE_SUMMARY = os.path.join(ROOT, "profiles", "features_flat_kernel_traffic.txt")
SENSOR_SCENES = 32768
SENSOR_PROFILE = os.path.join(ROOT, "profiles", "sensors_kernel_pipes.txt")
RAYS_PER_SCENE = 4096 + 16384
CHUNKS_RENDER = 4


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--batch", type=int, default=BATCH_PER_GPU, help="aircraft per GPU")
    p.add_argument("--e2e-steps", type=int, default=0, help="host-ABI steps (default: --steps, max 20)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=4.0, help="target wall time of the CPU sample")
    p.add_argument("--no-onboard", action="store_true", help="skip the onboard tactical/prior leg")
    p.add_argument("--no-f32cam", action="store_true", help="skip the FP32-camera entry-point leg")
    p.add_argument("--no-actor-inputs", action="store_true", help="skip the learner-input leg")
    p.add_argument("--no-sensors", action="store_true", help="skip the sensor-rendering leg")
    p.add_argument("--sensor-scenes", type=int, default=SENSOR_SCENES, help="scenes per GPU in the sensor leg")
    p.add_argument("--no-parity", action="store_true", help="skip the oracle check of the timed outputs")
    p.add_argument("--config1-only", action="store_true",
                   help="run only the config-1 latency leg (one GPU) and print its JSON")
    p.add_argument("--actor-inputs-only", action="store_true",
                   help="run only the learner-input entry point on --batch aircraft (one GPU) and print its JSON")
    p.add_argument("--all-scanning", action="store_true",
                   help="with --actor-inputs-only: every mission reads the LiDAR scans (half dodge, half slalom)")
    return p.parse_args()


# ---------------------------------------------------------------- helpers

def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def measured_hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic_per_sample():
    """DRAM bytes per aircraft of the staged kernel from the committed ncu summary."""
    try:
        with open(PROFILE_SUMMARY) as f:
            for line in f:
                if line.startswith("dram_bytes_per_sample:"):
                    return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clock and clock-event reasons of one GPU through NVML while
    active() is true (only samples taken inside timed regions are kept)."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self._on = threading.Event()
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            if visible:
                ids = [v.strip() for v in visible.split(",") if v.strip()]
                idx = int(ids[device_index]) if ids[device_index].isdigit() else device_index
            else:
                idx = device_index
            self._h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._nvml = pynvml
            self.ok = True
        except Exception:  # NVML unavailable: report no clocks rather than guess
            return
        self._t = threading.Thread(target=self._run, args=(period_s,), daemon=True)
        self._t.start()

    def _run(self, period):
        nv = self._nvml
        while not self._stop.is_set():
            if self._on.is_set():
                try:
                    mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                    try:
                        r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                    except AttributeError:
                        r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                    self.samples.append(mhz)
                    self.reasons |= int(r)
                except Exception:
                    pass
            time.sleep(period)

    def active(self, on: bool):
        (self._on.set if on else self._on.clear)()

    def close(self):
        self._stop.set()

    def summary(self):
        if not self.ok:
            return None
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples),
                "source": "nvml"}


def cpu_description():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def time_reference_cpu(obs, mission, cams, target_s: float):
    """Times the reference's tb_train_extract_features_cpu (oracle/_ref, or the
    restated oracle when the reference build is absent) on all host threads
    over a bounded leading sample of the batch.  Returns a dict."""
    import oracle  # test infrastructure: the CPU baseline only

    kind = "reference" if oracle.have_reference() else "port"
    timed = oracle.timed_reference if kind == "reference" else oracle.timed_port
    threads = host_threads()
    n = obs.shape[0]
    probe = min(n, max(threads * 64, 2048))
    out = np.empty((n, 142), np.float32)
    t = timed(obs[:probe], mission[:probe], cams[:probe], out[:probe], threads)
    rate = probe / max(t, 1e-9)
    sample = int(min(n, max(probe, rate * target_s)))
    # repeat passes over the sample until about target_s of wall time is spent
    passes, spent = 0, 0.0
    while passes == 0 or spent < 0.5 * target_s:
        spent += timed(obs[:sample], mission[:sample], cams[:sample], out[:sample], threads)
        passes += 1
    # the same function on one thread, over a smaller leading sample
    one_sample = int(min(n, max(256, rate / max(threads, 1) * target_s / 4)))
    one_t = timed(obs[:one_sample], mission[:one_sample], cams[:one_sample], out[:one_sample], 1)
    return {"value": sample * passes / spent, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"first {sample} of the {n}-aircraft batch x {passes} pass(es), {threads} threads "
                      f"over contiguous ranges, {spent:.2f} s wall; host CPU: {cpu_description()}",
            "single_thread": {"value": one_sample / one_t, "unit": UNIT, "cores": 1,
                              "sample": f"first {one_sample} aircraft, {one_t:.2f} s wall"}}


def scanning_fraction(mission) -> float:
    """Share of aircraft whose mission reads the onboard LiDAR scans (dodge:
    mission[5] > 0.75; slalom: mission[4] > 0.75 and mission[5] <= 0.25)."""
    m = np.nan_to_num(np.asarray(mission, np.float32), nan=0.0, posinf=1.0, neginf=-1.0)
    dodge = m[:, 5] > 0.75
    slalom = (m[:, 4] > 0.75) & ~(m[:, 5] > 0.25)
    return float(np.mean(dodge | slalom))


def onboard_bytes_per_aircraft(frac_scan: float) -> float:
    """Algorithmic bytes of the onboard path: observation head (192 B) and
    mission (40 B) read, 156 B written, plus the two 3,072 B LiDAR blocks of
    aircraft that scan."""
    return 192 + 40 + 156 + frac_scan * 2 * 3072


def all_scanning(mission):
    m = np.array(mission, copy=True)
    m[0::2, 5] = 1.0            # dodge
    m[1::2, 4] = 1.0            # slalom
    m[1::2, 5] = -0.5
    return m


def time_onboard(d_obs, mission_host, count, steps, warmup, stream, dev):
    import torch

    d_mis = torch.from_numpy(np.ascontiguousarray(mission_host)).to(dev)
    tac = torch.empty((count, 24), dtype=torch.float32, device=dev)
    pri = torch.empty((count, 15), dtype=torch.float32, device=dev)
    torch.cuda.synchronize(dev)
    for _ in range(max(warmup, 3)):
        assert tb.tb_cuda_extract_onboard_device(d_obs, d_mis, tac, pri, count, stream) == 1
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        tb.tb_cuda_extract_onboard_device(d_obs, d_mis, tac, pri, count, stream)
    end.record(stream)
    torch.cuda.synchronize(dev)
    if tb.tb_cuda_synchronize(stream.cuda_stream) != 1:
        raise RuntimeError("onboard kernel reported a pipeline timeout")
    return start.elapsed_time(end) / 1e3 / steps


def time_onboard_reference_cpu(obs, mission, target_s: float):
    import oracle  # test infrastructure: the CPU baseline only

    threads = host_threads()
    n = obs.shape[0]
    out = np.empty((n, 39), np.float32)
    probe = min(n, max(threads * 16, 1024))
    rate = probe / max(oracle.timed_onboard_reference(obs[:probe], mission[:probe], out[:probe], threads), 1e-9)
    sample = int(min(n, max(probe, rate * target_s)))
    t = oracle.timed_onboard_reference(obs[:sample], mission[:sample], out[:sample], threads)
    return {"value": sample / t, "unit": UNIT, "cores": threads, "kind": "reference",
            "sample": f"first {sample} aircraft, reference onboard header (glibc build), {threads} threads, "
                      f"{t:.2f} s wall"}


def profiled_sensor_pipes():
    """FP64-pipe and issue fractions of the sensor kernel from the committed
    ncu summary (name -> fraction), or {} if it is missing."""
    out = {}
    try:
        with open(SENSOR_PROFILE) as f:
            for line in f:
                if ":" in line and not line.startswith("#"):
                    k, v = line.split(":", 1)
                    out[k.strip()] = float(v)
    except (OSError, ValueError):
        pass
    return out


def time_actor_inputs_only(args, dev):
    """tb_cuda_prepare_actor_inputs_device alone on --batch aircraft of the
    seeded batch (the missions as generated, or with --all-scanning half
    dodge and half slalom): W warm-up calls, then K calls between one CUDA
    event pair on the launching stream.  A small command for profilers."""
    import torch

    n = args.batch
    obs, mission, cams, _ = tb.generate(SEED, 0, n, total=n, pinned=True)
    if args.all_scanning:
        mission = np.array(mission, copy=True)
        mission[0::2, 5] = 1.0
        mission[1::2, 4] = 1.0
        mission[1::2, 5] = -0.5
    d_obs, d_mis, d_cam = (torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in (obs, mission, cams))
    shapes = ((n, 91), (n, 49), (n, 24), (n, 15), (n, 6 * 2048), (n, 16384))
    outs = [torch.empty(sh, dtype=torch.float32, device=dev) for sh in shapes]
    stream = torch.cuda.Stream(dev)
    for _ in range(max(args.warmup, 3)):
        assert tb.tb_cuda_prepare_actor_inputs_device(d_obs, d_mis, d_cam, *outs, n, stream) == 1
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        tb.tb_cuda_prepare_actor_inputs_device(d_obs, d_mis, d_cam, *outs, n, stream)
    end.record(stream)
    torch.cuda.synchronize(dev)
    assert tb.tb_cuda_synchronize(stream) == 1
    ms = start.elapsed_time(end) / args.steps
    return {"leg": "actor_inputs", "entry_point": "tb_cuda_prepare_actor_inputs_device", "aircraft": n,
            "missions": "all scanning" if args.all_scanning else "as generated", "steps": args.steps,
            "ms_per_call": ms, "launches_per_call": 2}


def time_config1(stream, dev):
    """BASELINE config 1 (seed 1, 1,024 aircraft): launch latency.  Its
    34.4 MB of inputs fit in the 126 MB L2, so device time is reported
    L2-resident (back to back) and with L2 flushed before every launch, each
    the median of 20 launches timed with CUDA events queued back to back
    behind a GPU sleep (so the events bracket GPU work, not host latency).
    Two flushes: a 256 MiB buffer rewritten (the L2 then holds ~126 MB of
    dirty lines, which the launch's own reads must write back to HBM first),
    and the same followed by a read of the buffer (the L2 then holds clean
    lines of other data).  Launch-inclusive is host wall time from the call to
    the stream's completion (median of 20, L2-resident).  The entry point
    takes the flat one-CTA-per-aircraft kernel at this size; the staged
    kernel, forced, is timed beside it."""
    import torch

    n = 1024
    obs, mission, cams, _ = tb.generate(1, 0, n)
    d_obs, d_mis, d_cam = (torch.from_numpy(x).to(dev) for x in (obs, mission, cams))
    out = torch.empty((n, 142), dtype=torch.float32, device=dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    sink = torch.empty(1, dtype=torch.float32, device=dev)

    def entry():
        return tb.tb_cuda_extract_features_device(d_obs, d_mis, d_cam, out, n, stream)

    def staged():
        return tb.launch(d_obs, d_mis, d_cam, out, n, stream, flat=-1)

    for _ in range(5):
        assert entry() == 1 and staged() == 1
    torch.cuda.synchronize(dev)

    def device_ms(call, flushed):
        # the GPU first sleeps ~20 ms while the host queues all 20 (flush,)
        # event, launch, event groups, so each pair of events brackets the
        # GPU's own work and never the host's submission latency
        pairs = []
        with torch.cuda.stream(stream):
            torch.cuda._sleep(40_000_000)
            for _ in range(20):
                if flushed:
                    flush.zero_()
                    if flushed == "clean":
                        torch.sum(flush, dim=0, keepdim=True, out=sink)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                call()
                b.record(stream)
                pairs.append((a, b))
        stream.synchronize()
        return statistics.median(a.elapsed_time(b) for a, b in pairs)

    def amortised_us(call, flushed, k=20):
        # k launches (each after a flush when flushed) between one pair of
        # events, behind a GPU sleep; per launch, minus the flushes' own time
        def group(with_call, with_flush):
            with torch.cuda.stream(stream):
                torch.cuda._sleep(40_000_000)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(k):
                    if with_flush:
                        flush.zero_()
                    if with_call:
                        call()
                b.record(stream)
            stream.synchronize()
            return a.elapsed_time(b) * 1e3 / k
        both = statistics.median(group(True, flushed) for _ in range(5))
        return both - (statistics.median(group(False, True) for _ in range(5)) if flushed else 0.0)

    resident, flushed, clean = device_ms(entry, False), device_ms(entry, "dirty"), device_ms(entry, "clean")
    st_resident, st_flushed = device_ms(staged, False), device_ms(staged, "dirty")
    st_clean = device_ms(staged, "clean")
    am_resident, am_flushed = amortised_us(entry, False), amortised_us(entry, True)
    st_am_resident, st_am_flushed = amortised_us(staged, False), amortised_us(staged, True)
    host = []
    for _ in range(20):
        t0 = time.perf_counter()
        entry()
        stream.synchronize()
        host.append(time.perf_counter() - t0)
    if tb.tb_cuda_synchronize(stream.cuda_stream) != 1:
        raise RuntimeError("feature kernel reported a pipeline timeout (config 1)")
    expected_ok = np.isfinite(out.cpu().numpy()).all()
    launch_us = statistics.median(host) * 1e6
    peak, peak_kind = measured_hbm_peak()
    algo = n * tb.BYTES_PER_SAMPLE
    return {"workload": "config 1: seed 1, 1,024 aircraft, 34.4 MB of inputs (fit in the 126 MB L2)",
            "kernel": "features_flat_kernel (one CTA per aircraft)",
            "device_us_l2_resident": resident * 1e3, "device_us_l2_flushed": flushed * 1e3,
            "device_us_l2_flushed_clean": clean * 1e3,
            "launch_inclusive_us": launch_us, "value_l2_flushed": n / (flushed / 1e3), "unit": UNIT,
            "roofline_frac_l2_flushed": algo / (flushed / 1e3) / 1e9 / peak,
            "roofline_frac_l2_flushed_clean": algo / (clean / 1e3) / 1e9 / peak,
            "amortised_us_l2_resident": am_resident, "amortised_us_l2_flushed": am_flushed,
            "roofline_frac_amortised_l2_flushed": algo / (am_flushed / 1e6) / 1e9 / peak,
            "peak_source": f"{peak_kind} hbm_gbs",
            "staged_kernel": {"device_us_l2_resident": st_resident * 1e3, "device_us_l2_flushed": st_flushed * 1e3,
                              "device_us_l2_flushed_clean": st_clean * 1e3,
                              "amortised_us_l2_resident": st_am_resident, "amortised_us_l2_flushed": st_am_flushed},
            "amortised": "per launch over 20 launches between one event pair behind a GPU sleep (event ticks "
                         "here are ~2 us apart, so a single-launch pair cannot resolve the kernel); flushed: each "
                         "launch after a 256 MiB rewrite, minus the rewrites' own time; medians of 5 groups",
            "flush": "l2_flushed: a 256 MiB buffer rewritten before each launch (dirty L2); "
                     "l2_flushed_clean: rewritten, then read (clean L2 holding other data)",
            "finite": bool(expected_ok),
            "timing": "medians of 20; events around each launch; host wall clock call -> stream done",
            "launches": 10 + 6 * 20 + 20 + 4 * 5 * 20}


def time_sensors(scenes, steps, warmup, stream, dev):
    """Device time per launch of tb_cuda_render_sensors_device over the
    resident scenes (LiDAR, valid fractions and cameras of every scene), and
    the same call end to end: page-locked scenes copied in and every output
    copied back inside each step, on the same stream, host wall clock."""
    import torch

    from turbinator_c_b200.sensors import tb_cuda_render_sensors_device as render

    n = len(scenes)
    h_scenes = torch.from_numpy(scenes.view(np.uint8).reshape(-1).copy()).pin_memory()
    d_scenes = h_scenes.to(dev)
    lidar = torch.empty((n, 4096), dtype=torch.float32, device=dev)
    valid = torch.empty((n, 2), dtype=torch.float32, device=dev)
    cams = torch.empty((n, 16384), dtype=torch.uint8, device=dev)
    torch.cuda.synchronize(dev)
    for _ in range(max(warmup, 3)):
        assert render(d_scenes, n, lidar, 4096, valid, 2, cams, None, stream) == 1
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        render(d_scenes, n, lidar, 4096, valid, 2, cams, None, stream)
    end.record(stream)
    torch.cuda.synchronize(dev)
    per_launch = start.elapsed_time(end) / 1e3 / steps
    h_lidar = torch.empty((n, 4096), dtype=torch.float32, pin_memory=True)
    h_valid = torch.empty((n, 2), dtype=torch.float32, pin_memory=True)
    h_cams = torch.empty((n, 16384), dtype=torch.uint8, pin_memory=True)
    e2e_steps = max(1, min(steps, 5))
    with torch.cuda.stream(stream):
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            d_scenes.copy_(h_scenes, non_blocking=True)
            render(d_scenes, n, lidar, 4096, valid, 2, cams, None, stream)
            h_lidar.copy_(lidar, non_blocking=True)
            h_valid.copy_(valid, non_blocking=True)
            h_cams.copy_(cams, non_blocking=True)
            stream.synchronize()
        e2e = (time.perf_counter() - t0) / e2e_steps
    if not np.isfinite(h_valid.numpy()).all():
        raise RuntimeError("non-finite LiDAR valid fractions")
    return per_launch, e2e, n * (4096 * 4 + 8 + 16384)


def time_render_extract(scenes, head, ages, mission_host, steps, warmup, stream, dev):
    """The trainer's observation path kept on the device (the reference
    renders on the host, src/sim/sensors.c:28-82, and copies every
    observation row to the GPU, src/sim/c_api.c:104-112).  Each step copies
    in, from page-locked memory, the scene records (2,432 B per aircraft:
    what the renderers read), the rest of each observation row that the
    simulator fills on the host (48 proprioceptive values and 2 LiDAR ages,
    sensors.c:104-119: 200 B) and the mission rows (40 B); renders LiDAR
    (with its valid fractions) and cameras straight into device observation
    rows and camera buffers (tb_cuda_render_sensors_device, all sensors of
    every aircraft every step); extracts the 142 features
    (tb_cuda_extract_features_device); and copies only the features (568 B)
    back, in CHUNKS_RENDER chunks alternating two streams so that a chunk's
    copies overlap the previous chunk's rendering.  Host wall clock per step,
    after `warmup` steps.  Returns the timing and the final step's features."""
    import torch

    from turbinator_c_b200.sensors import tb_cuda_render_sensors_device as render

    n = len(scenes)
    h_scenes = torch.from_numpy(scenes.view(np.uint8).reshape(-1).copy()).pin_memory()
    h_head = torch.from_numpy(np.ascontiguousarray(np.concatenate([head, ages], axis=1))).pin_memory()
    h_mis = torch.from_numpy(np.ascontiguousarray(mission_host)).pin_memory()
    h_out = torch.empty((n, tb.FEATURE_DIM), dtype=torch.float32, pin_memory=True)
    d_scenes = torch.empty_like(h_scenes, device=dev)
    d_head = torch.empty_like(h_head, device=dev)
    d_mis = torch.empty_like(h_mis, device=dev)
    d_obs = torch.zeros((n, tb.OBS_DIM), dtype=torch.float32, device=dev)
    d_cams = torch.empty((n, tb.CAMERA_BYTES), dtype=torch.uint8, device=dev)
    d_out = torch.empty((n, tb.FEATURE_DIM), dtype=torch.float32, device=dev)
    torch.cuda.synchronize(dev)

    # chunks of the batch alternate two streams, so that one chunk's copies
    # overlap another's rendering (every copy stays inside the step)
    streams = (stream, torch.cuda.Stream(dev))
    chunk = max(1, -(-n // CHUNKS_RENDER))
    scene_bytes = scenes.dtype.itemsize

    def step():
        for c, a in enumerate(range(0, n, chunk)):
            z = min(n, a + chunk)
            st = streams[c % 2]
            with torch.cuda.stream(st):
                d_scenes[a * scene_bytes:z * scene_bytes].copy_(h_scenes[a * scene_bytes:z * scene_bytes],
                                                                non_blocking=True)
                d_head[a:z].copy_(h_head[a:z], non_blocking=True)
                d_mis[a:z].copy_(h_mis[a:z], non_blocking=True)
                d_obs[a:z, :48].copy_(d_head[a:z, :48])
                d_obs[a:z, 4144:4146].copy_(d_head[a:z, 48:50])
                if render(d_scenes.data_ptr() + a * scene_bytes, z - a, d_obs[a].data_ptr() + 48 * 4, tb.OBS_DIM,
                          d_obs[a].data_ptr() + 4146 * 4, tb.OBS_DIM, d_cams[a:z], None, st) != 1:
                    raise RuntimeError("sensor rendering launch failed")
                if tb.tb_cuda_extract_features_device(d_obs[a:z], d_mis[a:z], d_cams[a:z], d_out[a:z], z - a,
                                                      st) != 1:
                    raise RuntimeError("feature launch failed")
                h_out[a:z].copy_(d_out[a:z], non_blocking=True)
        for st in streams:
            st.synchronize()

    for _ in range(max(warmup, 3)):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    per_step = (time.perf_counter() - t0) / steps
    if any(tb.tb_cuda_synchronize(st.cuda_stream) != 1 for st in streams):
        raise RuntimeError("feature kernel reported a pipeline timeout (render leg)")
    out = h_out.numpy().copy()
    del d_scenes, d_head, d_mis, d_obs, d_cams, d_out
    torch.cuda.empty_cache()
    return per_step, out, n * (2432 + 200 + 40), n * tb.FEATURE_DIM * 4


def render_extract_reference(scenes, head, ages, mission_host, threads):
    """The reference's own CPU path for the same aircraft: its simulator's
    renderers (oracle/_ref) fill the observation rows and camera bytes, then
    tb_train_extract_features_cpu.  Returns (features, seconds rendering,
    seconds extracting) on `threads` host threads."""
    import oracle  # test infrastructure: the checker and the CPU baseline only

    n = len(scenes)
    t0 = time.perf_counter()
    if oracle.have_reference_sensors():
        lidar, valid, cams, _ = oracle.render_sensors_reference(scenes, threads=threads)
    else:  # the restatement, pinned bit for bit to the reference renderers
        lidar, valid, cams, _ = oracle.render_sensors_port(scenes)
    t_render = time.perf_counter() - t0
    obs = np.zeros((n, tb.OBS_DIM), np.float32)
    obs[:, :48] = head
    obs[:, 48:4144] = lidar
    obs[:, 4144:4146] = ages
    obs[:, 4146:4148] = valid
    out = np.empty((n, tb.FEATURE_DIM), np.float32)
    timed = oracle.timed_reference if oracle.have_reference() else oracle.timed_port
    t_feat = timed(obs, np.ascontiguousarray(mission_host), cams, out, threads)
    return out, t_render, t_feat


def time_sensors_reference_cpu(scenes, target_s: float):
    import oracle  # test infrastructure: the CPU baseline only

    threads = host_threads()
    n = len(scenes)
    probe = min(n, max(threads * 2, 64))
    rate = probe / max(oracle.timed_sensors_reference(scenes[:probe], threads), 1e-9)
    sample = int(min(n, max(probe, rate * target_s)))
    t = oracle.timed_sensors_reference(scenes[:sample], threads)
    return {"value": sample / t, "unit": "scenes/s", "cores": threads, "kind": "reference",
            "sample": f"first {sample} scenes, the reference simulator's tb_sim_render_lidar + "
                      f"tb_sim_render_camera (oracle/_ref, ISO C11 -O2), {threads} threads, {t:.2f} s wall"}


# ---------------------------------------------------------------- multi-rank helpers

def gpu_numa_node(local_rank: int):
    """NUMA node of this rank's GPU (sysfs through its NVML PCI bus id), or None."""
    try:
        import pynvml

        pynvml.nvmlInit()
        visible = os.environ.get("CUDA_VISIBLE_DEVICES")
        idx = local_rank
        if visible:
            ids = [v.strip() for v in visible.split(",") if v.strip()]
            idx = int(ids[local_rank]) if ids[local_rank].isdigit() else local_rank
        bus = pynvml.nvmlDeviceGetPciInfo(pynvml.nvmlDeviceGetHandleByIndex(idx)).busId
        bus = bus.decode() if isinstance(bus, bytes) else bus
        dom, rest = bus.split(":", 1)
        path = f"/sys/bus/pci/devices/{int(dom, 16):04x}:{rest.lower()}/numa_node"
        with open(path) as f:
            node = int(f.read().strip())
        return node if node >= 0 else None
    except Exception:
        return None


def node_cpus(node: int):
    """CPUs of a NUMA node (sysfs cpulist), or an empty set."""
    cpus = set()
    try:
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            for part in f.read().strip().split(","):
                if "-" in part:
                    lo, hi = part.split("-")
                    cpus.update(range(int(lo), int(hi) + 1))
                elif part:
                    cpus.add(int(part))
    except OSError:
        pass
    return cpus


def h2d_probe(dev, rank, world, local_rank, barrier):
    """Host-to-device copy rate of 1 GiB from page-locked memory, to tell
    which shared resource holds the host path back at N > 1: each rank alone
    in turn (its own PCIe link, nothing else busy), then all ranks at once
    from buffers allocated as the benchmark allocates them, then all ranks at
    once from buffers allocated by a thread bound to the GPU's own NUMA node
    (the pages land in that node's memory).  The same 1 GiB device-to-host,
    alone and all at once, bounds the gather (which copies the other way)."""
    import torch

    nbytes = 1 << 30
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    src = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)

    def copy_s(buf):
        t0 = time.perf_counter()
        dst.copy_(buf, non_blocking=True)
        torch.cuda.synchronize(dev)
        return time.perf_counter() - t0

    def back_s():
        t0 = time.perf_counter()
        src.copy_(dst, non_blocking=True)
        torch.cuda.synchronize(dev)
        return time.perf_counter() - t0

    copy_s(src)
    solo = None
    for r in range(world):
        barrier()
        if r == rank:
            solo = copy_s(src)
        barrier()
    barrier()
    together = copy_s(src)
    back_s()
    back_solo = None
    for r in range(world):
        barrier()
        if r == rank:
            back_solo = back_s()
        barrier()
    barrier()
    back_together = back_s()
    node = gpu_numa_node(local_rank)
    src_local = local = None
    if node is not None and node_cpus(node):
        saved = os.sched_getaffinity(0)
        try:
            os.sched_setaffinity(0, node_cpus(node))
            src_local = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
            src_local.fill_(1)
            copy_s(src_local)
        except Exception:  # affinity or allocation refused: report no NUMA-local figure
            src_local = None
        finally:
            os.sched_setaffinity(0, saved)
    barrier()  # every rank takes this one barrier, with or without a NUMA-local buffer
    if src_local is not None:
        local = copy_s(src_local)
    everyone = all_ranks({"solo_gbs": nbytes / solo / 1e9, "together_gbs": nbytes / together / 1e9,
                          "together_s": together, "numa_local_s": local, "gpu_numa_node": node,
                          "d2h_solo_gbs": nbytes / back_solo / 1e9, "d2h_together_gbs": nbytes / back_together / 1e9,
                          "d2h_together_s": back_together})
    del src, dst, src_local
    torch.cuda.empty_cache()
    if hasattr(torch._C, "_host_emptyCache"):
        torch._C._host_emptyCache()  # hand the 2 GiB of page-locked probe buffers back
    out = {"bytes_per_rank": nbytes,
           "solo_gbs": [e["solo_gbs"] for e in everyone],
           "together_gbs": [e["together_gbs"] for e in everyone],
           "together_aggregate_gbs": world * nbytes / max(e["together_s"] for e in everyone) / 1e9,
           "gpu_numa_node": [e["gpu_numa_node"] for e in everyone],
           "d2h_solo_gbs": [e["d2h_solo_gbs"] for e in everyone],
           "d2h_together_gbs": [e["d2h_together_gbs"] for e in everyone],
           "d2h_together_aggregate_gbs": world * nbytes / max(e["d2h_together_s"] for e in everyone) / 1e9,
           "method": "torch copy_ of a 1 GiB page-locked buffer to the device (and back: d2h_*), host wall "
                     "clock; solo: one rank at a time; together: all ranks at once, aggregate = N GiB / "
                     "slowest rank"}
    if all(e["numa_local_s"] for e in everyone):
        out["numa_local_aggregate_gbs"] = world * nbytes / max(e["numa_local_s"] for e in everyone) / 1e9
        out["numa_local_gbs"] = [nbytes / e["numa_local_s"] / 1e9 for e in everyone]
    return out


def parity_leg(dev, stream, rank, world, obs, mission, cams, out_timed, out_host, first, count, total,
               gatherer, threads):
    """Checks what the timed regions produced against the reference CPU path
    (the oracle is test infrastructure: the checker here, never timed and
    never on the product path), on every rank, after every timed region:

      timed    the feature launches timed for `value` (config 2 per rank, config
               3 over 8 ranks): every 97th aircraft of the whole batch that falls
               in this rank's shard, plus the shard's first and last aircraft,
               against the oracle on the same host inputs;
      gather   the shared host buffer after the gather: this rank's slice equal
               bit for bit to its timed output, and on rank 0 the same strided
               subsample of the WHOLE gathered batch against the oracle on
               inputs regenerated for just those indices;
      e2e      the host-ABI output (page-locked leg) equal bit for bit to the
               timed output (same inputs, same kernel arithmetic);
      config4  BASELINE config 4 (seed 4, 131,072 aircraft in four stress
               quarters): this rank's shard generated, extracted through
               tb_cuda_extract_features_device and checked in full.

    Counts are summed over ranks; the rule is tests/parity.py's (bit-exact
    f[0..61] and f[126..141], |d| <= 1e-6 + 1e-5*|ref| for f[62..125])."""
    import torch

    import oracle  # test infrastructure: the checker of the timed outputs only
    from tests.parity import mismatch_counts

    use_ref = oracle.have_reference()

    def expected(o, m, c):
        return oracle.features(np.ascontiguousarray(o), np.ascontiguousarray(m), np.ascontiguousarray(c),
                               threads=threads, use_reference=use_ref)

    def strided(lo, n):
        idx = set(range(-(-lo // 97) * 97, lo + n, 97))
        idx.update((lo, lo + n - 1))
        return np.array(sorted(i for i in idx if lo <= i < lo + n), dtype=np.int64)

    counts = {}
    # timed launches, this rank's shard
    idx = strided(first, count) - first
    e, l = mismatch_counts(out_timed[idx], expected(obs[idx], mission[idx], cams[idx]))
    counts["timed_checked"], counts["timed_mismatches"] = len(idx), e + l
    # the gathered host buffer
    mine = gatherer.array[first:first + count]
    counts["gather_rows_checked"] = count
    counts["gather_mismatches"] = int(np.count_nonzero(np.any(mine.view(np.uint32) != out_timed.view(np.uint32),
                                                                axis=1)))
    counts["gather_sample_checked"] = counts["gather_sample_mismatches"] = 0
    if rank == 0:
        whole = set()
        for r in range(world):
            f, c = shard_range(total, r, world)
            whole.update(strided(f, c).tolist())
        gidx = np.array(sorted(whole), dtype=np.int64)
        rows = [tb.generate(SEED, int(i), 1, total=total) for i in gidx]
        o = np.concatenate([r[0] for r in rows])
        m = np.concatenate([r[1] for r in rows])
        c = np.concatenate([r[2] for r in rows])
        e, l = mismatch_counts(gatherer.array[gidx], expected(o, m, c))
        counts["gather_sample_checked"], counts["gather_sample_mismatches"] = len(gidx), e + l
    # host ABI output
    counts["e2e_rows_checked"] = count
    counts["e2e_mismatches"] = int(np.count_nonzero(np.any(
        np.asarray(out_host).view(np.uint32) != out_timed.view(np.uint32), axis=1)))
    # config 4 stress shard
    c4_total = tb.CONFIGS[4][1]
    f4, n4 = shard_range(c4_total, rank, world)
    o4, m4, k4, _ = tb.generate(tb.CONFIGS[4][0], f4, n4, total=c4_total, stress=True, threads=threads)
    d4 = [torch.from_numpy(x).to(dev) for x in (o4, m4, k4)]
    out4 = torch.full((n4, tb.FEATURE_DIM), float("nan"), dtype=torch.float32, device=dev)
    torch.cuda.synchronize(dev)
    if tb.tb_cuda_extract_features_device(*d4, out4, n4, stream) != 1 or \
            tb.tb_cuda_synchronize(stream.cuda_stream) != 1:
        raise RuntimeError("config-4 launch failed")
    e, l = mismatch_counts(out4.cpu().numpy(), expected(o4, m4, k4))
    counts["config4_checked"], counts["config4_mismatches"] = n4, e + l
    del d4, out4, o4, m4, k4
    torch.cuda.empty_cache()

    keys = sorted(counts)
    summed = dict(zip(keys, sum_over_ranks([counts[k] for k in keys])))
    total_bad = sum(v for k, v in summed.items() if k.endswith("mismatches"))
    return {"checked": summed["timed_checked"], "mismatches": summed["timed_mismatches"],
            "config4_checked": summed["config4_checked"], "config4_mismatches": summed["config4_mismatches"],
            "gather_rows_checked": summed["gather_rows_checked"], "gather_mismatches": summed["gather_mismatches"],
            "gather_sample_checked": summed["gather_sample_checked"],
            "gather_sample_mismatches": summed["gather_sample_mismatches"],
            "e2e_rows_checked": summed["e2e_rows_checked"], "e2e_mismatches": summed["e2e_mismatches"],
            "all_mismatches": total_bad, "ranks": world,
            "oracle": ("the reference's tb_train_extract_features_cpu (oracle/_ref)" if use_ref
                       else "the C restatement of the reference CPU path (oracle/)"),
            "rule": "bit-exact f[0..61], f[126..141]; |d| <= 1e-6 + 1e-5*|ref| for f[62..125]",
            "sample": "every 97th aircraft of the timed batch plus each shard's first and last; config 4 in full"}


# ---------------------------------------------------------------- arms

def run_reference_arm(args, rank: int, world: int):
    if rank != 0:
        return
    import oracle  # test infrastructure: the reference arm times the reference CPU code

    obs, mission, cams, _ = tb.generate(SEED, 0, args.batch, total=args.batch * world,
                                        threads=host_threads())
    kind = "reference" if oracle.have_reference() else "port"
    timed = oracle.timed_reference if kind == "reference" else oracle.timed_port
    threads = host_threads()
    out = np.empty((args.batch, 142), np.float32)
    probe = min(args.batch, max(threads * 64, 2048))
    rate = probe / max(timed(obs[:probe], mission[:probe], cams[:probe], out[:probe], threads), 1e-9)
    # each step: the whole batch if it takes <= ~3 s, else a leading sample of it
    per_step = int(min(args.batch, max(probe, rate * 3.0)))
    for _ in range(args.warmup):
        timed(obs[:per_step], mission[:per_step], cams[:per_step], out[:per_step], threads)
    total_t = 0.0
    for _ in range(args.steps):
        total_t += timed(obs[:per_step], mission[:per_step], cams[:per_step], out[:per_step], threads)
    value = per_step * args.steps / total_t
    sample = (f"{per_step} of the {args.batch}-aircraft batch per step, {threads} threads; "
              f"host CPU: {cpu_description()}")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total_t / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded SplitMix64 generator, BASELINE value model)",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(args, world):
    return {
        "workload": f"config2-per-GPU: {args.batch} aircraft per GPU (seed {SEED}); "
                    f"{world} GPU(s) -> {args.batch * world} aircraft"
                    + (" (= config 3)" if args.batch * world == 524288 else ""),
        "batch_per_gpu": args.batch,
        "global_batch": args.batch * world,
        "abi": "u8 cameras (reference cuda_features.h)",
        "bytes_per_sample": tb.BYTES_PER_SAMPLE,
        "parallelism": f"sample-sharded x{world}, no collective on the data path",
        "l2": f"inputs {args.batch * tb.BYTES_PER_SAMPLE / 1e9:.2f} GB per GPU > 126 MB L2; no flush needed",
    }


def run_ours(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    tb.load_library()
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", world))
    gen_threads = max(1, host_threads() // max(local_world, 1))

    total = args.batch * world
    first, count = shard_range(total, rank, world)
    obs, mission, cams, _ = tb.generate(SEED, first, count, total=total, threads=gen_threads, pinned=True)
    d_obs = torch.from_numpy(obs).to(dev)
    d_mis = torch.from_numpy(mission).to(dev)
    d_cam = torch.from_numpy(cams).to(dev)
    d_out = torch.empty((count, 142), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(dev)
    torch.cuda.synchronize(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    clocks = ClockSampler(local_rank)

    # ---- value: kernel only, inputs resident in HBM
    for _ in range(max(args.warmup, 3)):
        assert tb.tb_cuda_extract_features_device(d_obs, d_mis, d_cam, d_out, count, stream) == 1
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.active(True)
    start.record(stream)
    for _ in range(args.steps):
        tb.tb_cuda_extract_features_device(d_obs, d_mis, d_cam, d_out, count, stream)
    end.record(stream)
    torch.cuda.synchronize(dev)
    clocks.active(False)
    if tb.tb_cuda_synchronize(stream.cuda_stream) != 1:
        raise RuntimeError("feature kernel reported a pipeline timeout during the timed region")
    barrier()
    kernel_s = start.elapsed_time(end) / 1e3
    kernel_s_max = max_over_ranks(kernel_s)
    value = total * args.steps / kernel_s_max
    out_timed = d_out.cpu().numpy()  # checked against the oracle after the other legs

    # ---- FP32-camera entry point (BASELINE's byte sizes): same rows, float cameras
    f32cam = None
    if not args.no_f32cam:
        _, _, _, camf = tb.generate(SEED, first, count, total=total, threads=gen_threads, f32_cameras=True)
        d_camf = torch.from_numpy(camf).to(dev)
        del camf
        for _ in range(max(args.warmup, 3)):
            assert tb.tb_cuda_extract_features_device_f32cam(d_obs, d_mis, d_camf, d_out, count, stream) == 1
        torch.cuda.synchronize(dev)
        barrier()
        f_start, f_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f_start.record(stream)
        for _ in range(args.steps):
            tb.tb_cuda_extract_features_device_f32cam(d_obs, d_mis, d_camf, d_out, count, stream)
        f_end.record(stream)
        torch.cuda.synchronize(dev)
        if tb.tb_cuda_synchronize(stream.cuda_stream) != 1:
            raise RuntimeError("FP32-camera kernel reported a pipeline timeout")
        f_per = f_start.elapsed_time(f_end) / 1e3 / args.steps
        f_per_max = max_over_ranks(f_per)
        peak_gbs, _ = measured_hbm_peak()
        f_ach = count * tb.BYTES_PER_SAMPLE_F32CAM / f_per / 1e9
        f32cam = {"entry_point": "tb_cuda_extract_features_device_f32cam",
                  "value": total / f_per_max, "unit": UNIT, "ms_per_launch": f_per_max * 1e3,
                  "bytes_per_sample": tb.BYTES_PER_SAMPLE_F32CAM,
                  "roofline": {"bound": "hbm", "achieved": f_ach, "peak": peak_gbs, "unit": "GB/s",
                               "frac": f_ach / peak_gbs},
                  "launches": args.steps}
        del d_camf
        torch.cuda.empty_cache()

    # ---- learner input tensors (tb_cuda_prepare_actor_inputs_device) on the same rows
    actor = None
    if not args.no_actor_inputs:
        shapes = ((count, 91), (count, 49), (count, 24), (count, 15), (count, 6 * 2048), (count, 16384))
        a_outs = [torch.empty(sh, dtype=torch.float32, device=dev) for sh in shapes]
        for _ in range(max(args.warmup, 3)):
            assert tb.tb_cuda_prepare_actor_inputs_device(d_obs, d_mis, d_cam, *a_outs, count, stream) == 1
        torch.cuda.synchronize(dev)
        barrier()
        a_start, a_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_steps = max(1, min(args.steps, 20))
        a_start.record(stream)
        for _ in range(a_steps):
            tb.tb_cuda_prepare_actor_inputs_device(d_obs, d_mis, d_cam, *a_outs, count, stream)
        a_end.record(stream)
        torch.cuda.synchronize(dev)
        a_per = a_start.elapsed_time(a_end) / 1e3 / a_steps
        a_per_max = max_over_ranks(a_per)
        bpa = tb.BYTES_PER_SAMPLE_ACTOR_INPUTS
        peak_gbs, peak_kind = measured_hbm_peak()
        a_ach = count * bpa / a_per / 1e9
        actor = {"entry_point": "tb_cuda_prepare_actor_inputs_device",
                 "outputs": "proprio 91, mission 49, tactical 24, prior 15, LiDAR 6x2048, luma 16384 per aircraft",
                 "value": total / a_per_max, "unit": UNIT, "ms_per_launch": a_per_max * 1e3,
                 "bytes_per_sample": bpa,
                 "roofline": {"bound": "hbm (78 % writes)", "achieved": a_ach, "peak": peak_gbs, "unit": "GB/s",
                              "frac": a_ach / peak_gbs, "peak_source": f"{peak_kind} hbm_gbs (copy)"},
                 "launches": 2 * a_steps}  # the streaming kernel (with the scans), then the control law
        del a_outs
        torch.cuda.empty_cache()

    # ---- secondary path: onboard tactical/prior values on the same resident inputs
    onboard = None
    if not args.no_onboard:
        legs = {}
        for name, mis_host in (("mission_mix", mission), ("all_scanning", all_scanning(mission))):
            per_launch = time_onboard(d_obs, mis_host, count, args.steps, args.warmup, stream, dev)
            per_launch_max = max_over_ranks(per_launch)
            frac = scanning_fraction(mis_host)
            bpa = onboard_bytes_per_aircraft(frac)
            legs[name] = {"value": total / per_launch_max, "unit": UNIT,
                          "ms_per_launch": per_launch_max * 1e3, "scanning_fraction": frac,
                          "algorithmic_bytes_per_aircraft": bpa,
                          "achieved_gbs": count * bpa / per_launch / 1e9}
        onboard = {"entry_point": "tb_cuda_extract_onboard_device", "outputs": "24 tactical + 15 prior",
                   "bound": "SM instruction issue (control law + LiDAR scans), not HBM", **legs,
                   "launches": 4 * args.steps}  # 2 mission sets x (scan + control kernels)

    # ---- simulator sensor rendering (tb_cuda_render_sensors_device), its own scenes
    sensors = None
    sensor_scene_sets = {}
    if not args.no_sensors:
        from turbinator_c_b200.sensors import synthetic_scenes

        legs = {}
        for name, balls in (("flight_mix", "flight"), ("heaviest", "max")):
            # weak scaling: each rank renders its own seeded scenes
            scount = args.sensor_scenes
            total_s = scount * world
            scenes = synthetic_scenes(SEED * 1000 + rank, scount, balls=balls)
            sensor_scene_sets[name] = scenes
            s_steps = max(1, min(args.steps, 10))
            per, e2e_per, d2h = time_sensors(scenes, s_steps, args.warmup, stream, dev)
            per_max, e2e_max = max_over_ranks(per), max_over_ranks(e2e_per)
            legs[name] = {"value": total_s / per_max, "unit": "scenes/s", "ms_per_launch": per_max * 1e3,
                          "rays_per_s": total_s * RAYS_PER_SCENE / per_max, "scenes_per_gpu": scount,
                          "mean_spheres_per_scene": float(np.mean(
                              np.clip(scenes["obstacle_count"], 0, 24) + np.clip(scenes["ball_count"], 0, 64))),
                          "e2e": {"value": total_s / e2e_max, "unit": "scenes/s", "ms_per_step": e2e_max * 1e3,
                                  "h2d_bytes_per_step": scount * 2432, "d2h_bytes_per_step": d2h,
                                  "api": "scenes copied in from page-locked memory, LiDAR + valid + cameras "
                                         "copied back, every step (host wall clock)"},
                          "launches": 2 * (s_steps + max(1, min(s_steps, 5)))}  # LiDAR + camera kernels
        pipes = profiled_sensor_pipes()
        sensors = {"entry_point": "tb_cuda_render_sensors_device",
                   "roofline": {"bound": "fp64 pipe / instruction issue (not HBM, not tensor)",
                                "fp64_pipe_frac": {"flight_mix": pipes.get("fp64_pipe_frac_flight_mix"),
                                                   "heaviest": pipes.get("fp64_pipe_frac_heaviest")},
                                "issue_active_frac": {"flight_mix": pipes.get("issue_active_frac_flight_mix"),
                                                      "heaviest": pipes.get("issue_active_frac_heaviest")},
                                "source": "ncu --set full of 4,096 scenes (profiles/sensors_kernel_s4096.md)"},
                   "outputs": "4,096 LiDAR ranges + 2 valid fractions + 4 x 64 x 64 camera bytes per scene",
                   "bound": "FP64 pipe (double-precision ray/sphere tests, no FMA contraction), not HBM",
                   "data": "synthetic scenes with the simulator's geometry (seeded); flight_mix: uniform over "
                           "the 28 scenarios, 0-12 cannon balls in arena scenes; heaviest: 24 obstacles in "
                           "every course scene and 64 balls in every arena scene",
                   **legs, "launches": sum(v["launches"] for v in legs.values())}

    # ---- observations kept on the device: scenes in, render -> extract, features out
    render_leg = render_check = None
    if not args.no_sensors:
        from turbinator_c_b200.sensors import synthetic_scenes

        r_scenes = synthetic_scenes(SEED * 1000 + 500 + rank, count, balls="flight")
        r_steps = max(1, min(args.steps, 10))
        r_per, r_feats, r_h2d, r_d2h = time_render_extract(r_scenes, obs[:, :48], obs[:, 4144:4146], mission,
                                                           r_steps, args.warmup, stream, dev)
        r_max = max_over_ranks(r_per)
        render_leg = {"value": total / r_max, "unit": UNIT, "ms_per_step": r_max * 1e3, "steps": r_steps,
                      "h2d_bytes_per_step": r_h2d, "d2h_bytes_per_step": r_d2h,
                      "api": "per step: scene records + 48 proprioceptive values + 2 LiDAR ages + mission copied "
                             "in from page-locked memory, tb_cuda_render_sensors_device into device observation "
                             "rows and cameras, tb_cuda_extract_features_device, features copied back, in "
                             f"{CHUNKS_RENDER} chunks on two alternating streams (host wall clock, max over ranks)",
                      "data": "synthetic flight-mix scenes (uniform over the 28 scenarios) with the benchmark "
                              "batch's proprioceptive values and missions; every sensor of every aircraft "
                              "rendered every step",
                      "launches": 3 * CHUNKS_RENDER * (r_steps + max(args.warmup, 3))}
        render_check = (r_scenes, r_feats)

    # ---- config 1 latency (1,024 aircraft)
    config1 = time_config1(stream, dev) if rank == 0 else None

    # ---- the final gather to host memory, and kernel + gather end to end
    # (config 3 at N = 8): every rank copies its own [n,142] slice over its
    # own PCIe link into its offset of one shared page-locked host buffer
    gatherer = SharedHostGather(total, tb.FEATURE_DIM)
    reps = 5
    g_times, c3_times = [], []
    for _ in range(reps):
        barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        gatherer.gather(d_out, stream)
        stream.synchronize()
        g_times.append(time.perf_counter() - t0)
    for _ in range(reps):
        barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        tb.tb_cuda_extract_features_device(d_obs, d_mis, d_cam, d_out, count, stream)
        gatherer.gather(d_out, stream)
        stream.synchronize()
        c3_times.append(time.perf_counter() - t0)
    # the same slices copied into each rank's own page-locked buffer (which no
    # other rank can read): what the shared mapping itself costs
    private = torch.empty((count, tb.FEATURE_DIM), dtype=torch.float32, pin_memory=True)
    p_times = []
    for _ in range(reps):
        barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            private.copy_(d_out, non_blocking=True)
        stream.synchronize()
        p_times.append(time.perf_counter() - t0)
    del private
    barrier()
    if tb.tb_cuda_synchronize(stream.cuda_stream) != 1:
        raise RuntimeError("feature kernel reported a pipeline timeout (gather leg)")
    g_max = statistics.median(max_over_ranks_list(g_times))
    p_max = statistics.median(max_over_ranks_list(p_times))
    c3_max = statistics.median(max_over_ranks_list(c3_times))
    gather_bytes = total * tb.FEATURE_DIM * 4
    gather = {"ms": g_max * 1e3, "bytes_to_host": gather_bytes, "gbs": gather_bytes / g_max / 1e9,
              "buffer": os.path.dirname(gatherer.path), "page_locked_ranks": sum(all_ranks(int(gatherer.registered))),
              "op": "each rank copies its [n,142] slice device-to-host into its offset of one page-locked "
                    "host buffer shared by all ranks (/dev/shm, cudaHostRegister per rank), concurrently; "
                    "no GPU collective",
              "timing": f"host wall clock from a barrier to the copy's completion, max over ranks per "
                        f"repetition, median of {reps}",
              "private_buffers_ms": p_max * 1e3,
              "private_buffers_note": "the same copies into each rank's own page-locked torch buffer at once"}
    config3_e2e = {"value": total / c3_max, "unit": UNIT, "ms": c3_max * 1e3,
                   "op": "one feature launch on resident inputs plus the gather of its output to host memory",
                   "timing": f"host wall clock from a barrier, max over ranks per repetition, median of {reps}"}

    # ---- e2e: the reference-facing host ABI on page-locked host buffers
    e2e_steps = args.e2e_steps or min(args.steps, 20)
    out_host = torch.empty((count, 142), dtype=torch.float32, pin_memory=True).numpy()
    fb = tb.FeatureBatch(local_rank, count)
    for _ in range(max(1, min(args.warmup, 3))):
        if fb.extract(obs, mission, cams, count, out_host) != 1:
            raise RuntimeError(f"host ABI failed: {fb.error()}")
    barrier()
    clocks.active(True)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        if fb.extract(obs, mission, cams, count, out_host) != 1:
            raise RuntimeError(f"host ABI failed: {fb.error()}")
    e2e_s = time.perf_counter() - t0
    clocks.active(False)
    # the same through pageable host buffers (what the reference trainer passes)
    p_obs, p_mis, p_cams = np.array(obs), np.array(mission), np.array(cams)
    p_out = np.empty((count, 142), np.float32)
    if fb.extract(p_obs, p_mis, p_cams, count, p_out) != 1:
        raise RuntimeError(f"host ABI failed: {fb.error()}")
    barrier()
    p_steps = max(1, min(e2e_steps, 5))
    t0 = time.perf_counter()
    for _ in range(p_steps):
        if fb.extract(p_obs, p_mis, p_cams, count, p_out) != 1:
            raise RuntimeError(f"host ABI failed: {fb.error()}")
    pageable_s = max_over_ranks((time.perf_counter() - t0) / p_steps)
    del p_obs, p_mis, p_cams, p_out
    fb.close()
    e2e_s_max = max_over_ranks(e2e_s)
    e2e_value = total * e2e_steps / e2e_s_max
    chunks = -(-count // 8192)
    h2d_per_step = count * (tb.OBS_DIM * 4 + tb.MISSION_DIM * 4 + tb.CAMERA_BYTES)
    per_rank_h2d = all_ranks(h2d_per_step * e2e_steps / e2e_s / 1e9)

    # ---- where the host path's bandwidth goes at N > 1
    h2d = h2d_probe(dev, rank, world, local_rank, barrier) if world > 1 else None

    # ---- parity of what was timed (after every timed region)
    parity = None if args.no_parity else parity_leg(
        dev, stream, rank, world, obs, mission, cams, out_timed, out_host, first, count, total,
        gatherer, gen_threads)
    gatherer.close()
    if render_leg is not None and parity is not None:
        from tests.parity import mismatch_counts

        r_scenes, r_feats = render_check
        idx = np.unique(np.r_[np.arange(0, count, 97), count - 1])
        ref, _, _ = render_extract_reference(r_scenes[idx], obs[idx, :48], obs[idx, 4144:4146], mission[idx],
                                             gen_threads)
        e, l = mismatch_counts(r_feats[idx], ref)
        checked, bad = sum_over_ranks([len(idx), e + l])
        parity["render_extract_checked"], parity["render_extract_mismatches"] = checked, bad
        parity["all_mismatches"] += bad
        render_leg["parity"] = {"checked": checked, "mismatches": bad,
                                "against": "the reference simulator's renderers then tb_train_extract_features_cpu "
                                           "(oracle/_ref), every 97th aircraft"}

    clk = clocks.summary()
    clocks.close()
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, clk)
        if clk is not None:
            mhz = [g["sm_mhz"] for g in gathered if g and g["sm_mhz"] is not None]
            clk = dict(clk)
            clk["sm_mhz"] = statistics.median(mhz) if mhz else None
            clk["reasons"] = sorted({r for g in gathered if g for r in g["reasons"]})
            clk["per_rank_sm_mhz"] = [g["sm_mhz"] if g else None for g in gathered]

    failed = parity is not None and parity["all_mismatches"] != 0
    if rank != 0:
        if failed:
            raise SystemExit(1)
        return
    avg_launch_s = kernel_s / args.steps
    peak, peak_kind = measured_hbm_peak()
    achieved = count * tb.BYTES_PER_SAMPLE / avg_launch_s / 1e9
    tps = profiled_traffic_per_sample()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": 1e3 * kernel_s_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded SplitMix64 generator, BASELINE value model)",
        "config": workload_config(args, world),
        "e2e": {"value": e2e_value, "unit": UNIT,
                "h2d_bytes_per_step": count * (tb.OBS_DIM * 4 + tb.MISSION_DIM * 4 + tb.CAMERA_BYTES),
                "d2h_bytes_per_step": count * tb.FEATURE_DIM * 4,
                "ms_per_step": 1e3 * e2e_s_max / e2e_steps, "steps": e2e_steps,
                "api": "tb_cuda_extract_features_host, page-locked host buffers, host wall clock "
                       "(the call returns after its stream sync), max over ranks",
                "pageable": {"value": total / pageable_s, "unit": UNIT, "ms_per_step": pageable_s * 1e3,
                             "steps": p_steps,
                             "note": "same call with pageable (malloc'd) host buffers, as the reference "
                                     "trainer passes them"}},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                     "peak_note": "the copy peak is a device copy (half writes, fixed grid); this kernel "
                                  "reads 98 % of its bytes, and the best read-only stream measured on "
                                  "this pool is 7,094 GB/s (profiles/hbm_patterns_b200.md)",
                     "traffic": (tps * count) if tps else None,
                     "traffic_source": "not measured in this run: DRAM bytes per aircraft of the committed ncu "
                                       "capture (16,384 aircraft, profiles/features_flat_kernel_b16384.md) "
                                       "times this launch's aircraft",
                     "algorithmic_bytes_per_launch": count * tb.BYTES_PER_SAMPLE,
                     "kernel": "features_flat_kernel", "avg_launch_ms": avg_launch_s * 1e3},
        "gpu_launches": (args.steps + e2e_steps * chunks + (onboard["launches"] if onboard else 0) +
                         (f32cam["launches"] if f32cam else 0) + (actor["launches"] if actor else 0) +
                         (sensors["launches"] if sensors else 0) + (config1["launches"] if config1 else 0) +
                         reps + (render_leg["launches"] if render_leg else 0)),
        "gpu_launches_detail": {"value_region": args.steps, "e2e_region": e2e_steps * chunks,
                                "onboard_regions": onboard["launches"] if onboard else 0,
                                "f32cam_region": f32cam["launches"] if f32cam else 0,
                                "actor_inputs_region": actor["launches"] if actor else 0,
                                "sensors_regions": sensors["launches"] if sensors else 0,
                                "config1_region": config1["launches"] if config1 else 0,
                                "config3_e2e_region": reps,
                                "render_extract_region": render_leg["launches"] if render_leg else 0},
        "clocks": clk,
    }
    if f32cam is not None:
        line["f32_cameras"] = f32cam
    if actor is not None:
        line["actor_inputs"] = actor
    if onboard is not None:
        line["onboard"] = onboard
    if sensors is not None:
        line["sensors"] = sensors
    if config1 is not None:
        line["config1_latency"] = config1
    line["gather"] = gather
    line["config3_e2e"] = config3_e2e
    line["e2e"]["per_rank_h2d_gbs"] = per_rank_h2d
    if h2d is not None:
        line["host_to_device"] = h2d
    if parity is not None:
        line["parity"] = parity
    if render_leg is not None:
        line["render_extract"] = render_leg
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = time_reference_cpu(obs, mission, cams, args.cpu_seconds)
        if render_leg is not None:
            import oracle  # test infrastructure: the CPU baseline only

            if oracle.have_reference_sensors():
                threads = host_threads()
                k = min(count, threads * 256)
                r_scenes = render_check[0]
                _, t_r, t_f = render_extract_reference(r_scenes[:k], obs[:k, :48], obs[:k, 4144:4146],
                                                       mission[:k], threads)
                render_leg["cpu_baseline"] = {
                    "value": k / (t_r + t_f), "unit": UNIT, "cores": threads, "kind": "reference",
                    "sample": f"first {k} aircraft: the reference simulator's renderers ({t_r:.2f} s) then "
                              f"tb_train_extract_features_cpu ({t_f:.2f} s), oracle/_ref, {threads} threads"}
        if onboard is not None:
            onboard["cpu_baseline"] = time_onboard_reference_cpu(obs, mission, args.cpu_seconds / 2)
        if sensors is not None:
            import oracle  # test infrastructure: the CPU baseline only

            if oracle.have_reference_sensors():
                for name, scenes in sensor_scene_sets.items():
                    sensors[name]["cpu_baseline"] = time_sensors_reference_cpu(scenes, args.cpu_seconds / 2)
    print(json.dumps(line), flush=True)
    if failed:
        print(f"parity: {parity['all_mismatches']} mismatches against the oracle", file=sys.stderr)
        raise SystemExit(1)


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world != 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.config1_only:
        import torch

        torch.cuda.set_device(local_rank)
        tb.load_library()
        if rank == 0:
            print(json.dumps(time_config1(torch.cuda.Stream(), torch.device("cuda", local_rank))), flush=True)
        return
    if args.actor_inputs_only:
        import torch

        torch.cuda.set_device(local_rank)
        tb.load_library()
        if rank == 0:
            print(json.dumps(time_actor_inputs_only(args, torch.device("cuda", local_rank))), flush=True)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

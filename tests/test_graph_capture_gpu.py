"""The device entry points inside a CUDA graph: after a first call on the
device (which sets up launch attributes and, for the renderer, uploads the ray
tables), tb_cuda_extract_features_device, its FP32-camera variant,
tb_cuda_extract_onboard_device, tb_cuda_prepare_actor_inputs_device and
tb_cuda_render_sensors_device are plain launches on the caller's stream,
so a trainer can capture one step's calls and replay them.  Checked: the
replayed outputs equal the direct calls', and (printed) a config-1 replay's
latency against direct launches."""
from __future__ import annotations

import time

import numpy as np
import pytest

import turbinator_c_b200 as tb
from tests.sensor_cases import edge_scenes
from turbinator_c_b200.sensors import tb_cuda_render_sensors_device

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def test_step_captured_in_a_cuda_graph():
    n = 1024  # config 1
    obs, mission, cams, _ = tb.generate(1, 0, n)
    d_obs, d_mis, d_cam = (torch.from_numpy(x).cuda() for x in (obs, mission, cams))
    feats = torch.empty((n, 142), device="cuda")
    feats_f32 = torch.empty((n, 142), device="cuda")
    camf = d_cam.float() / 255.0
    tac, pri = torch.empty((n, 24), device="cuda"), torch.empty((n, 15), device="cuda")
    actor = [torch.empty(sh, device="cuda") for sh in
             ((n, 91), (n, 49), (n, 24), (n, 15), (n, 6 * 2048), (n, 16384))]
    scenes = edge_scenes()
    scenes["sensors"] = 3
    m = len(scenes)
    d_scenes = torch.from_numpy(scenes.view(np.uint8).reshape(-1).copy()).cuda()
    lidar = torch.empty((m, 4096), device="cuda")
    valid = torch.empty((m, 2), device="cuda")
    cams_out = torch.empty((m, 16384), dtype=torch.uint8, device="cuda")

    s = torch.cuda.Stream()

    def step():
        assert tb.tb_cuda_extract_features_device(d_obs, d_mis, d_cam, feats, n, s) == 1
        assert tb.tb_cuda_extract_features_device_f32cam(d_obs, d_mis, camf, feats_f32, n, s) == 1
        assert tb.tb_cuda_extract_onboard_device(d_obs, d_mis, tac, pri, n, s) == 1
        assert tb.tb_cuda_prepare_actor_inputs_device(d_obs, d_mis, d_cam, *actor, n, s) == 1
        assert tb_cuda_render_sensors_device(d_scenes, m, lidar, 4096, valid, 2, cams_out, None, s) == 1

    with torch.cuda.stream(s):
        step()  # first calls: per-device set-up happens here, outside the capture
    torch.cuda.synchronize()
    direct = [t.clone() for t in (feats, feats_f32, tac, pri, *actor, lidar, valid, cams_out)]
    for t in (feats, feats_f32, tac, pri, *actor, lidar, valid):
        t.fill_(float("nan"))
    cams_out.fill_(0)
    torch.cuda.synchronize()

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        step()
    with torch.cuda.stream(s):
        g.replay()
    torch.cuda.synchronize()
    assert tb.tb_cuda_synchronize(None) == 1
    for a, b in zip(direct, (feats, feats_f32, tac, pri, *actor, lidar, valid, cams_out)):
        if a.dtype == torch.uint8:
            assert torch.equal(a, b)
        else:
            assert torch.equal(a.view(torch.int32), b.view(torch.int32))

    # config-1 feature launch alone: graph replay against direct launch, host wall clock per call
    g1 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g1, stream=s):
        tb.tb_cuda_extract_features_device(d_obs, d_mis, d_cam, feats, n, s)

    def per_call(fn, iters=200):
        fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(iters):
            fn()
            s.synchronize()
        return (time.perf_counter() - t0) / iters * 1e6

    with torch.cuda.stream(s):  # graph replays go to the current stream: the same s as the direct calls
        direct_us = per_call(lambda: tb.tb_cuda_extract_features_device(d_obs, d_mis, d_cam, feats, n, s))
        replay_us = per_call(g1.replay)
    print(f"\nconfig 1 (1,024 aircraft), call to completion: direct {direct_us:.1f} us, graph replay {replay_us:.1f} us")
    assert tb.tb_cuda_synchronize(None) == 1

"""TEST INFRASTRUCTURE ONLY -- ctypes access to the CPU oracle.

Loads oracle/liboracle.so (the restated 142-feature oracle and its threaded
runner) and, when built, the reference's own CPU code in oracle/_ref/
(training.c's tb_train_extract_features_cpu and the onboard tactical/prior
header compiled for the host).  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs import this package; the shipped library never
does.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_PATH = os.path.join(HERE, "liboracle.so")
# the renderer restatement with the product kernel's square-root skip (test build)
ORACLE_SKIP_PATH = os.path.join(HERE, "liboracle_skip.so")
ORACLE_FLOAT_PATH = os.path.join(HERE, "liboracle_float.so")
REF_TRAINING_PATH = os.path.join(HERE, "_ref", "libtb_ref_training.so")
REF_ONBOARD_PATH = os.path.join(HERE, "_ref", "libtb_ref_onboard.so")
REF_ONBOARD_CR_PATH = os.path.join(HERE, "_ref", "libtb_ref_onboard_cr.so")
REF_ACTOR_INPUTS_PATH = os.path.join(HERE, "_ref", "libtb_ref_actor_inputs.so")

_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_oracle = None
_ref_training = None
_ref_onboard = None
_ref_onboard_cr = None


def _addr(a) -> Optional[int]:
    if a is None:
        return None
    return a.ctypes.data


def lib() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_PATH):
            raise RuntimeError(f"{ORACLE_PATH} missing: run `make -C oracle`")
        l = ctypes.CDLL(ORACLE_PATH)
        l.oracle_extract_features.restype = None
        l.oracle_extract_features.argtypes = [_vp, _vp, _vp, _vp]
        l.oracle_extract_batch.restype = ctypes.c_double
        l.oracle_extract_batch.argtypes = [_vp, _vp, _vp, _vp, _sz, _vp, ctypes.c_int]
        l.oracle_quantize_cameras.restype = None
        l.oracle_quantize_cameras.argtypes = [_vp, _sz, _vp]
        l.oracle_onboard_batch.restype = ctypes.c_double
        l.oracle_onboard_batch.argtypes = [_vp, _vp, _vp, _sz, _vp, ctypes.c_int]
        l.oracle_extract_batch_self.restype = ctypes.c_double
        l.oracle_extract_batch_self.argtypes = [_vp, _vp, _vp, _sz, _vp, ctypes.c_int]
        _oracle = l
    return _oracle


def have_reference() -> bool:
    return os.path.exists(REF_TRAINING_PATH)


def ref_training() -> ctypes.CDLL:
    global _ref_training
    if _ref_training is None:
        if not have_reference():
            raise RuntimeError(f"{REF_TRAINING_PATH} missing (reference build not available)")
        l = ctypes.CDLL(REF_TRAINING_PATH)
        l.tb_train_extract_features_cpu.restype = None
        l.tb_train_extract_features_cpu.argtypes = [_vp, _vp, _vp, _vp]
        _ref_training = l
    return _ref_training


def ref_onboard() -> ctypes.CDLL:
    global _ref_onboard
    if _ref_onboard is None:
        if not os.path.exists(REF_ONBOARD_PATH):
            raise RuntimeError(f"{REF_ONBOARD_PATH} missing (reference build not available)")
        l = ctypes.CDLL(REF_ONBOARD_PATH)
        l.tb_ref_onboard_batch.restype = None
        l.tb_ref_onboard_batch.argtypes = [_vp, _vp, _sz, _vp]
        l.tb_ref_onboard_tactical_prior.restype = None
        l.tb_ref_onboard_tactical_prior.argtypes = [_vp, _vp, _vp, _vp]
        _ref_onboard = l
    return _ref_onboard


def _check(obs, mission, cams):
    n = obs.shape[0]
    assert obs.dtype == np.float32 and obs.shape == (n, 4148) and obs.flags.c_contiguous
    assert mission.dtype == np.float32 and mission.shape == (n, 10) and mission.flags.c_contiguous
    if cams is not None:
        assert cams.dtype == np.uint8 and cams.shape == (n, 16384) and cams.flags.c_contiguous
    return n


def features(obs, mission, cams, threads: int = 0, use_reference: bool = False):
    """[n,142] features from the restated oracle (or the reference build)."""
    n = _check(obs, mission, cams)
    out = np.empty((n, 142), np.float32)
    if n == 0:
        return out
    threads = threads or os.cpu_count() or 1
    if use_reference:
        fn = ctypes.cast(ref_training().tb_train_extract_features_cpu, _vp).value
        t = lib().oracle_extract_batch(fn, _addr(obs), _addr(mission), _addr(cams), n, _addr(out), threads)
    else:
        t = lib().oracle_extract_batch_self(_addr(obs), _addr(mission), _addr(cams), n, _addr(out), threads)
    if t < 0:
        raise RuntimeError("oracle batch runner failed")
    return out


def timed_reference(obs, mission, cams, out, threads: int) -> float:
    """Wall seconds for the reference's own CPU function over the batch."""
    n = _check(obs, mission, cams)
    fn = ctypes.cast(ref_training().tb_train_extract_features_cpu, _vp).value
    t = lib().oracle_extract_batch(fn, _addr(obs), _addr(mission), _addr(cams), n, _addr(out), threads)
    if t < 0:
        raise RuntimeError("oracle batch runner failed")
    return t


def timed_port(obs, mission, cams, out, threads: int) -> float:
    """Wall seconds for the restated oracle over the batch."""
    n = _check(obs, mission, cams)
    t = lib().oracle_extract_batch_self(_addr(obs), _addr(mission), _addr(cams), n, _addr(out), threads)
    if t < 0:
        raise RuntimeError("oracle batch runner failed")
    return t


def onboard_reference(obs, mission):
    """[n,39] onboard tactical(24)+prior(15) from the reference header built for the host."""
    n = obs.shape[0]
    assert obs.dtype == np.float32 and obs.shape == (n, 4148) and obs.flags.c_contiguous
    assert mission.dtype == np.float32 and mission.shape == (n, 10) and mission.flags.c_contiguous
    out = np.empty((n, 39), np.float32)
    ref_onboard().tb_ref_onboard_batch(_addr(obs), _addr(mission), n, _addr(out))
    return out


def ref_onboard_cr() -> ctypes.CDLL:
    global _ref_onboard_cr
    if _ref_onboard_cr is None:
        if not os.path.exists(REF_ONBOARD_CR_PATH):
            raise RuntimeError(f"{REF_ONBOARD_CR_PATH} missing (reference build not available)")
        l = ctypes.CDLL(REF_ONBOARD_CR_PATH)
        l.tb_ref_onboard_cr_batch.restype = None
        l.tb_ref_onboard_cr_batch.argtypes = [_vp, _vp, _sz, _vp]
        _ref_onboard_cr = l
    return _ref_onboard_cr


def onboard_reference_cr(obs, mission):
    """[n,39] from the reference header with correctly rounded float transcendentals."""
    n = obs.shape[0]
    assert obs.dtype == np.float32 and obs.shape == (n, 4148) and obs.flags.c_contiguous
    assert mission.dtype == np.float32 and mission.shape == (n, 10) and mission.flags.c_contiguous
    out = np.empty((n, 39), np.float32)
    ref_onboard_cr().tb_ref_onboard_cr_batch(_addr(obs), _addr(mission), n, _addr(out))
    return out


def timed_onboard_reference(obs, mission, out, threads: int) -> float:
    """Wall seconds for the reference onboard header (glibc build) over the
    batch on `threads` host threads; fills out [n,39]."""
    n = obs.shape[0]
    assert obs.flags.c_contiguous and mission.flags.c_contiguous and out.shape == (n, 39)
    fn = ctypes.cast(ref_onboard().tb_ref_onboard_tactical_prior, _vp).value
    t = lib().oracle_onboard_batch(fn, _addr(obs), _addr(mission), n, _addr(out), threads)
    if t < 0:
        raise RuntimeError("oracle onboard runner failed")
    return t


def quantize_cameras(cameras_f32):
    """u8 cameras from float luma with the simulator's rule (sensors.c:67)."""
    c = np.ascontiguousarray(cameras_f32, np.float32)
    out = np.empty(c.shape, np.uint8)
    lib().oracle_quantize_cameras(_addr(c), c.size, _addr(out))
    return out


def actor_inputs_cpu(obs, mission, cameras, tactical, prior):
    """CPU restatement of the reference's learner input preparation
    (src/network/network_gpu.cu:274-303 scalar_inputs, :467-479
    lidar_channels, :480-483 camera_luma), given the onboard tactical/prior
    values.  float32 arithmetic; the symlog uses numpy's log1p, so it may
    differ from the GPU's log1pf in the last bits (the other tensors are
    exact: IEEE divisions, and the luma multiply-add evaluated exactly and
    rounded once, as the GPU's fused multiply-add does)."""
    n = obs.shape[0]
    f32 = np.float32
    raw = np.concatenate([obs[:, :48], obs[:, 4144:4148]], axis=1).astype(f32)
    raw = np.where(np.isfinite(raw), np.clip(raw, f32(-1000), f32(1000)), f32(0)).astype(f32)
    scale = np.ones(52, f32)
    scale[0:3] = 0.05; scale[3:6] = 0.10; scale[10:13] = 0.20; scale[13:16] = 0.10
    scale[28:32] = 0.50; scale[32:36] = 0.20
    symlog = np.copysign(np.log1p(np.abs(raw * scale)).astype(f32), raw).astype(f32)
    proprio = np.empty((n, 91), f32)
    proprio[:, :52] = np.clip(symlog / np.sqrt(f32(1.0001)).astype(f32), f32(-8), f32(8))
    proprio[:, 52:76] = tactical
    proprio[:, 76:91] = prior
    mission_vec = np.empty((n, 49), f32)
    mission_vec[:, :10] = np.where(np.isfinite(mission), mission, f32(0))
    mission_vec[:, 10:34] = tactical
    mission_vec[:, 34:49] = prior
    r = obs[:, 48:4144].reshape(n, 2, 2048).astype(f32)
    with np.errstate(invalid="ignore"):
        valid = (r > 0) & np.isfinite(r)
        clamped = np.maximum(f32(0.05), np.minimum(f32(30), np.nan_to_num(r, nan=0.0))).astype(f32)
        inverse = np.where(valid, (f32(1) / np.maximum(f32(0.2), clamped)).astype(f32), f32(0))
        scaled = np.where(valid, (clamped / f32(30)).astype(f32), f32(1))
    lidar = np.concatenate([inverse, scaled, valid.astype(f32)], axis=1).astype(f32)
    k = np.float64(f32(1) / f32(255))
    luma = (cameras.astype(np.float64) * k - 0.5).astype(f32)
    return {"proprio": proprio, "mission": mission_vec, "lidar": lidar, "luma": luma}


def have_reference_actor_inputs() -> bool:
    return os.path.exists(REF_ACTOR_INPUTS_PATH)


_ref_actor = None


def actor_inputs_reference_gpu(d_obs, d_mission, d_cameras, outs, n: int) -> None:
    """Run the reference's own GPU input-preparation kernels (oracle/_ref) on
    device buffers: outs = (proprio, mission_vec, tactical, prior, lidar, luma)
    torch tensors; synchronous."""
    global _ref_actor
    if _ref_actor is None:
        l = ctypes.CDLL(REF_ACTOR_INPUTS_PATH)
        l.tb_ref_actor_inputs.restype = ctypes.c_int
        l.tb_ref_actor_inputs.argtypes = [_vp] * 9 + [ctypes.c_int]
        _ref_actor = l
    ptrs = [t.data_ptr() for t in (d_obs, d_mission, d_cameras, *outs)]
    if not _ref_actor.tb_ref_actor_inputs(*ptrs, n):
        raise RuntimeError("reference input-preparation launch failed")
    import torch
    torch.cuda.synchronize()


# ---- sensor rendering (tb_cuda_render_sensors_device's checker) ----

REF_SENSORS_PATH = os.path.join(HERE, "_ref", "libtb_ref_sensors.so")
_ref_sensors = None
_sensor_port_bound = False


def _sensor_port() -> ctypes.CDLL:
    global _sensor_port_bound
    l = lib()
    if not _sensor_port_bound:
        l.oracle_render_sensors.restype = None
        l.oracle_render_sensors.argtypes = [_vp, ctypes.c_int64, _vp, ctypes.c_int64, _vp, ctypes.c_int64, _vp, _vp]
        l.oracle_sensor_scene_layout.restype = None
        l.oracle_sensor_scene_layout.argtypes = [_vp]
        _sensor_port_bound = True
    return l


def have_reference_sensors() -> bool:
    return os.path.exists(REF_SENSORS_PATH)


def ref_sensors() -> ctypes.CDLL:
    global _ref_sensors
    if _ref_sensors is None:
        if not have_reference_sensors():
            raise RuntimeError(f"{REF_SENSORS_PATH} missing (reference build not available)")
        l = ctypes.CDLL(REF_SENSORS_PATH)
        l.ref_sensors_render.restype = ctypes.c_double
        l.ref_sensors_render.argtypes = [_vp, ctypes.c_int64, _vp, ctypes.c_int64, _vp, ctypes.c_int64, _vp, _vp,
                                         ctypes.c_int]
        l.ref_sensors_simulate.restype = ctypes.c_int
        l.ref_sensors_simulate.argtypes = [ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]
        _ref_sensors = l
    return _ref_sensors


def sensor_scene_layout():
    """(sizeof, offsets of the 14 fields) of tb_sensor_scene as C lays it out."""
    out = np.zeros(15, np.int64)
    _sensor_port().oracle_sensor_scene_layout(_addr(out))
    return out


def _sensor_outputs(n: int, raw: bool):
    lidar = np.full((n, 4096), np.nan, np.float32)
    valid = np.full((n, 2), np.nan, np.float32)
    cams = np.zeros((n, 16384), np.uint8)
    raws = np.zeros((n, 147456), np.uint8) if raw else None
    return lidar, valid, cams, raws


_oracle_skip = None


def _sensor_port_skip() -> ctypes.CDLL:
    global _oracle_skip
    if _oracle_skip is None:
        if not os.path.exists(ORACLE_SKIP_PATH):
            raise RuntimeError(f"{ORACLE_SKIP_PATH} missing: run `make -C oracle`")
        l = ctypes.CDLL(ORACLE_SKIP_PATH)
        l.oracle_render_sensors.restype = None
        l.oracle_render_sensors.argtypes = [_vp, ctypes.c_int64, _vp, ctypes.c_int64, _vp, ctypes.c_int64, _vp, _vp]
        l.oracle_sqrt_skips.restype = ctypes.c_uint64
        l.oracle_sqrt_skips.argtypes = []
        _oracle_skip = l
    return _oracle_skip


_oracle_float = None


def _sensor_port_float() -> ctypes.CDLL:
    global _oracle_float
    if _oracle_float is None:
        if not os.path.exists(ORACLE_FLOAT_PATH):
            raise RuntimeError(f"{ORACLE_FLOAT_PATH} missing: run `make -C oracle`")
        l = ctypes.CDLL(ORACLE_FLOAT_PATH)
        l.oracle_render_sensors.restype = None
        l.oracle_render_sensors.argtypes = [_vp, ctypes.c_int64, _vp, ctypes.c_int64, _vp, ctypes.c_int64, _vp, _vp]
        l.oracle_float_pixels.restype = ctypes.c_uint64
        l.oracle_float_pixels.argtypes = []
        _oracle_float = l
    return _oracle_float


def float_pixels() -> int:
    """Camera pixels the float-decision build has decided so far in this process."""
    return int(_sensor_port_float().oracle_float_pixels())


def render_sensors_port(scenes, raw: bool = False, sqrt_skip: bool = False, float_camera: bool = False):
    """Restated renderers (sensors_oracle.c): (lidar [n,4096], valid [n,2],
    cameras [n,16384], raw [n,147456] or None); unrendered rows keep NaN / 0.
    sqrt_skip=True renders with the test build that drops spheres without the
    square root under the product kernel's condition; float_camera=True with
    the test build that first offers every camera pixel to the product
    kernel's float decision (tb_camera_float.h)."""
    scenes = np.ascontiguousarray(scenes)
    n = scenes.shape[0]
    lidar, valid, cams, raws = _sensor_outputs(n, raw)
    port = _sensor_port_skip() if sqrt_skip else (_sensor_port_float() if float_camera else _sensor_port())
    port.oracle_render_sensors(_addr(scenes), n, _addr(lidar), 4096, _addr(valid), 2, _addr(cams), _addr(raws))
    return lidar, valid, cams, raws


def sqrt_skips() -> int:
    """Spheres the skip build has dropped so far in this process."""
    return int(_sensor_port_skip().oracle_sqrt_skips())


def render_sensors_reference(scenes, raw: bool = False, threads: int = 0):
    """The reference simulator's own renderers on the same scenes (same
    outputs as render_sensors_port)."""
    scenes = np.ascontiguousarray(scenes)
    n = scenes.shape[0]
    lidar, valid, cams, raws = _sensor_outputs(n, raw)
    t = ref_sensors().ref_sensors_render(_addr(scenes), n, _addr(lidar), 4096, _addr(valid), 2, _addr(cams),
                                         _addr(raws), threads or min(os.cpu_count() or 1, 64))
    if t < 0:
        raise RuntimeError("reference sensor renderer failed")
    return lidar, valid, cams, raws


def timed_sensors_reference(scenes, threads: int) -> float:
    """Wall seconds for the reference renderers over the scenes on `threads`
    host threads (LiDAR, valid fractions and cameras)."""
    scenes = np.ascontiguousarray(scenes)
    n = scenes.shape[0]
    lidar, valid, cams, _ = _sensor_outputs(n, False)
    t = ref_sensors().ref_sensors_render(_addr(scenes), n, _addr(lidar), 4096, _addr(valid), 2, _addr(cams), None,
                                         threads)
    if t < 0:
        raise RuntimeError("reference sensor renderer failed")
    return t


def simulate_sensor_scenes(scenarios, seeds, steps, players, scene_dtype):
    """Scenes packed from simulated episodes plus the reference's renders of
    those environments: (scenes, lidar, valid, cameras)."""
    n = len(scenarios)
    sc = np.ascontiguousarray(scenarios, np.int32)
    sd = np.ascontiguousarray(seeds, np.uint64)
    st = np.ascontiguousarray(steps, np.int32)
    pl = np.ascontiguousarray(players, np.int32)
    scenes = np.zeros(n, scene_dtype)
    lidar = np.empty((n, 4096), np.float32)
    valid = np.empty((n, 2), np.float32)
    cams = np.empty((n, 16384), np.uint8)
    if ref_sensors().ref_sensors_simulate(n, _addr(sc), _addr(sd), _addr(st), _addr(pl), _addr(scenes),
                                          _addr(lidar), _addr(valid), _addr(cams)) != 0:
        raise RuntimeError("reference simulation failed")
    return scenes, lidar, valid, cams


# ---- the reference's own GPU feature path (src/cuda/features.cu for sm_100a) ----

REF_CUDA_FEATURES_PATH = os.path.join(HERE, "_ref", "libtb_ref_cuda_features.so")
_ref_cuda_features = None


def have_reference_gpu_features() -> bool:
    return os.path.exists(REF_CUDA_FEATURES_PATH)


def ref_cuda_features() -> ctypes.CDLL:
    """The reference's GPU feature library, loaded privately (RTLD_LOCAL): its
    symbols carry the same names as this repository's library."""
    global _ref_cuda_features
    if _ref_cuda_features is None:
        if not have_reference_gpu_features():
            raise RuntimeError(f"{REF_CUDA_FEATURES_PATH} missing (reference build not available)")
        l = ctypes.CDLL(REF_CUDA_FEATURES_PATH, mode=ctypes.RTLD_LOCAL)
        l.tb_cuda_extract_features_device.restype = ctypes.c_int
        l.tb_cuda_extract_features_device.argtypes = [_vp, _vp, _vp, _vp, _sz, _vp]
        l.tb_cuda_synchronize.restype = ctypes.c_int
        l.tb_cuda_synchronize.argtypes = [_vp]
        _ref_cuda_features = l
    return _ref_cuda_features

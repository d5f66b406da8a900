"""B200-native batched sensor features for Turbinator C -- Python view of the C ABI.

The product is the C-ABI shared library ``libturbinator_cuda.so`` built from
``turbinator_c_b200/csrc`` (sm_100a CUDA kernels + C11 host code), whose
entry points are declared in ``include/turbinator/training/cuda_features.h``
and replace the reference's ``include/turbinator/training/cuda_features.h``.
This module binds those entry points with ctypes under the same names, so the
parity tests and the benchmark call exactly what a C11 trainer links.  There
is no Python or CPU implementation of the features here: if the library is
missing, every entry point raises.

Layouts (row-major, one row per aircraft): obs [B,4148] f32, mission [B,10]
f32, cameras [B,16384] u8, features [B,142] f32.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import numpy as np

OBS_DIM = 4148
MISSION_DIM = 10
CAMERA_BYTES = 16384
FEATURE_DIM = 142
ONBOARD_DIM = 39

#: Algorithmic HBM bytes per aircraft for the u8-camera entry point
#: (16,592 obs + 40 mission + 16,384 cameras read, 568 features written).
BYTES_PER_SAMPLE = OBS_DIM * 4 + MISSION_DIM * 4 + CAMERA_BYTES + FEATURE_DIM * 4
#: The same for the FP32-camera entry point (65,536 camera bytes read).
BYTES_PER_SAMPLE_F32CAM = OBS_DIM * 4 + MISSION_DIM * 4 + 4 * CAMERA_BYTES + FEATURE_DIM * 4
#: Learner input tensors: 33,016 bytes read; proprio 91 + mission 49 + tactical 24 + prior 15
#: + LiDAR 6 x 2048 + luma 16,384 floats written.
BYTES_PER_SAMPLE_ACTOR_INPUTS = (OBS_DIM * 4 + MISSION_DIM * 4 + CAMERA_BYTES +
                                 4 * (91 + 49 + 24 + 15 + 6 * 2048 + CAMERA_BYTES))

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libturbinator_cuda.so")
#: The same library with the feature kernels' bounds checks compiled in
#: (TB_FEATURES_DEBUG): tests load it in a separate process by setting
#: TB_CUDA_LIBRARY to this path.
DEBUG_LIB_PATH = os.path.join(_HERE, "libturbinator_cuda_debug.so")
if os.environ.get("TB_CUDA_LIBRARY"):
    LIB_PATH = os.environ["TB_CUDA_LIBRARY"]
SYNTH_PATH = os.path.join(_HERE, "libtb_synth.so")

_lib: Optional[ctypes.CDLL] = None
_synth: Optional[ctypes.CDLL] = None

_c = ctypes
_vp = _c.c_void_p
_sz = _c.c_size_t


class LaunchOpts(_c.Structure):
    """Mirror of ``tb_features_launch_opts`` (csrc/tb_features_internal.h)."""

    _fields_ = [
        ("force_direct", _c.c_int),
        ("grid_limit", _c.c_int),
        ("wait_ns", _c.c_ulonglong),
        ("stall_sample", _c.c_longlong),
        ("flat", _c.c_int),
    ]


def _bind(lib: ctypes.CDLL, name: str, restype, argtypes) -> None:
    fn = getattr(lib, name)
    fn.restype = restype
    fn.argtypes = argtypes


def load_library() -> ctypes.CDLL:
    """Load the in-tree C-ABI library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(there is no fallback implementation)")
    lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
    _bind(lib, "tb_cuda_extract_features_device", _c.c_int, [_vp, _vp, _vp, _vp, _sz, _vp])
    _bind(lib, "tb_cuda_synchronize", _c.c_int, [_vp])
    _bind(lib, "tb_cuda_feature_batch_create", _vp, [_c.c_int, _sz])
    _bind(lib, "tb_cuda_feature_batch_create_multi", _vp, [_c.POINTER(_c.c_int), _c.c_int, _sz])
    _bind(lib, "tb_cuda_feature_batch_destroy", None, [_vp])
    _bind(lib, "tb_cuda_feature_batch_error", _c.c_char_p, [_vp])
    _bind(lib, "tb_cuda_extract_features_host", _c.c_int, [_vp, _vp, _vp, _vp, _sz, _vp])
    _bind(lib, "tb_cuda_extract_features_host_noalloc", _c.c_int, [_vp, _vp, _vp, _sz, _vp, _vp])
    _bind(lib, "tb_cuda_extract_onboard_device", _c.c_int, [_vp, _vp, _vp, _vp, _sz, _vp])
    _bind(lib, "tb_cuda_extract_features_device_f32cam", _c.c_int, [_vp, _vp, _vp, _vp, _sz, _vp])
    _bind(lib, "tb_cuda_prepare_actor_inputs_device", _c.c_int, [_vp] * 9 + [_sz, _vp])
    _bind(lib, "tb_cuda_render_sensors_device", _c.c_int, [_vp, _sz, _vp, _sz, _vp, _sz, _vp, _vp, _vp])
    _bind(lib, "tb_cuda_extract_features_device_sharded", _c.c_int,
          [_c.c_int, _c.POINTER(_c.c_int)] + [_c.POINTER(_vp)] * 4 + [_c.POINTER(_sz), _c.POINTER(_vp)])
    _bind(lib, "tb_onboard_launch", _c.c_int, [_vp] * 4 + [_sz, _vp, _c.POINTER(LaunchOpts)])
    _bind(lib, "tb_actor_inputs_launch", _c.c_int, [_vp] * 9 + [_sz, _vp, _c.POINTER(LaunchOpts)])
    _bind(lib, "tb_actor_inputs_scan_launch", _c.c_int, [_vp] * 8 + [_sz, _vp, _c.POINTER(LaunchOpts)])
    _bind(lib, "tb_features_launch_f32cam", _c.c_int,
          [_vp, _vp, _vp, _vp, _sz, _vp, _c.POINTER(LaunchOpts)])
    _bind(lib, "tb_features_launch", _c.c_int,
          [_vp, _vp, _vp, _vp, _sz, _vp, _c.POINTER(LaunchOpts)])
    _bind(lib, "tb_status_take", _c.c_int, [_vp, _c.POINTER(_c.c_uint)])
    _bind(lib, "tb_features_staged_config", _c.c_int,
          [_c.POINTER(_c.c_int)] * 5)
    _lib = lib
    return lib


def _ptr(x) -> Optional[int]:
    """Address of a torch tensor, numpy array, raw int or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    raise TypeError(f"cannot take the address of {type(x)!r}")


def _stream_handle(stream) -> Optional[int]:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream  # torch.cuda.Stream


# ---- the six reference entry points, same names and return values ----

def tb_cuda_extract_features_device(obs, mission, cameras, features, batch_size: int,
                                    stream=None) -> int:
    return load_library().tb_cuda_extract_features_device(
        _ptr(obs), _ptr(mission), _ptr(cameras), _ptr(features), batch_size, _stream_handle(stream))


def tb_cuda_synchronize(stream=None) -> int:
    return load_library().tb_cuda_synchronize(_stream_handle(stream))


def tb_cuda_feature_batch_create(device_id: int, max_batch: int) -> Optional[int]:
    return load_library().tb_cuda_feature_batch_create(device_id, max_batch)


def tb_cuda_feature_batch_destroy(handle: Optional[int]) -> None:
    load_library().tb_cuda_feature_batch_destroy(handle)


def tb_cuda_feature_batch_error(handle: Optional[int]) -> str:
    return load_library().tb_cuda_feature_batch_error(handle).decode()


def tb_cuda_extract_features_host(handle: Optional[int], obs, mission, cameras, count: int,
                                  out_features) -> int:
    return load_library().tb_cuda_extract_features_host(
        handle, _ptr(obs), _ptr(mission), _ptr(cameras), count, _ptr(out_features))


# ---- additive entry points ----

def tb_cuda_prepare_actor_inputs_device(obs, mission, cameras, proprio_91, mission_49, tactical_24, prior_15,
                                        lidar_6x2048, camera_luma, batch_size: int, stream=None) -> int:
    """The 618M learner's input tensors (device pointers)."""
    return load_library().tb_cuda_prepare_actor_inputs_device(
        _ptr(obs), _ptr(mission), _ptr(cameras), _ptr(proprio_91), _ptr(mission_49), _ptr(tactical_24),
        _ptr(prior_15), _ptr(lidar_6x2048), _ptr(camera_luma), batch_size, _stream_handle(stream))


def tb_cuda_extract_features_device_f32cam(obs, mission, cameras_f32, features, batch_size: int,
                                           stream=None) -> int:
    """142 features from FP32 cameras [B,16384] quantised like the simulator."""
    return load_library().tb_cuda_extract_features_device_f32cam(
        _ptr(obs), _ptr(mission), _ptr(cameras_f32), _ptr(features), batch_size, _stream_handle(stream))


def launch_f32cam(obs, mission, cameras_f32, features, batch_size: int, stream=None, *,
                  force_direct: bool = False, grid_limit: int = 0) -> int:
    opts = LaunchOpts(int(force_direct), int(grid_limit), 0, -1, 0)
    return load_library().tb_features_launch_f32cam(
        _ptr(obs), _ptr(mission), _ptr(cameras_f32), _ptr(features), batch_size,
        _stream_handle(stream), _c.byref(opts))


def tb_cuda_extract_onboard_device(obs, mission, tactical_24, prior_15, batch_size: int,
                                   stream=None) -> int:
    """Onboard tactical [B,24] and prior [B,15] values (device pointers)."""
    return load_library().tb_cuda_extract_onboard_device(
        _ptr(obs), _ptr(mission), _ptr(tactical_24), _ptr(prior_15), batch_size, _stream_handle(stream))


def tb_cuda_extract_features_device_sharded(device_ids, obs, mission, cameras, features, batch_sizes,
                                            streams=None) -> int:
    """Per-shard lists (device ids, device tensors or pointers, batch sizes,
    optional streams); cameras may be None or a list with None entries."""
    n = len(device_ids)
    arr = lambda xs: (_vp * n)(*[_ptr(x) for x in xs])
    cams = None if cameras is None else arr(cameras)
    st = None if streams is None else (_vp * n)(*[_stream_handle(x) for x in streams])
    return load_library().tb_cuda_extract_features_device_sharded(
        n, (_c.c_int * n)(*device_ids), arr(obs), arr(mission), cams, arr(features), (_sz * n)(*batch_sizes), st)


#: Largest count accepted by tb_cuda_extract_features_host_noalloc (cuda_features.h).
NOALLOC_MAX_BATCH = 64


def tb_cuda_extract_features_host_noalloc(obs, mission, cameras, count: int, out_features,
                                          stream=None) -> int:
    """Handle-free host extraction staged through the library's fixed device
    array (for callers that cannot allocate device memory).  1 = success,
    -1 = count is 0 or above NOALLOC_MAX_BATCH, 0 = NULL pointer or CUDA error."""
    return load_library().tb_cuda_extract_features_host_noalloc(
        _ptr(obs), _ptr(mission), _ptr(cameras), count, _ptr(out_features), _stream_handle(stream))


# ---- internal hooks used by tests and the benchmark ----

def launch(obs, mission, cameras, features, batch_size: int, stream=None, *,
           force_direct: bool = False, grid_limit: int = 0, wait_ns: int = 0,
           stall_sample: int = -1, flat: int = 0) -> int:
    """``tb_features_launch`` with explicit options (kernel choice, grid cap,
    pipeline wait limit, the test-only stalled-sample hook, and the u8 kernel:
    flat >= 0 the one-CTA-per-aircraft kernel (the default), -1 the staged
    ring kernel)."""
    opts = LaunchOpts(int(force_direct), int(grid_limit), int(wait_ns), int(stall_sample), int(flat))
    return load_library().tb_features_launch(
        _ptr(obs), _ptr(mission), _ptr(cameras), _ptr(features), batch_size,
        _stream_handle(stream), _c.byref(opts))


def launch_onboard(obs, mission, tactical, prior, batch_size: int, stream=None, *, wait_ns: int = 0,
                   stall_sample: int = -1) -> int:
    """tb_cuda_extract_onboard_device with the test hook (bounded waits)."""
    opts = LaunchOpts(0, 0, wait_ns, stall_sample, 0)
    return load_library().tb_onboard_launch(_ptr(obs), _ptr(mission), _ptr(tactical), _ptr(prior), batch_size,
                                            _stream_handle(stream), _c.byref(opts))


def launch_actor_inputs(obs, mission, cameras, tactical, prior, proprio, mission_vec, lidar, luma, batch_size: int,
                        stream=None, *, wait_ns: int = 0, stall_sample: int = -1) -> int:
    """The learner-input streaming kernel alone (test hook: bounded waits)."""
    opts = LaunchOpts(0, 0, wait_ns, stall_sample, 0)
    return load_library().tb_actor_inputs_launch(
        _ptr(obs), _ptr(mission), _ptr(cameras), _ptr(tactical), _ptr(prior), _ptr(proprio), _ptr(mission_vec),
        _ptr(lidar), _ptr(luma), batch_size, _stream_handle(stream), _c.byref(opts))


def launch_actor_inputs_scan(obs, mission, cameras, prior, proprio, mission_vec, lidar, luma, batch_size: int,
                             stream=None, *, wait_ns: int = 0, stall_sample: int = -1) -> int:
    """The learner-input streaming kernel as the learner-input entry point
    launches it (it also scans the LiDAR rows of the dodge and slalom aircraft
    and parks the results in `prior`); test hook: bounded waits."""
    opts = LaunchOpts(0, 0, wait_ns, stall_sample, 0)
    return load_library().tb_actor_inputs_scan_launch(
        _ptr(obs), _ptr(mission), _ptr(cameras), _ptr(prior), _ptr(proprio), _ptr(mission_vec), _ptr(lidar),
        _ptr(luma), batch_size, _stream_handle(stream), _c.byref(opts))


def take_status(stream=None) -> int:
    """Read and clear `stream`'s kernel status word on the current device (0 = clean)."""
    value = _c.c_uint(0)
    if not load_library().tb_status_take(_stream_handle(stream), _c.byref(value)):
        raise RuntimeError("could not read the feature kernel status word")
    return value.value


def staged_config() -> dict:
    vals = [_c.c_int(0) for _ in range(5)]
    if not load_library().tb_features_staged_config(*[_c.byref(v) for v in vals]):
        raise RuntimeError("tb_features_staged_config failed (no CUDA device?)")
    keys = ("blocks_per_sm", "sms", "smem_bytes", "threads", "stages")
    return {k: v.value for k, v in zip(keys, vals)}


def tb_cuda_feature_batch_create_multi(device_ids, max_batch: int) -> Optional[int]:
    ids = (_c.c_int * len(device_ids))(*device_ids)
    return load_library().tb_cuda_feature_batch_create_multi(ids, len(device_ids), max_batch)


class FeatureBatch:
    """RAII wrapper over a ``tb_cuda_feature_batch`` handle (host-pointer ABI).
    ``device_id`` may be a list of devices for a sample-sharded handle."""

    def __init__(self, device_id, max_batch: int):
        if isinstance(device_id, (list, tuple)):
            self.handle = tb_cuda_feature_batch_create_multi(list(device_id), max_batch)
        else:
            self.handle = tb_cuda_feature_batch_create(device_id, max_batch)
        if not self.handle:
            raise RuntimeError(f"tb_cuda_feature_batch_create({device_id}, {max_batch}) failed")
        self.max_batch = max_batch

    def extract(self, obs, mission, cameras, count: int, out) -> int:
        return tb_cuda_extract_features_host(self.handle, obs, mission, cameras, count, out)

    def error(self) -> str:
        return tb_cuda_feature_batch_error(self.handle)

    def close(self) -> None:
        if self.handle:
            tb_cuda_feature_batch_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass


# ---- seeded synthetic batches (libtb_synth.so) ----

SYNTH_STANDARD, SYNTH_CAMERA_EXTREME, SYNTH_LIDAR_NORETURN, SYNTH_LIDAR_DUPMIN, SYNTH_LIDAR_HALF = range(5)

#: Benchmark configurations: (seed, batch, stress quarters?)
CONFIGS = {
    0: (0, 8, False),
    1: (1, 1024, False),
    2: (2, 65536, False),
    3: (3, 524288, False),
    4: (4, 131072, True),
}


def _load_synth() -> ctypes.CDLL:
    global _synth
    if _synth is None:
        if not os.path.exists(SYNTH_PATH):
            raise RuntimeError(f"{SYNTH_PATH} is missing: run the build first")
        lib = ctypes.CDLL(SYNTH_PATH)
        _bind(lib, "tb_synth_generate", _c.c_int,
              [_c.c_uint64, _c.c_uint64, _sz, _c.c_int, _vp, _vp, _vp, _vp, _c.c_int])
        _synth = lib
    return _synth


def allocate_batch(count: int, pinned: bool = False, f32_cameras: bool = False):
    """Host arrays for `count` samples; page-locked (via torch) if pinned."""
    if pinned:
        import torch
        obs = torch.empty((count, OBS_DIM), dtype=torch.float32, pin_memory=True).numpy()
        mission = torch.empty((count, MISSION_DIM), dtype=torch.float32, pin_memory=True).numpy()
        cams = torch.empty((count, CAMERA_BYTES), dtype=torch.uint8, pin_memory=True).numpy()
        camf = (torch.empty((count, CAMERA_BYTES), dtype=torch.float32, pin_memory=True).numpy()
                if f32_cameras else None)
    else:
        obs = np.empty((count, OBS_DIM), np.float32)
        mission = np.empty((count, MISSION_DIM), np.float32)
        cams = np.empty((count, CAMERA_BYTES), np.uint8)
        camf = np.empty((count, CAMERA_BYTES), np.float32) if f32_cameras else None
    return obs, mission, cams, camf


def generate_into(seed: int, first: int, count: int, mode: int, obs, mission, cams, camf=None,
                  threads: int = 0) -> None:
    if count == 0:
        return
    ok = _load_synth().tb_synth_generate(seed, first, count, mode, _ptr(obs), _ptr(mission),
                                         _ptr(cams), _ptr(camf), threads)
    if not ok:
        raise RuntimeError("tb_synth_generate rejected its arguments")


def stress_mode(index: int, total: int) -> int:
    """Stress quarter (a..d -> modes 1..4) of sample `index` in a `total` batch."""
    return 1 + (4 * index) // total


def generate(seed: int, first: int, count: int, *, total: Optional[int] = None,
             stress: bool = False, threads: int = 0, pinned: bool = False,
             f32_cameras: bool = False):
    """Samples [first, first+count) of a seeded batch of `total` samples.

    With stress=True the batch is split into four equal quarters of stress
    modes (a) camera extremes, (b) all no-return, (c) duplicated sector
    minima, (d) all 0.5 m; quarters are positions in the whole batch, so any
    shard is generated consistently.  Returns (obs, mission, cameras_u8,
    cameras_f32 or None).
    """
    total = first + count if total is None else total
    obs, mission, cams, camf = allocate_batch(count, pinned, f32_cameras)
    if not stress:
        generate_into(seed, first, count, SYNTH_STANDARD, obs, mission, cams, camf, threads)
        return obs, mission, cams, camf
    i, end = first, first + count
    while i < end:
        mode = stress_mode(i, total)
        # first index of the next quarter: smallest j with 4*j >= mode*total
        j = min(end, -(-mode * total // 4))
        s = slice(i - first, j - first)
        generate_into(seed, i, j - i, mode, obs[s], mission[s], cams[s],
                      None if camf is None else camf[s], threads)
        i = j
    return obs, mission, cams, camf

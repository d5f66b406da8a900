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
REF_TRAINING_PATH = os.path.join(HERE, "_ref", "libtb_ref_training.so")
REF_ONBOARD_PATH = os.path.join(HERE, "_ref", "libtb_ref_onboard.so")
REF_ONBOARD_CR_PATH = os.path.join(HERE, "_ref", "libtb_ref_onboard_cr.so")

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

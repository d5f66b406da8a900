"""The reference's own GPU feature kernel (src/cuda/features.cu:113-169,
compiled unchanged for sm_100a into oracle/_ref) as a second reference
column: on the same resident inputs its features and this library's both
agree with the reference CPU path within the parity tolerance (bit-exact for
the integer-derived features), and this library's kernel is timed against it
at config 2 (65,536 aircraft; CUDA events, inputs far above the L2 size)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import turbinator_c_b200 as tb
from tests.parity import check_features

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not oracle.have_reference_gpu_features(),
                                 reason="reference GPU build (oracle/_ref) not available")]


def _device(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrays]


@pytest.mark.parametrize("seed,n,stress", [(1, 1024, False), (4, 4096, True)])
def test_reference_kernel_and_this_library_agree_with_the_cpu_path(seed, n, stress):
    obs, mission, cams, _ = tb.generate(seed, 0, n, total=n, stress=stress)
    expected = oracle.features(obs, mission, cams)
    d_obs, d_mis, d_cam = _device(obs, mission, cams)
    ref_out = torch.full((n, 142), float("nan"), device="cuda")
    ours = torch.full((n, 142), float("nan"), device="cuda")
    ref = oracle.ref_cuda_features()
    assert ref.tb_cuda_extract_features_device(d_obs.data_ptr(), d_mis.data_ptr(), d_cam.data_ptr(),
                                               ref_out.data_ptr(), n, None) == 1
    assert ref.tb_cuda_synchronize(None) == 1
    assert tb.tb_cuda_extract_features_device(d_obs, d_mis, d_cam, ours, n, None) == 1
    assert tb.tb_cuda_synchronize(None) == 1
    check_features(ref_out.cpu().numpy(), expected, f"reference GPU kernel, seed {seed}")
    check_features(ours.cpu().numpy(), expected, f"this library, seed {seed}")


def test_timed_against_the_reference_kernel():
    n = 65536
    obs, mission, cams, _ = tb.generate(2, 0, n)
    d_obs, d_mis, d_cam = _device(obs, mission, cams)
    out = torch.empty((n, 142), device="cuda")
    ref = oracle.ref_cuda_features()
    ptrs = (d_obs.data_ptr(), d_mis.data_ptr(), d_cam.data_ptr(), out.data_ptr())

    def timed(fn, iters=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(iters):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
        return float(np.median(times))

    mine = timed(lambda: tb.tb_cuda_extract_features_device(d_obs, d_mis, d_cam, out, n, None))
    theirs = timed(lambda: ref.tb_cuda_extract_features_device(*ptrs, n, None))
    gb = n * tb.BYTES_PER_SAMPLE / 1e9
    print(f"\nfeatures, 65,536 aircraft (median of 20): this library {mine:.3f} ms ({gb / mine * 1e3:.0f} GB/s), "
          f"reference kernel for sm_100a {theirs:.3f} ms ({gb / theirs * 1e3:.0f} GB/s), {theirs / mine:.1f}x")
    assert ref.tb_cuda_synchronize(None) == 1 and tb.tb_cuda_synchronize(None) == 1
    assert mine < theirs

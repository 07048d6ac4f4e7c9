"""The allocation-free entry point, iec_realesrgan_run_device_noalloc.

Some callers cannot allocate device memory while they run (a process that
gives all device memory to its own pool allocator at start-up, or a
real-time frame pipeline that cannot absorb the device-wide synchronisation
of cudaMalloc and cudaFree). For them the library keeps Real-ESRGAN's
feature maps in a fixed scratch array of its own instead of growing buffers.
This test calls that entry point through the C ABI, twice in a row, and
checks each result against the ordinary device entry point
(iec_realesrgan_run_device) within the parity tolerance of the other GPU
tests. The second call is smaller than the first and narrower than a TMA
box, so it also checks that values the first call left in the shared
scratch do not leak into it. The file name makes pytest collect it last.
"""

import ctypes

import numpy as np
import pytest

from iec import weights as W

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_PSNR = 45.0


def psnr(a, b):
    mse = np.mean((np.clip(a, 0, 1).astype(np.float64) - np.clip(b, 0, 1)) ** 2)
    return float("inf") if mse == 0 else 10 * np.log10(1.0 / mse)


def test_no_alloc_entry_point_matches_run_device(realesrgan_weights):
    import torch

    import iec

    L = iec.lib()
    fn = L.iec_realesrgan_run_device_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                   ctypes.c_void_p, ctypes.c_void_p]
    model = iec.RealEsrgan(realesrgan_weights)
    stream = torch.cuda.current_stream().cuda_stream
    try:
        for count, width, height, seed in [(1, 384, 256, 21), (3, 7, 12, 22)]:
            images = np.stack([W.realesrgan_input(width, height, seed + i) for i in range(count)])
            d_in = torch.from_numpy(images).cuda()
            want = torch.empty((count, 4 * height, 4 * width, 3), dtype=torch.float32, device="cuda")
            got = torch.full_like(want, float("nan"))
            model.run_device(d_in.data_ptr(), count, width, height, want.data_ptr(), stream)
            status = fn(model._h, d_in.data_ptr(), count, width, height, got.data_ptr(), stream)
            assert status == iec.OK, L.iec_last_error()
            torch.cuda.synchronize()
            g, w = got.cpu().numpy(), want.cpu().numpy()
            assert np.isfinite(g).all()
            assert np.abs(g - w).max() <= MAX_ABS
            assert psnr(g, w) >= MIN_PSNR
        # Beyond the fixed scratch: a clear input error, and nothing runs.
        status = fn(model._h, d_in.data_ptr(), 2, 384, 256, got.data_ptr(), stream)
        assert status == iec.ERR_INPUT
        assert b"scratch" in L.iec_last_error()
    finally:
        model.close()

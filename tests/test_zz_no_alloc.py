"""The allocation-free entry point, iec_realesrgan_run_device_noalloc.

Some callers cannot allocate device memory while they run (a process that
gives all device memory to its own pool allocator at start-up, or a
real-time frame pipeline that cannot absorb the device-wide synchronisation
of cudaMalloc and cudaFree). For them the library keeps Real-ESRGAN's
feature maps in a fixed scratch array of its own instead of growing buffers.
This test calls that entry point through the C ABI and checks its results
bit for bit against the ordinary device entry point
(iec_realesrgan_run_device): both run the same convolution arithmetic, so
any difference would be a stale value leaking out of the shared scratch.
It then makes two calls in a row with every buffer already allocated and
checks that the device's free memory did not move: the call allocates
nothing. The second shape is smaller than the first and narrower than a TMA
box, so values the first call left in the shared scratch would show up in
it. The file name makes pytest collect it last.
"""

import ctypes

import numpy as np
import pytest

from iec import weights as W

pytestmark = pytest.mark.gpu


def test_no_alloc_entry_point_matches_run_device(realesrgan_weights):
    import torch

    import iec

    L = iec.lib()
    fn = L.iec_realesrgan_run_device_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                   ctypes.c_void_p, ctypes.c_void_p]
    model = iec.RealEsrgan(realesrgan_weights)
    stream = torch.cuda.current_stream().cuda_stream
    shapes = [(1, 384, 256, 21), (3, 7, 12, 22)]
    try:
        cases = []
        for count, width, height, seed in shapes:
            images = np.stack([W.realesrgan_input(width, height, seed + i) for i in range(count)])
            d_in = torch.from_numpy(images).cuda()
            want = torch.empty((count, 4 * height, 4 * width, 3), dtype=torch.float32, device="cuda")
            model.run_device(d_in.data_ptr(), count, width, height, want.data_ptr(), stream)
            got = torch.empty_like(want)
            cases.append((count, width, height, d_in, want, got))
        # One warm call per shape, with every torch operation this test
        # uses around it: the first call on a device looks up the scratch
        # array's address, and the first use of a kernel loads its code.
        for count, width, height, d_in, _, got in cases:
            got.fill_(float("nan"))
            assert fn(model._h, d_in.data_ptr(), count, width, height, got.data_ptr(), stream) == iec.OK
            torch.cuda.synchronize()
            got.cpu()
        for case in cases:
            case[5].fill_(float("nan"))
        torch.cuda.synchronize()
        # The two calls in a row, and nothing else, between the two readings
        # of the device's free memory.
        free_before = torch.cuda.mem_get_info()[0]
        for count, width, height, d_in, _, got in cases:
            status = fn(model._h, d_in.data_ptr(), count, width, height, got.data_ptr(), stream)
            assert status == iec.OK, L.iec_last_error()
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info()[0]
        for count, width, height, d_in, want, got in cases:
            g, w = got.cpu().numpy(), want.cpu().numpy()
            assert np.isfinite(g).all()
            assert np.array_equal(g, w), float(np.abs(g - w).max())
        assert free_after == free_before, (free_before - free_after, "bytes of device memory taken")
        # Beyond the fixed scratch: a clear input error, and nothing runs.
        d_in, got = cases[0][3], cases[0][5]
        status = fn(model._h, d_in.data_ptr(), 2, 384, 256, got.data_ptr(), stream)
        assert status == iec.ERR_INPUT
        assert b"scratch" in L.iec_last_error()
        # A size whose pixel count would wrap around size_t is refused too.
        status = fn(model._h, d_in.data_ptr(), 1 << 40, 1 << 20, 1 << 20, got.data_ptr(), stream)
        assert status == iec.ERR_INPUT
    finally:
        model.close()

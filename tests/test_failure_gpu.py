"""Failure detection on the GPU without a fault (GPU tests).

A kernel waits on something nothing provides: an mbarrier no thread arrives
on, or the shared word through which the fused Real-ESRGAN body's tracker
releases items to its producer. Every device wait in the library is bounded:
after about 2 s the wait gives up, sets the device error word and returns,
the kernel exits, and the host call reports IEC_ERR_TIMEOUT. No trap, no
fault, no hang; the context stays usable for the next call.
"""

import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("which", [0, 1])
def test_bounded_wait_expires_with_a_timeout_status(which):
    import iec

    t0 = time.monotonic()
    status = iec.selftest_wait_timeout(which)
    took = time.monotonic() - t0
    assert status == iec.ERR_TIMEOUT, iec.lib().iec_last_error()
    assert 1.5 < took < 60.0
    # The CUDA context is still usable: a Fourier transform round trip.
    x = np.linspace(0.0, 1.0, 8 * 8 * 8, dtype=np.float32).reshape(8, 8, 8)
    _, back = iec.selftest_rfft2(x)
    assert np.abs(back - x).max() <= 1e-2


def test_wait_self_test_rejects_bad_arguments():
    import iec

    assert iec.selftest_wait_timeout(7) == iec.ERR_INPUT

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "image-engine-native_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def workdir(tmp_path_factory):
    return tmp_path_factory.mktemp("iec")


@pytest.fixture(scope="session")
def realesrgan_weights(workdir):
    """Seed-0 random-init Real-ESRGAN weights, as the golden fixtures use."""
    from iec import weights as W

    path = str(workdir / "realesrgan.weights")
    W.write_realesrgan(path, 0)
    return path

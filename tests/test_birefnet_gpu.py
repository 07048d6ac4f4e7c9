"""BiRefNet-lite on the CUDA backend against the CPU oracle and the float64
torch fixture (GPU tests).

Tolerance (the project's parity bar for masks): the sigmoid of the logits
within 1/255 of the reference's, max abs over every pixel. The oracle's
faithful mode reproduces the reference's CPU path, whose f16-rounded Winograd
weights move its own logits by up to about 1e-2 from exact arithmetic
(tests/test_oracle_birefnet.py); the tests against the float64 fixture bound
the backend's distance from exact arithmetic the same way.
"""

import os

import numpy as np
import pytest

from iec import weights as W

pytestmark = pytest.mark.gpu

MASK_TOL = 1.0 / 255.0
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "birefnet_torch.npz")


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x.astype(np.float64)))


def within(got, want, tol=MASK_TOL):
    assert got.shape == want.shape
    assert np.isfinite(got).all()
    err = float(np.abs(sigmoid(got) - sigmoid(want)).max())
    assert err <= tol, (err, float(np.abs(got - want).max()))
    return err


@pytest.fixture(scope="module")
def birefnet_weights(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("birefnet") / "birefnet.weights")
    W.write_birefnet(path, 0)
    return path


@pytest.fixture(scope="module")
def gpu_model(birefnet_weights):
    import iec

    m = iec.Birefnet(birefnet_weights)
    yield m
    m.close()


@pytest.fixture(scope="module")
def cpu_model(birefnet_weights):
    from oracle import refcpu

    return refcpu.Birefnet(birefnet_weights)


def test_matches_torch_fixture(gpu_model):
    g = np.load(GOLDEN)
    for i in range(2):
        within(gpu_model.run(g[f"case{i}_rgb"]), g[f"case{i}_logits"])


@pytest.mark.parametrize("side,seed", [(64, 3), (128, 4), (256, 5)])
def test_matches_oracle(gpu_model, cpu_model, side, seed):
    rgb = W.birefnet_input(side, seed)
    within(gpu_model.run(rgb), cpu_model.run(rgb))


def test_matches_oracle_at_config_size(gpu_model, cpu_model):
    """The benchmark's 1024 x 1024 input."""
    rgb = W.birefnet_input(1024, 0)
    within(gpu_model.run(rgb), cpu_model.run(rgb))


def test_run_normalized_and_repeatable(gpu_model):
    rgb = W.birefnet_input(128, 9)
    a = gpu_model.run(rgb)
    b = gpu_model.run_normalized(W.birefnet_normalize(rgb))
    assert np.abs(a - b).max() < 1e-3
    gpu_model.run(W.birefnet_input(64, 1))  # another size in between
    assert np.array_equal(gpu_model.run(rgb), a)


def test_size_check(gpu_model):
    import iec

    for side in (32, 96):
        with pytest.raises(iec.IecError):
            gpu_model.run(np.zeros((side, side, 3), np.uint8))


def test_run_device(gpu_model, cpu_model):
    import torch

    rgb = W.birefnet_input(128, 11)
    t = torch.from_numpy(rgb).cuda()
    out = torch.empty((128, 128), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    gpu_model.run_device(t.data_ptr(), True, 128, out.data_ptr(), s.cuda_stream)
    s.synchronize()
    within(out.cpu().numpy(), cpu_model.run(rgb))


def test_batch_matches_single_runs(gpu_model):
    """iec_birefnet_run_batch: 8-bit images in host buffers, each image's
    logits as run gives them, bit for bit."""
    images = np.stack([W.birefnet_input(128, s) for s in range(3)])
    singles = np.stack([gpu_model.run(im) for im in images])
    batch = gpu_model.run_batch(images)
    assert np.array_equal(batch.view(np.uint32), singles.view(np.uint32))


def test_fused_mlp_matches_separate_launches(gpu_model):
    """The fused backbone MLPs (widths 96 and 192) against LayerNorm + fc1 +
    fc2 as separate launches: the same f16 roundings, the LayerNorm sums in
    another order; the masks agree far inside the 1/255 bar."""
    rgb = W.birefnet_input(256, 7)
    try:
        fused = gpu_model.run(rgb)
        gpu_model.set_fused(False)
        apart = gpu_model.run(rgb)
    finally:
        gpu_model.set_fused(True)
    assert np.isfinite(fused).all()
    sig = lambda z: 1.0 / (1.0 + np.exp(-z.astype(np.float64)))  # noqa: E731
    err = float(np.abs(sig(fused) - sig(apart)).max())
    print(f"fused vs separate: mask max abs {err:.3g}")
    assert err <= 1.0 / 1020

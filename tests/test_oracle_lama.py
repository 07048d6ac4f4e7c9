"""The CPU oracle's LaMa restatement: its Fourier transforms against the
reference's own test (crates/lama-native/src/fourier.rs:448-484: the sizes,
the input sequence and the 1e-5 bound, restated), the network against the
float64 PyTorch formulation of tests/golden/gen_lama_golden.py run on the
upstream checkpoint whose exported file the oracle reads, and the
public API's checks, progress and compositing (lib.rs:118-194)."""

import os

import numpy as np
import pytest

from iec import weights as W
from oracle import refcpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "lama_torch.npz")


def values(n, seed):
    """fourier.rs:452-456: sin(0.7 i + seed) * 2."""
    return (np.sin(np.arange(n, dtype=np.float64) * 0.7 + seed) * 2.0).astype(np.float32)


@pytest.mark.parametrize("h,w,c", [(4, 6, 3), (5, 7, 2), (16, 12, 2), (9, 10, 2), (1, 8, 1)])
def test_spectrum_matches_definition(h, w, c):
    x = values(h * w * c, 0.3).reshape(h, w, c)
    spec = refcpu.rfft2(x, h, w, c)
    want = np.fft.rfft2(x.astype(np.float64), axes=(0, 1), norm="ortho")
    assert np.abs(spec[:, :, :c] - want.real).max() < 1e-5
    assert np.abs(spec[:, :, c:] - want.imag).max() < 1e-5
    back = refcpu.irfft2_add(spec, h, w, c, np.ones((h, w, c), np.float32))
    assert np.abs(back - 1.0 - x).max() < 1e-5


def test_inverse_reads_only_real_edge_columns():
    """The inverse of a spectrum that is not Hermitian: after the column
    transforms it reads only the real part of column 0 and, for an even
    width, of column w / 2, as numpy's and torch's irfft2 do (fourier.rs:7-9)."""
    h, w, c = 6, 8, 2
    rng = np.random.default_rng(3)
    spec = rng.standard_normal((h, w // 2 + 1, 2 * c)).astype(np.float32)
    got = refcpu.irfft2_add(spec, h, w, c, np.zeros((h, w, c), np.float32))
    z = spec[:, :, :c] + 1j * spec[:, :, c:]
    want = np.fft.irfft2(z.astype(np.complex128), s=(h, w), axes=(0, 1), norm="ortho")
    assert np.abs(got - want).max() < 1e-5


@pytest.fixture(scope="module")
def lama(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("lama") / "lama.weights")
    sha = W.write_lama(path, 0)
    return refcpu.Lama(path), sha


def test_golden_matches_float64_torch(lama):
    model, sha = lama
    g = np.load(GOLDEN)
    assert str(g["weights_sha256"]) == sha, "weights generator changed: regenerate the fixture"
    for i in range(3):
        out = model.run_float(g[f"case{i}_image"], g[f"case{i}_mask"])
        ref = g[f"case{i}_out"]
        assert out.shape == ref.shape
        # f32 weights file: the oracle's f32 arithmetic is the only difference
        assert np.abs(out - ref).max() < 5e-5


def test_check_size(lama):
    model, _ = lama
    image, mask = W.lama_input(9, 9, 0)
    with pytest.raises(refcpu.OracleError):
        model.run_float(image[:8], mask[:8])
    with pytest.raises(refcpu.OracleError):
        model.run_float(image[:, :8], mask[:, :8])


def test_progress_steps_and_cancel(lama):
    model, _ = lama
    image, mask = W.lama_input(16, 16, 0)
    seen = []
    model.run_float(image, mask, progress=lambda f: seen.append(f) and False)
    assert len(seen) == refcpu.Lama.STEPS and seen[-1] == 1.0
    calls = []

    def cancel(f):
        calls.append(f)
        return len(calls) >= 5

    with pytest.raises(refcpu.OracleError) as e:
        model.run_float(image, mask, progress=cancel)
    assert e.value.code == 4 and len(calls) == 5


def test_run_composites_only_holes(lama):
    model, _ = lama
    image, mask = W.lama_input(24, 16, 5)
    rgb = np.round(image * 255).astype(np.uint8)
    m8 = (mask * 255).astype(np.uint8)
    out = model.run(rgb, m8)
    keep = mask == 0
    assert np.array_equal(out[keep], rgb[keep])
    pred = model.run_float(rgb.astype(np.float32) / np.float32(255), mask)
    want = np.floor((np.clip(pred, 0, 1) * np.float32(255)).astype(np.float64) + 0.5)
    assert np.array_equal(out[~keep], want[~keep].astype(np.uint8))

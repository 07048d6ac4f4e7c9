"""The CPU oracle's Real-ESRGAN, pinned to the reference.

The golden fixture holds outputs of the reference's own PyTorch definition
of the network (tools/realesrgan/torch_reference.py:25-43) on the seeded
weights; the bound is the reference's CPU-vs-PyTorch bound
(crates/realesrgan-native/tests/reference.rs:61-80): under 5e-4 and no
8-bit value more than one step away. Progress, cancel and margin behaviour
follow crates/realesrgan-native/tests/reference.rs:85-152.
"""

import os

import numpy as np
import pytest

from iec import weights as W
from oracle import refcpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "realesrgan_torch.npz")


def to_8bit(v):
    return np.round(np.clip(v, 0.0, 1.0) * 255.0).astype(np.int32)


@pytest.fixture(scope="module")
def model(realesrgan_weights):
    return refcpu.RealEsrgan(realesrgan_weights)


def test_seeded_weights_are_the_golden_ones(realesrgan_weights):
    import hashlib

    golden = np.load(GOLDEN)
    with open(realesrgan_weights, "rb") as f:
        assert hashlib.sha256(f.read()).hexdigest() == str(golden["weights_sha256"])


@pytest.mark.parametrize("size", ["20x12", "33x17"])
def test_matches_pytorch_reference(model, size):
    golden = np.load(GOLDEN)
    image, want = golden[f"input_{size}"], golden[f"torch_{size}"]
    got = model.run_float(image)
    assert got.shape == want.shape
    assert np.isfinite(got).all()
    assert np.abs(got - want).max() < 5e-4
    assert np.abs(to_8bit(got) - to_8bit(want)).max() <= 1


def test_direct_mode_agrees(model):
    golden = np.load(GOLDEN)
    image = golden["input_33x17"]
    a = model.run_float(image)
    refcpu.set_direct(True)
    try:
        b = model.run_float(image)
    finally:
        refcpu.set_direct(False)
    assert np.abs(a - b).max() < 5e-4


def reference_image():
    # tests/reference.rs:89-91
    return ((np.arange(128 * 96 * 3) % 251) / 250.0).astype(np.float32).reshape(96, 128, 3)


def test_progress_reaches_one_and_cancel_stops(model):
    image = reference_image()
    seen = []
    whole = model.run_float_tiled(image, 64, 16, lambda f: seen.append(f) or False)
    assert len(seen) == 4 * 34
    assert all(a < b for a, b in zip(seen, seen[1:]))
    assert seen[-1] == 1.0
    other = np.full_like(image, 0.5)
    calls = [0]

    def stop(f):
        calls[0] += 1
        return f >= 0.4

    with pytest.raises(refcpu.OracleError) as e:
        model.run_float_tiled(other, 64, 16, stop)
    assert e.value.code == 4
    assert calls[0] == 55
    again = model.run_float_tiled(image, 64, 16)
    assert np.array_equal(again.view(np.uint32), whole.view(np.uint32))


def test_unbounded_margin_runs_whole_image(model):
    image = reference_image()
    whole = model.run_float(image)
    for margin in [128, 2**63]:
        tiled = model.run_float_tiled(image, 64, margin)
        assert np.array_equal(tiled.view(np.uint32), whole.view(np.uint32))


def test_tiles_with_the_receptive_field_match_within_rounding(model):
    image = W.realesrgan_input(70, 45, 5)
    whole = model.run_float(image)
    tiled = model.run_float_tiled(image, 32, 34)
    assert np.abs(tiled - whole).max() < 1e-4


def test_bad_sizes_are_input_errors(model):
    with pytest.raises(refcpu.OracleError) as e:
        model.run_float_tiled(np.zeros((4, 4, 3), np.float32), 0, 34)
    assert e.value.code == 3

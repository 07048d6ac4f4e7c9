"""The CPU oracle's BiRefNet restatement against the float64 torch formulation
of tests/golden/gen_birefnet_golden.py, its aligned-corner resize against
PyTorch's, and the public API's size check (lib.rs:175-187).

With the direct product (no Winograd) the oracle equals the float64
formulation to f32 rounding; in its faithful mode, which like the reference
uses F(2x2,3x3) Winograd with f16-rounded transformed weights for these f16
files (winograd.rs:107-146), the logits move by up to about 1e-2: that spread
is the CPU path's own noise floor."""

import os

import numpy as np
import pytest

from iec import weights as W
from oracle import refcpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "birefnet_torch.npz")


@pytest.fixture(scope="module")
def birefnet(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("birefnet") / "birefnet.weights")
    sha = W.write_birefnet(path, 0)
    return refcpu.Birefnet(path), sha


def test_golden_direct_and_faithful(birefnet):
    model, sha = birefnet
    g = np.load(GOLDEN)
    assert str(g["weights_sha256"]) == sha, "weights generator changed: regenerate the fixture"
    for i in range(2):
        rgb, ref = g[f"case{i}_rgb"], g[f"case{i}_logits"]
        refcpu.set_direct(True)
        try:
            direct = model.run(rgb)
        finally:
            refcpu.set_direct(False)
        assert np.abs(direct - ref).max() < 5e-5
        faithful = model.run(rgb)
        assert np.abs(faithful - ref).max() < 2e-2


def test_run_normalized_equals_run(birefnet):
    model, _ = birefnet
    rgb = W.birefnet_input(64, 7)
    assert np.array_equal(model.run(rgb), model.run_normalized(W.birefnet_normalize(rgb)))


@pytest.mark.parametrize("sh,sw,dh,dw", [(4, 4, 9, 9), (16, 16, 2, 2), (7, 5, 3, 11), (8, 8, 1, 1), (1, 1, 4, 4)])
def test_resize_matches_align_corners(sh, sw, dh, dw):
    import torch
    import torch.nn.functional as F

    rng = np.random.default_rng(sh * 100 + dh)
    src = rng.standard_normal((sh, sw, 3)).astype(np.float32)
    got = refcpu.resize(src, dh, dw)
    want = F.interpolate(torch.from_numpy(src.astype(np.float64)).permute(2, 0, 1)[None], size=(dh, dw),
                         mode="bilinear", align_corners=True)[0].permute(1, 2, 0).numpy()
    assert np.abs(got - want).max() < 1e-5
    added = refcpu.resize(src, dh, dw, out=np.ones((dh, dw, 3), np.float32), add=True)
    assert np.abs(added - 1.0 - got).max() < 1e-6


def test_check_size(birefnet):
    model, _ = birefnet
    for side in (32, 96):
        with pytest.raises(refcpu.OracleError):
            model.run(np.zeros((side, side, 3), np.uint8))

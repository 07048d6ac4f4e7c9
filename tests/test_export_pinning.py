"""The weights files against the reference's own exporters (CPU tests).

tests/golden/gen_export_fixtures.py ran the reference's
tools/{realesrgan,scunet,lama}/export_weights.py on seeded checkpoints in
the upstream PyTorch layouts (iec.weights.*_checkpoint) and recorded the
SHA-256 of each file they wrote, in tests/golden/export_sha256.json. These
tests check that iec.weights' restatement of each exporter still writes
those exact bytes (convolution, transposed-convolution and linear layouts,
batch-norm folding, LaMa's planar real|imaginary order and phase split,
SCUNet's position-bias gather, Real-ESRGAN's denoise-strength blend, f16
storage rules, tensor names and order), and that the seeded files every
other test and the benchmark load are exactly those files.
"""

import hashlib
import json
import os

import pytest

from iec import weights as W

FIXTURE = os.path.join(os.path.dirname(__file__), "golden", "export_sha256.json")
RECORD = json.load(open(FIXTURE))


def sha(data: bytes) -> str:
    return hashlib.sha256(data).hexdigest()


def restated(case) -> bytes:
    model, seed, half = case["model"], case["seed"], "--half" in case["flags"]
    if model == "realesrgan":
        weak = W.realesrgan_checkpoint(case["weak_seed"]) if case["weak_seed"] is not None else None
        tensors = W.export_realesrgan(W.realesrgan_checkpoint(seed), weak, case["strength"], half)
    elif model == "scunet":
        tensors = W.export_scunet(W.scunet_checkpoint(seed), half)
    else:
        tensors = W.export_lama(W.lama_checkpoint(seed), half)
    return W.encode(W.MAGIC[model], tensors)


@pytest.mark.parametrize("name", sorted(RECORD))
def test_restated_exporter_writes_the_reference_exporters_bytes(name):
    case = RECORD[name]
    data = restated(case)
    assert len(data) == case["bytes"]
    assert sha(data) == case["sha256"], f"{name}: the export mapping changed"


@pytest.mark.parametrize("model,case", [("realesrgan", "realesrgan"), ("scunet", "scunet_half"), ("lama", "lama")])
def test_seeded_files_are_the_reference_exporters_files(tmp_path, model, case):
    writer = getattr(W, f"write_{model}")
    assert writer(str(tmp_path / f"{model}.weights"), 0) == RECORD[case]["sha256"]


def test_blend_is_the_strong_file_at_strength_one():
    strong = W.realesrgan_checkpoint(0)
    weak = W.realesrgan_checkpoint(1)
    a = W.encode(W.MAGIC["realesrgan"], W.export_realesrgan(strong, weak, 1.0))
    assert sha(a) == RECORD["realesrgan"]["sha256"]
    with pytest.raises(ValueError):
        W.export_realesrgan(strong, {k: v for k, v in list(weak.items())[:-1]}, 0.5)


def test_position_bias_is_the_relative_gather():
    import numpy as np

    params = np.arange(2 * 15 * 15, dtype=np.float32).reshape(2, 15, 15)
    bias = W.scunet_position_bias(params)
    assert bias.shape == (2, 64, 64)
    # tokens (y1, x1) = (1, 2) and (y2, x2) = (5, 0): params[:, -4 + 7, 2 + 7]
    assert np.array_equal(bias[:, 1 * 8 + 2, 5 * 8 + 0], params[:, 3, 9])
    assert np.array_equal(np.diagonal(bias, axis1=1, axis2=2), np.repeat(params[:, 7, 7][:, None], 64, 1))

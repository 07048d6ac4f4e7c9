"""The CPU oracle's Swin pieces and SCUNet restatement against the
reference's own unit tests (crates/native-engine/src/attention.rs:215-254,
math.rs:172-278, restated with their inputs and tolerances) and its tiling
behaviour (crates/scunet-native/src/lib.rs:164-247)."""

import math

import numpy as np
import pytest

from iec import weights as W
from oracle import refcpu


@pytest.mark.parametrize("n", [49, 64])
def test_attention_matches_definition(n):
    d, c, head = 32, 96, 1
    qkv = np.sin(np.arange(n * 3 * c, dtype=np.float32) * np.float32(0.618)).astype(np.float32).reshape(n, 3 * c)
    i = np.arange(n * n, dtype=np.float32)
    bias = (np.cos(i * np.float32(0.31)) - 100.0 * (np.arange(n * n) % 17 == 0)).astype(np.float32).reshape(n, n)
    out = refcpu.attention(qkv, c, head, bias, n)
    q = qkv[:, head * d:(head + 1) * d].astype(np.float64)
    k = qkv[:, c + head * d:c + (head + 1) * d].astype(np.float64)
    v = qkv[:, 2 * c + head * d:2 * c + (head + 1) * d].astype(np.float64)
    s = q @ k.T / math.sqrt(d) + bias.astype(np.float64)
    p = np.exp(s - s.max(1, keepdims=True))
    want = (p / p.sum(1, keepdims=True)) @ v
    assert np.abs(out[:, head * d:(head + 1) * d] - want).max() < 1e-5


def test_gelu_matches_erf_definition():
    x = (np.arange(-800, 801) / 100.0).astype(np.float32)
    z = np.clip(x.astype(np.float64) / math.sqrt(2), -4, 4)
    want = 0.5 * x.astype(np.float64) * (1 + np.array([math.erf(v) if abs(v) < 4 else math.copysign(1, v) for v in z]))
    got = refcpu.gelu(x)
    assert np.all(np.abs(got - want) < 2e-6 * (1 + np.abs(want)))


def test_sigmoid_matches_libm_and_saturates():
    x = (np.arange(-2000, 2001) / 20.0).astype(np.float32)
    want = (1 / (1 + np.exp(-x.astype(np.float64)))).astype(np.float32)
    assert np.abs(refcpu.sigmoid(x) - want).max() <= 2 * np.finfo(np.float32).eps
    assert list(refcpu.sigmoid(np.array([-1e30, 1e30, 0.0], np.float32))) == [0.0, 1.0, 0.5]


def test_layer_norm_matches_definition():
    c = 37
    x = (np.cos(np.arange(3 * c, dtype=np.float32) * np.float32(1.3)) * 4 + 2).astype(np.float32).reshape(3, c)
    gamma = (1 + np.arange(c) / 50.0).astype(np.float32)
    beta = (np.arange(c) / 10.0).astype(np.float32)
    got = refcpu.layer_norm(x, gamma, beta)
    xd = x.astype(np.float64)
    mean = xd.mean(1, keepdims=True)
    var = ((xd - mean) ** 2).mean(1, keepdims=True)
    want = (xd - mean) / np.sqrt(var + 1e-5) * gamma + beta
    assert np.abs(got - want).max() < 1e-5


@pytest.fixture(scope="module")
def scunet(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("scunet") / "scunet.weights")
    W.write_scunet(path, 0)
    return refcpu.Scunet(path)


def test_scunet_tiles_progress_and_unbounded_margin(scunet):
    image = W.scunet_input(90, 70, 3)
    whole = scunet.run_float(image)
    assert np.isfinite(whole).all() and np.abs(whole).max() < 10
    seen = []
    tiled = scunet.run_float_tiled(image, 48, 2**63, lambda f: seen.append(f) or False)
    assert len(seen) == 2 * 2 * 28 and seen[-1] == 1.0
    assert np.array_equal(tiled.view(np.uint32), whole.view(np.uint32))


def test_scunet_weights_file_is_checked(tmp_path):
    tensors = W.scunet_tensors(0)
    path = str(tmp_path / "bad.weights")
    W.write(path, W.MAGIC["scunet"], tensors[:-1])
    with pytest.raises(refcpu.OracleError) as e:
        refcpu.Scunet(path)
    assert e.value.code == 2

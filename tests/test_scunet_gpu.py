"""SCUNet on the CUDA backend against the CPU oracle (GPU tests), and its
fused window attention alone.

Tolerance (the project's parity bar for RGB outputs): max abs <= 2e-2 on raw
outputs and PSNR >= 45 dB on outputs clamped to [0, 1]. The behaviour tests
follow crates/scunet-native/tests (progress 28 times per tile, cancel, an
unbounded margin giving the whole image's result).
"""

import numpy as np
import pytest

from iec import weights as W

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_PSNR = 45.0


def psnr(a, b):
    mse = np.mean((np.clip(a, 0, 1).astype(np.float64) - np.clip(b, 0, 1)) ** 2)
    return float("inf") if mse == 0 else 10 * np.log10(1.0 / mse)


def within(got, want, max_abs=MAX_ABS):
    assert got.shape == want.shape
    assert np.isfinite(got).all()
    err = float(np.abs(got - want).max())
    p = psnr(got, want)
    assert err <= max_abs and p >= MIN_PSNR, (err, p)
    return err, p


@pytest.fixture(scope="module")
def scunet_weights(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("scunet") / "scunet.weights")
    W.write_scunet(path, 0)
    return path


@pytest.fixture(scope="module")
def gpu_model(scunet_weights):
    import iec

    m = iec.Scunet(scunet_weights)
    yield m
    m.close()


@pytest.fixture(scope="module")
def cpu_model(scunet_weights):
    from oracle import refcpu

    return refcpu.Scunet(scunet_weights)


def bias_tables(position, shifted):
    """swin.rs:26-50."""
    if not shifted:
        return position
    heads = position.shape[0]
    ids = lambda last_row, last_col: np.array(  # noqa: E731
        [(int(last_row and i // 8 >= 4)) * 2 + int(last_col and i % 8 >= 4) for i in range(64)])
    out = []
    for cls in range(4):
        id_ = ids(bool(cls & 2), bool(cls & 1))
        mask = np.where(id_[:, None] == id_[None, :], 0.0, -np.inf).astype(np.float32)
        out.append(position + mask[None])
    return np.stack(out).reshape(4, heads, 64, 64)


@pytest.mark.parametrize("c,rows_w,cols_w,shifted", [(32, 2, 3, False), (64, 3, 2, True), (128, 2, 2, True)])
def test_window_attention_matches_oracle(c, rows_w, cols_w, shifted):
    import iec
    from oracle import refcpu

    rng = np.random.default_rng(c + rows_w)
    windows = rows_w * cols_w
    qkv = rng.standard_normal((windows * 64, 3 * c)).astype(np.float16).astype(np.float32)
    position = (0.5 * rng.standard_normal((c // 32, 64, 64))).astype(np.float32)
    tables = bias_tables(position, shifted).astype(np.float32)
    got = iec.selftest_attention(qkv, windows, c, tables, shifted, rows_w, cols_w)
    want = np.zeros_like(got)
    for w in range(windows):
        cls = 0
        if shifted:
            cls = int(w % cols_w == cols_w - 1) + 2 * int(w // cols_w == rows_w - 1)
        for h in range(c // 32):
            want[w * 64:(w + 1) * 64] += refcpu.attention(qkv[w * 64:(w + 1) * 64], c, h, tables.reshape(-1, c // 32, 64, 64)[cls, h], 64)
    assert np.abs(got - want).max() < 5e-3


@pytest.mark.parametrize("w,h,seed", [(64, 64, 1), (100, 70, 2), (192, 128, 3)])
def test_matches_oracle(gpu_model, cpu_model, w, h, seed):
    image = W.scunet_input(w, h, seed)
    err, p = within(gpu_model.run_float(image), cpu_model.run_float(image))
    print(f"scunet {w}x{h}: max abs {err:.3g}, PSNR {p:.1f} dB")


def test_full_config_matches_oracle(gpu_model, cpu_model):
    # The benchmark configuration: 3 x 512 x 768.
    image = W.scunet_input(768, 512, 0)
    err, p = within(gpu_model.run_float(image), cpu_model.run_float(image))
    print(f"scunet 768x512: max abs {err:.3g}, PSNR {p:.1f} dB")


def test_tiles_progress_and_cancel(gpu_model):
    import iec

    image = W.scunet_input(150, 90, 4)
    seen = []
    tiled = gpu_model.run_float_tiled(image, 80, 32, lambda f: seen.append(f) or False)
    assert len(seen) == 2 * 2 * 28
    assert all(a < b for a, b in zip(seen, seen[1:])) and seen[-1] == 1.0
    calls = [0]

    def stop(f):
        calls[0] += 1
        return f >= 0.5

    with pytest.raises(iec.Cancelled):
        gpu_model.run_float_tiled(image, 80, 32, stop)
    assert calls[0] == 56
    again = gpu_model.run_float_tiled(image, 80, 32)
    assert np.array_equal(again.view(np.uint32), tiled.view(np.uint32))


def test_unbounded_margin_is_the_whole_image(gpu_model):
    image = W.scunet_input(100, 70, 5)
    whole = gpu_model.run_float(image)
    tiled = gpu_model.run_float_tiled(image, 64, 2**64 - 1)
    assert np.array_equal(tiled.view(np.uint32), whole.view(np.uint32))


def test_8bit_run(gpu_model, cpu_model):
    rng = np.random.default_rng(6)
    rgb = rng.integers(0, 256, (70, 90, 3), dtype=np.uint8)
    got = gpu_model.run(rgb)
    want = cpu_model.run_float(rgb.astype(np.float32) / np.float32(255.0))
    want8 = np.round(np.clip(want, 0, 1) * 255).astype(np.int32)
    assert np.abs(got.astype(np.int32) - want8).max() <= 6
    assert psnr(got / 255.0, want8 / 255.0) > 45.0


def test_batch_matches_single_runs(gpu_model):
    """iec_scunet_run_batch: host buffers, copies overlapped with the
    kernels, two alternating device buffer pairs; each image as run_float
    gives it, bit for bit."""
    images = np.stack([W.scunet_input(40, 24, s) for s in range(5)])
    singles = np.stack([gpu_model.run_float(im) for im in images])
    batch = gpu_model.run_batch(images)
    assert np.array_equal(batch.view(np.uint32), singles.view(np.uint32))


@pytest.mark.parametrize("w,h,seed", [(768, 512, 0), (100, 70, 8)])
def test_fused_mlp_matches_separate_launches(gpu_model, w, h, seed):
    """The fused transformer MLP (LayerNorm in shared memory, fc1, GELU and
    fc2 in one kernel) against LayerNorm + fc1 + fc2 as separate launches.
    Both round the normalised rows, the hidden layer and the sums to f16 at
    the same points; only the LayerNorm sums run in another order, which can
    move an f16 rounding by one step."""
    image = W.scunet_input(w, h, seed)
    try:
        fused = gpu_model.run_float(image)
        gpu_model.set_fused(False)
        apart = gpu_model.run_float(image)
    finally:
        gpu_model.set_fused(True)
    assert np.isfinite(fused).all()
    err = float(np.abs(fused - apart).max())
    p = psnr(fused, apart)
    print(f"{w}x{h}: fused vs separate max abs {err:.3g}, PSNR {p:.1f} dB")
    assert err <= 1e-2 and p >= 60.0, (err, p)

"""Real-ESRGAN on the CUDA backend against the CPU oracle (GPU tests).

Tolerance (the project's parity bar for RGB outputs): max abs <= 2e-2 on raw
outputs and PSNR >= 45 dB on outputs clamped to [0, 1]. The behaviour tests
follow crates/realesrgan-native/tests/gpu.rs:49-72 (tiles of 64 with MARGIN
are bit for bit the whole image) and tests/reference.rs:85-152 (progress,
cancel, unbounded margin).
"""

import os

import numpy as np
import pytest

from iec import weights as W

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "realesrgan_torch.npz")
MAX_ABS = 2e-2
MIN_PSNR = 45.0


def psnr(a, b):
    a = np.clip(a.astype(np.float64), 0, 1)
    b = np.clip(b.astype(np.float64), 0, 1)
    mse = np.mean((a - b) ** 2)
    return float("inf") if mse == 0 else 10 * np.log10(1.0 / mse)


def within(got, want):
    assert got.shape == want.shape
    assert np.isfinite(got).all()
    err = np.abs(got - want).max()
    p = psnr(got, want)
    assert err <= MAX_ABS and p >= MIN_PSNR, (err, p)
    return err, p


@pytest.fixture(scope="module")
def gpu_model(realesrgan_weights):
    import iec

    m = iec.RealEsrgan(realesrgan_weights)
    yield m
    m.close()


@pytest.fixture(scope="module")
def cpu_model(realesrgan_weights):
    from oracle import refcpu

    return refcpu.RealEsrgan(realesrgan_weights)


def test_device_is_a_b200(gpu_model):
    assert "B200" in gpu_model.gpu()


@pytest.mark.parametrize("size", ["20x12", "33x17"])
def test_matches_reference_pytorch_network(gpu_model, size):
    golden = np.load(GOLDEN)
    within(gpu_model.run_float(golden[f"input_{size}"]), golden[f"torch_{size}"])


@pytest.mark.parametrize("w,h,seed", [(8, 16, 3), (1, 1, 4), (5, 40, 5), (130, 70, 6), (67, 129, 7)])
def test_matches_oracle(gpu_model, cpu_model, w, h, seed):
    image = W.realesrgan_input(w, h, seed)
    within(gpu_model.run_float(image), cpu_model.run_float(image))


def test_full_config_matches_oracle(gpu_model, cpu_model):
    # The single-image benchmark configuration: 3 x 256 x 384.
    image = W.realesrgan_input(384, 256, 0)
    err, p = within(gpu_model.run_float(image), cpu_model.run_float(image))
    print(f"384x256: max abs {err:.3g}, PSNR {p:.1f} dB")


def test_tiles_are_bit_identical_to_the_whole_image(gpu_model):
    # tests/gpu.rs:59-72: 64-pixel tiles with MARGIN give the whole image
    # bit for bit.
    image = W.realesrgan_input(150, 97, 8)
    whole = gpu_model.run_float(image)
    tiled = gpu_model.run_float_tiled(image, 64, gpu_model.MARGIN)
    assert np.array_equal(tiled.view(np.uint32), whole.view(np.uint32))


def test_unbounded_margin_runs_whole_image(gpu_model):
    image = ((np.arange(128 * 96 * 3) % 251) / 250.0).astype(np.float32).reshape(96, 128, 3)
    whole = gpu_model.run_float(image)
    for margin in [128, 2**64 - 1]:
        tiled = gpu_model.run_float_tiled(image, 64, margin)
        assert np.array_equal(tiled.view(np.uint32), whole.view(np.uint32))


def test_progress_reaches_one_and_cancel_stops(gpu_model):
    import iec

    image = ((np.arange(128 * 96 * 3) % 251) / 250.0).astype(np.float32).reshape(96, 128, 3)
    seen = []
    whole = gpu_model.run_float_tiled(image, 64, 16, lambda f: seen.append(f) or False)
    assert len(seen) == 4 * 34
    assert all(a < b for a, b in zip(seen, seen[1:]))
    assert seen[-1] == 1.0
    calls = [0]

    def stop(f):
        calls[0] += 1
        return f >= 0.4

    with pytest.raises(iec.Cancelled):
        gpu_model.run_float_tiled(np.full_like(image, 0.5), 64, 16, stop)
    assert calls[0] == 55
    again = gpu_model.run_float_tiled(image, 64, 16)
    assert np.array_equal(again.view(np.uint32), whole.view(np.uint32))


def test_8bit_run_matches_oracle(gpu_model, cpu_model):
    rng = np.random.default_rng(11)
    rgb = rng.integers(0, 256, (45, 61, 3), dtype=np.uint8)
    got = gpu_model.run(rgb)
    want = cpu_model.run_float(rgb.astype(np.float32) / np.float32(255.0))
    want8 = np.round(np.clip(want, 0, 1) * 255).astype(np.int32)
    diff = np.abs(got.astype(np.int32) - want8)
    # tests/gpu.rs:49-58: half floats move a share of 8-bit values by a step
    # or a few; the 8-bit PSNR against the CPU engine stays above 48 dB. The
    # raw tolerance (2e-2) allows at most 6 steps.
    assert diff.max() <= 6
    assert psnr(got / 255.0, want8 / 255.0) > 48.0


def test_batch_and_device_paths_match_single_runs(gpu_model):
    import torch

    images = np.stack([W.realesrgan_input(40, 24, s) for s in range(5)])
    singles = np.stack([gpu_model.run_float(im) for im in images])
    batch = gpu_model.run_batch(images)
    assert np.array_equal(batch.view(np.uint32), singles.view(np.uint32))
    d_in = torch.from_numpy(images).cuda()
    d_out = torch.empty((5, 96, 160, 3), dtype=torch.float32, device="cuda")
    gpu_model.run_device(d_in.data_ptr(), 5, 40, 24, d_out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(d_out.cpu().numpy().view(np.uint32), singles.view(np.uint32))


def test_8bit_batch_matches_8bit_single_runs(gpu_model):
    # iec_realesrgan_run_batch_u8: Model::run's byte semantics over a batch
    # of whole images, equal to the tiled single-image run byte for byte.
    rng = np.random.default_rng(17)
    images = rng.integers(0, 256, (9, 20, 36, 3), dtype=np.uint8)
    singles = np.stack([gpu_model.run(im) for im in images])
    batch = gpu_model.run_batch_u8(images)
    assert batch.dtype == np.uint8 and batch.shape == (9, 80, 144, 3)
    assert np.array_equal(batch, singles)


def test_runs_are_deterministic(gpu_model):
    image = W.realesrgan_input(100, 60, 12)
    a = gpu_model.run_float(image)
    b = gpu_model.run_float(image)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_bad_inputs_are_input_errors(gpu_model):
    import iec

    with pytest.raises(iec.IecError) as e:
        gpu_model.run_float_tiled(np.zeros((4, 4, 3), np.float32), 0, 34)
    assert e.value.code == iec.ERR_INPUT
    with pytest.raises(iec.IecError) as e:
        gpu_model.run_float(np.zeros((0, 4, 3), np.float32))
    assert e.value.code == iec.ERR_INPUT
    # The model stays usable.
    gpu_model.run_float(np.zeros((4, 4, 3), np.float32))


def test_weight_file_errors(workdir):
    import iec

    tensors = W.realesrgan_tensors(0)
    bad = str(workdir / "missing.weights")
    W.write(bad, W.MAGIC["realesrgan"], tensors[:-1])
    with pytest.raises(iec.IecError) as e:
        iec.RealEsrgan(bad)
    assert e.value.code == iec.ERR_WEIGHTS
    wrong = str(workdir / "wrong.weights")
    W.write(wrong, W.MAGIC["lama"], tensors)
    with pytest.raises(iec.IecError) as e:
        iec.RealEsrgan(wrong)
    assert e.value.code == iec.ERR_WEIGHTS
    with pytest.raises(iec.IecError) as e:
        iec.RealEsrgan(str(workdir / "does-not-exist.weights"))
    assert e.value.code == iec.ERR_IO


def test_tile_ranges_stitch_to_the_tiled_run(gpu_model):
    # The sharded large-image path: each rank runs a contiguous range of
    # tiles; the ranges here run one after another on one GPU.
    from iec import shard

    image = W.realesrgan_input(200, 130, 13)
    tiles = shard.tile_grid(200, 130, 64, 34)
    want = gpu_model.run_float_tiled(image, 64, 34)
    out = np.full((520, 800, 3), np.nan, np.float32)
    for first, last in shard.split_ranges([t.cost for t in tiles], 3):
        gpu_model.run_float_tiles(image, 64, 34, first, last, out)
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("w,h,count", [(384, 256, 1), (40, 24, 5), (131, 67, 3), (16, 10, 40)])
def test_fused_body_matches_per_layer_launches(gpu_model, w, h, count):
    # The persistent 32-layer body launch computes every tile as the
    # per-layer kernel does: outputs bit for bit, including partial image
    # groups (3 images = groups of 2 + 1) and tiny maps.
    images = np.stack([W.realesrgan_input(w, h, 20 + s) for s in range(count)])
    fused = gpu_model.run_batch(images)
    gpu_model.set_fused(False)
    try:
        layered = gpu_model.run_batch(images)
    finally:
        gpu_model.set_fused(True)
    assert np.array_equal(fused.view(np.uint32), layered.view(np.uint32))


def test_fused_body_is_the_path_taken(gpu_model):
    # One 384 x 256 image: prep, the first layer, the fused body, the last
    # layer; the timing record shows the fused launch (kind 4) and no
    # per-layer 64 -> 64 launch.
    assert gpu_model.launches(1, 384, 256) == 4
    image = W.realesrgan_input(384, 256, 1)
    gpu_model.set_timing(16)
    try:
        gpu_model.run_batch(image[None])
        kinds, ms = gpu_model.timing(16)
    finally:
        gpu_model.set_timing(0)
    assert list(kinds) == [0, 1, 4, 3]
    assert (ms > 0).all()


def test_progress_runs_use_fused_stages_with_the_same_output(gpu_model):
    # With a progress callback the body runs as fused launches of 8 layers,
    # the 8 reports following each launch: still one report per layer, in
    # order, and the per-layer launches' output bit for bit.
    image = W.realesrgan_input(200, 120, 31)
    seen = []
    staged = gpu_model.run_float_tiled(image, 256, 34, lambda f: seen.append(f) or False)
    assert len(seen) == 34 and seen[-1] == 1.0
    assert all(a < b for a, b in zip(seen, seen[1:]))
    gpu_model.set_fused(False)
    try:
        layered = gpu_model.run_float_tiled(image, 256, 34, lambda f: False)
    finally:
        gpu_model.set_fused(True)
    assert np.array_equal(staged.view(np.uint32), layered.view(np.uint32))
    assert np.array_equal(staged.view(np.uint32), gpu_model.run_float(image).view(np.uint32))

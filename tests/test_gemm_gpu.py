"""The general tcgen05 implicit GEMM (igemm_sm100) against the CPU oracle's
gemm::multiply (crates/native-engine/src/gemm.rs:514-667) on the same
f16-rounded inputs: rows and 3x3 convolutions, every tile shape the models
use, bias, ReLU / GELU, and accumulation onto an existing output. The GPU
rounds its result to f16; the tolerance is 2e-3 (1 + |v|)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def close(got, want, tol=2e-3):
    err = np.abs(got - want) / (1 + np.abs(want))
    assert np.isfinite(got).all()
    assert err.max() <= tol, (err.max(), np.unravel_index(err.argmax(), err.shape))


@pytest.mark.parametrize("m,k,n,act", [
    (256, 32, 96, 0), (128, 64, 64, 1), (384, 256, 768, 0), (512, 128, 32, 2), (256, 64, 192, 2),
    (1024, 512, 256, 0), (128, 1024, 512, 1), (256, 64, 3, 0),
])
def test_rows_match_oracle(m, k, n, act):
    import iec
    from oracle import refcpu

    rng = np.random.default_rng(m + k + n)
    a = f16(rng.standard_normal((m, k)))
    w = f16(rng.standard_normal((k, n)) / np.sqrt(k))
    bias = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    want = refcpu.multiply(a.ravel(), w, bias, kind="rows", act=act).reshape(m, n)
    got = iec.selftest_gemm(a, w, bias, act=act)
    close(got, want)


def test_rows_accumulate_onto_output():
    import iec
    from oracle import refcpu

    rng = np.random.default_rng(5)
    m, k, n = 256, 128, 64
    a = f16(rng.standard_normal((m, k)))
    w = f16(rng.standard_normal((k, n)) / np.sqrt(k))
    old = f16(rng.standard_normal((m, n)))
    want = refcpu.multiply(a.ravel(), w, None, kind="rows", out=old.ravel().copy(), accumulate=True).reshape(m, n)
    got = iec.selftest_gemm(a, w, None, accumulate_onto=old)
    close(got, want)


@pytest.mark.parametrize("h,w,k,n,act", [
    (16, 24, 32, 32, 1), (8, 8, 256, 256, 0), (24, 40, 64, 128, 0), (16, 16, 128, 128, 1), (32, 48, 16, 64, 0),
    (8, 16, 64, 3, 0),
])
def test_conv3_matches_oracle(h, w, k, n, act):
    import iec
    from oracle import refcpu

    rng = np.random.default_rng(h * w + k + n)
    img = f16(rng.standard_normal((h, w, k)))
    wt = f16(rng.standard_normal((9 * k, n)) / np.sqrt(9 * k))
    bias = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    want = refcpu.multiply(img.ravel(), wt, bias, kind="conv", shape=(h, w, k), size=3, act=act).reshape(h * w, n)
    got = iec.selftest_gemm(img, wt, bias, conv=True, shape=(h, w), act=act)
    close(got, want)


@pytest.mark.parametrize("h,w,k,n,size", [
    (24, 40, 64, 32, 3), (30, 70, 64, 64, 3), (20, 45, 32, 128, 3), (40, 64, 64, 3, 7), (24, 33, 16, 32, 5),
    (12, 50, 128, 96, 3), (9, 61, 256, 256, 3), (23, 97, 64, 3, 7), (40, 32, 64, 32, 1), (17, 100, 32, 48, 3),
    (64, 64, 128, 64, 3), (33, 47, 16, 32, 3), (13, 64, 256, 32, 3),
])
def test_conv_halo_tiles_match_oracle(h, w, k, n, size):
    """Square convolutions through halo tiles (one box per channel chunk, one
    MMA per kernel row with the row's taps side by side in N, the taps'
    products added across lanes in the epilogue) and through one box per
    tap, both against the oracle; partial tiles on both axes."""
    import iec
    from oracle import refcpu

    rng = np.random.default_rng(h * w * size + k + n)
    img = f16(rng.standard_normal((h, w, k)))
    taps = size * size
    wt = f16(rng.standard_normal((taps * k, n)) / np.sqrt(taps * k))
    bias = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    want = refcpu.multiply(img.ravel(), wt, bias, kind="conv", shape=(h, w, k), size=size, act=1).reshape(h * w, n)
    for halo in (1, 0):
        got, _ = iec.selftest_conv(img, wt, bias, size=size, halo=halo, act=1)
        close(got, want)


def test_mma_rate_diagnostic_runs():
    """The issue-rate diagnostic runs for every MMA width and both issue
    forms and returns a finite positive cycle count (no rate is asserted)."""
    import iec

    for n in (32, 96, 256):
        for variant in (0, 1):
            c = iec.selftest_mma_rate(n, variant)
            assert np.isfinite(c) and c > 0


@pytest.mark.parametrize("rows,c", [(1000, 64), (128 * 37, 64), (300, 128), (128 * 41 + 7, 128), (49152, 64),
                                    (200, 256), (128 * 150 + 33, 256), (24576, 256)])
def test_joinsplit_matches_separate_launches_and_oracle(rows, c):
    """SCUNet's fused block boundary (x += y Wj + bj; y = x Ws + bs in one
    kernel) equals the join and split as two GEMM launches bit for bit, and
    both follow the oracle's multiply (network.rs:190-212: conv1_2, the
    residual add, conv1_1 of the next block; f16 between the steps)."""
    import iec
    from oracle import refcpu

    rng = np.random.default_rng(rows + c)
    x = f16(rng.standard_normal((rows, c)))
    y = f16(rng.standard_normal((rows, c)))
    wj = f16(rng.standard_normal((c, c)) / np.sqrt(c))
    ws = f16(rng.standard_normal((c, c)) / np.sqrt(c))
    bj = rng.uniform(-0.5, 0.5, c).astype(np.float32)
    bs = rng.uniform(-0.5, 0.5, c).astype(np.float32)
    fx, fy, _ = iec.selftest_joinsplit(x, y, wj, bj, ws, bs, fused=True)
    sx, sy, _ = iec.selftest_joinsplit(x, y, wj, bj, ws, bs, fused=False)
    assert np.array_equal(fx.view(np.uint32), sx.view(np.uint32)), float(np.abs(fx - sx).max())
    assert np.array_equal(fy.view(np.uint32), sy.view(np.uint32)), float(np.abs(fy - sy).max())
    if rows <= 5000:
        want_x = f16(refcpu.multiply(y.ravel(), wj, bj, kind="rows", out=x.ravel().copy(),
                                     accumulate=True).reshape(rows, c))
        want_y = refcpu.multiply(fx.ravel(), ws, bs, kind="rows").reshape(rows, c)
        close(fx, want_x)
        close(fy, want_y)


@pytest.mark.parametrize("m,k,n,act,accumulate", [
    (256, 4096, 64, 0, False), (304, 2048, 96, 2, False), (256, 4096, 32, 0, True), (640, 2048, 128, 1, False),
])
def test_split_k_rows_match_oracle(m, k, n, act, accumulate):
    """Products with few row tiles and at least 32 K steps run their K steps
    in slices on more CTAs; the CTA that completes a tile's last slice adds
    the slices in order and applies the epilogue (bias, activation, the
    accumulated output)."""
    import iec
    from oracle import refcpu

    rng = np.random.default_rng(m + k + n + act)
    a = f16(rng.standard_normal((m, k)))
    w = f16(rng.standard_normal((k, n)) / np.sqrt(k))
    bias = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    old = f16(rng.standard_normal((m, n))) if accumulate else None
    want = refcpu.multiply(a.ravel(), w, bias, kind="rows", act=act,
                           out=None if old is None else old.ravel().copy(), accumulate=accumulate).reshape(m, n)
    for _ in range(2):  # the tile counters are left at zero for the next launch
        got = iec.selftest_gemm(a, w, bias, act=act, accumulate_onto=old)
        close(got, want)


def test_split_k_conv_matches_oracle():
    """A 3x3 convolution over 512 channels of a small map (72 K steps, few
    tiles) through the split-K path."""
    import iec
    from oracle import refcpu

    rng = np.random.default_rng(11)
    h, w, k, n = 12, 20, 512, 128
    a = f16(rng.standard_normal((h, w, k)))
    wt = f16(rng.standard_normal((9 * k, n)) / np.sqrt(9 * k))
    bias = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    want = refcpu.multiply(a.ravel(), wt, bias, kind="conv", shape=(h, w, k), size=3, act=1).reshape(h * w, n)
    for _ in range(2):
        got = iec.selftest_gemm(a, wt, bias, conv=True, shape=(h, w), act=1)
        close(got, want)

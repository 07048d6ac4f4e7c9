"""The CPU oracle's engine against the reference's own unit tests, restated.

Each test follows a test of crates/native-engine, with its inputs (the sin
sequences of gemm.rs:673-678, the LCG of winograd.rs:801-805) and its
tolerances; the f64 "textbook" products are the reference tests' oracles.
"""

import struct

import numpy as np
import pytest

from oracle import refcpu


def values(n, seed):
    """gemm.rs:673-678: ((i * 0.37 + seed).sin()) * 0.5, in f32."""
    i = np.arange(n, dtype=np.float32)
    return (np.sin(i * np.float32(0.37) + np.float32(seed)).astype(np.float32) * np.float32(0.5)).astype(np.float32)


def textbook(a_rows, w, bias):
    """gemm.rs:681-700: the f64 product."""
    return a_rows.astype(np.float64) @ w.astype(np.float64) + bias.astype(np.float64)


def close(got, want, tol=1e-4):
    """gemm.rs:702-713: |g - v| <= 1e-4 (1 + |v|)."""
    assert np.all(np.abs(got.astype(np.float64) - want) <= tol * (1 + np.abs(want))), np.abs(got - want).max()


@pytest.mark.parametrize("m,k,n", [(1, 3, 1), (7, 40, 17), (13, 1100, 48), (6, 512, 16)])
def test_dense_rows_match_reference(m, k, n):
    # gemm.rs:819-850
    a = values(m * k, 0.3)
    w = values(k * n, 1.1).reshape(k, n)
    bias = values(n, 2.0)
    stride = n + 3
    out = refcpu.multiply(a, w, bias, kind="rows", out_stride=stride)
    got = np.stack([out[r * stride:r * stride + n] for r in range(m)])
    close(got, textbook(a.reshape(m, k), w, bias))


def test_row_ranges_accumulate_onto_output():
    # gemm.rs:852-880
    m, k, n = 20, 70, 33
    a = values(m * k, 0.7)
    w = values(k * n, -0.4).reshape(k, n)
    want = textbook(a.reshape(m, k), w, np.zeros(n)) + 1.0
    out = np.ones(m * n, np.float32)
    for r0, r1 in [(0, 5), (5, 17), (17, 20)]:
        part = out[r0 * n:r1 * n]
        refcpu.multiply(a, w, None, kind="rows", rows=(r0, r1), out=part, accumulate=True)
    close(out.reshape(m, n), want)


def test_half_panels_match_reference():
    # gemm.rs:791-817: half-float weights are their halves, widened exactly.
    m, k, n = 11, 600, 40
    a = values(m * k, 0.1)
    halves = 0x3000 + (np.arange(k * n) % 977)
    w = np.array([refcpu.half_to_f32(int(h)) for h in halves], np.float32).reshape(k, n)
    bias = values(n, 0.5)
    out = refcpu.multiply(a, w, bias, kind="rows", half=True)
    close(out.reshape(m, n), textbook(a.reshape(m, k), w, bias))


@pytest.mark.parametrize("h,wd,c,gap,size,n", [
    (5, 7, 3, 0, 3, 20), (4, 9, 64, 0, 7, 16), (3, 3, 600, 0, 3, 5), (6, 5, 2, 0, 1, 3), (5, 6, 32, 32, 3, 32),
])
def test_same_convolution_matches_reference(h, wd, c, gap, size, n):
    # gemm.rs:882-926, with ReLU.
    stride = c + gap
    img = values(h * wd * stride, 0.9)
    k = size * size * c
    w = values(k * n, 0.2).reshape(k, n)
    bias = values(n, -1.0)
    out = refcpu.multiply(img, w, bias, kind="conv", shape=(h, wd, c), stride=stride, size=size, act=1)
    half = size // 2
    rows = np.zeros((h * wd, k), np.float32)
    for r in range(h * wd):
        for x in range(k):
            tap, ch = divmod(x, c)
            y = r // wd + tap // size - half
            xx = r % wd + tap % size - half
            if 0 <= y < h and 0 <= xx < wd:
                rows[r, x] = img[(y * wd + xx) * stride + ch]
    close(out.reshape(h * wd, n), np.maximum(textbook(rows, w, bias), 0.0))


def lcg(seed=1):
    # winograd.rs:801-805
    state = [seed]

    def nxt():
        state[0] = (state[0] * 1664525 + 1013904223) & 0xFFFFFFFF
        return np.float32((state[0] >> 8) / float(1 << 24) - 0.5)

    return nxt


def test_winograd_matches_direct_convolution():
    # winograd.rs:796-861: F(4x4) below 576 channels in+out, F(2x2) above,
    # zero and reflect padding, f32 (1e-4) and f16 (0.05) weights, strided
    # input and output, accumulation and a finishing closure.
    nxt = lcg(1)
    for height, width, cin, cout, reflect in [
        (7, 9, 8, 24, False), (6, 5, 16, 16, True), (1, 4, 3, 5, False),
        (5, 2, 20, 33, True), (6, 7, 400, 200, True), (3, 5, 300, 300, False),
    ]:
        for half, tol in [(False, 1e-4), (True, 0.05)]:
            stride = cin + 2
            data = np.array([nxt() for _ in range(height * width * stride)], np.float32)
            weights = np.array([nxt() for _ in range(9 * cin * cout)], np.float32)
            bias = np.array([nxt() for _ in range(cout)], np.float32)
            if half:
                weights = np.array([refcpu.half_to_f32(refcpu.f32_to_half(float(v))) for v in weights], np.float32)
            w = weights.reshape(9 * cin, cout)
            want = refcpu.multiply(data, w, bias, kind="conv", shape=(height, width, cin), stride=stride,
                                   size=3, reflect=reflect).reshape(height * width, cout)
            out_stride = cout + 1
            got = np.ones(height * width * out_stride, np.float32)
            refcpu.conv3(data, (height, width, cin), w, bias, stride=stride, reflect=reflect, half=half,
                         out=got, out_stride=out_stride, accumulate=True, double_first=True)
            got = got.reshape(height * width, out_stride)[:, :cout]
            expect = want + 1.0
            expect[:, 0] *= 2.0
            assert np.abs(got - expect).max() < tol, (height, width, cin, cout, half)


def test_half_conversion_round_trips_every_half():
    # half.rs: every finite half widens exactly and narrows back to itself.
    for h in range(0, 0x10000, 7):
        e = (h >> 10) & 0x1F
        v = refcpu.half_to_f32(h)
        want = np.frombuffer(struct.pack("<H", h), np.float16)[0].astype(np.float32)
        if e == 0x1F and (h & 0x3FF):
            assert np.isnan(v)
            continue
        assert v == want or (np.isnan(v) and np.isnan(want))
        assert refcpu.f32_to_half(v) == h


def test_half_rounds_to_nearest_even():
    for v in [1.0 + 2**-11, 1.0 + 3 * 2**-11, 65520.0, 1e-8, -2.0**-25, 2.0**-24 * 1.5, 3.14159]:
        with np.errstate(over="ignore"):
            want = int(np.frombuffer(np.float32(v).astype(np.float16).tobytes(), np.uint16)[0])
        assert refcpu.f32_to_half(v) == want, v


def weights_bytes(entries, magic=b"TESTFILE"):
    """weight_file.rs:189-209."""
    out = bytearray(magic)
    out += struct.pack("<II", 1, len(entries))
    for name, shape, data in entries:
        out += struct.pack("<H", len(name)) + name.encode() + bytes([0, len(shape)])
        for d in shape:
            out += struct.pack("<I", d)
        for v in data:
            out += struct.pack("<f", v)
    return bytes(out)


def test_weights_parse_truncation_and_huge_dims():
    # weight_file.rs:211-235
    good = weights_bytes([("a", [2, 1], [1.0, -2.5]), ("b", [], [7.0])])
    refcpu.parse_weights(good, b"TESTFILE")
    data = weights_bytes([("a", [4], [1.0, 2.0, 3.0, 4.0])])
    for cut in [3, 20, len(data) - 1]:
        with pytest.raises(refcpu.OracleError):
            refcpu.parse_weights(data[:cut], b"TESTFILE")
    huge = weights_bytes([("a", [0xFFFFFFFF] * 3, [])])
    with pytest.raises(refcpu.OracleError):
        refcpu.parse_weights(huge, b"TESTFILE")
    with pytest.raises(refcpu.OracleError):
        refcpu.parse_weights(good, b"OTHERMAG")
    with pytest.raises(refcpu.OracleError):
        refcpu.parse_weights(good + b"\0", b"TESTFILE")

"""Weights files in the reference's format, and seeded random-init weights.

The container (crates/native-engine/src/weight_file.rs:1-117, written by
tools/*/export_weights.py): 8 magic bytes naming the model, u32 version 1,
u32 tensor count, then per tensor a u16 name length, the UTF-8 name, a u8
type (0 float32, 1 float16), a u8 rank, u32 dimensions and the values, all
little-endian. Convolution weights are matrices of (ky, kx, cin) rows by cout
columns (tools/realesrgan/export_weights.py:48-55).

The real checkpoints are not available here, so benchmarks and tests use
seeded random-init weights of each architecture with exactly the tensor
names and shapes the reference's loaders take.
"""

from __future__ import annotations

import hashlib
import struct

import numpy as np

MAGIC = {
    "realesrgan": b"REALESRG",
    "scunet": b"SCUNET\0\0",
    "lama": b"LAMA\0\0\0\0",
    "birefnet": b"BIREFNET",
}


def encode(magic: bytes, tensors) -> bytes:
    """The bytes of a weights file holding `tensors`: (name, array, half)."""
    assert len(magic) == 8
    out = [magic, struct.pack("<II", 1, len(tensors))]
    for name, array, half in tensors:
        array = np.ascontiguousarray(array)
        encoded = name.encode()
        out.append(struct.pack("<H", len(encoded)))
        out.append(encoded)
        out.append(struct.pack("<BB", int(half), array.ndim))
        out.append(struct.pack(f"<{array.ndim}I", *array.shape))
        out.append(array.astype("<f2" if half else "<f4").tobytes())
    return b"".join(out)


def write(path, magic: bytes, tensors) -> str:
    """Write a weights file; returns its SHA-256."""
    data = encode(magic, tensors)
    with open(path, "wb") as f:
        f.write(data)
    return hashlib.sha256(data).hexdigest()


def realesrgan_tensors(seed: int = 0, bias_scale: float = 0.05):
    """SRVGGNetCompact (realesr-general-x4v3) tensors as
    crates/realesrgan-native/src/network.rs:54-74 loads them: for i in 0..34,
    body.{2i}.weight [9 cin, cout] He-normal (std sqrt(2 / (9 cin))),
    body.{2i}.bias [cout] uniform in +-bias_scale, and for i < 33 the PReLU
    slopes body.{2i+1}.weight [64] = 0.25. float32, as export_weights.py
    writes without --half."""
    rng = np.random.default_rng(seed)
    tensors = []
    for i in range(34):
        cin = 3 if i == 0 else 64
        cout = 48 if i == 33 else 64
        std = np.sqrt(2.0 / (9 * cin))
        w = (rng.standard_normal((9 * cin, cout)) * std).astype(np.float32)
        b = rng.uniform(-bias_scale, bias_scale, cout).astype(np.float32)
        tensors.append((f"body.{2 * i}.weight", w, False))
        tensors.append((f"body.{2 * i}.bias", b, False))
        if i < 33:
            tensors.append((f"body.{2 * i + 1}.weight", np.full(64, 0.25, np.float32), False))
    return tensors


def write_realesrgan(path, seed: int = 0) -> str:
    return write(path, MAGIC["realesrgan"], realesrgan_tensors(seed))


def realesrgan_input(width: int, height: int, seed: int = 0) -> np.ndarray:
    """A seeded RGB image, NHWC float32 uniform in [0, 1)."""
    rng = np.random.default_rng(seed)
    return rng.random((height, width, 3), dtype=np.float32)

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


def scunet_tensors(seed: int = 0, branch_gain: float = 0.25, tail_gain: float = 0.1):
    """SCUNet tensors as crates/scunet-native/src/network.rs:113-260 and
    swin.rs:101-119 load them, 2-D matrices in f16 (export --half), biases,
    norms and position biases f32. Convolutions He-normal, linear layers
    LeCun-normal; the last layer of each residual branch (conv_block.2,
    msa.linear, mlp.2, conv1_2) is scaled by `branch_gain` and the tail by
    `tail_gain`, so that the 28 residual blocks keep activations of order one
    and the output stays within a few units, as a trained denoiser's does
    (plain He/LeCun init compounds to outputs of several hundred). Position
    bias N(0, 0.02^2),
    LayerNorm weight 1 + N(0, 0.05^2), bias N(0, 0.02^2), biases U(+-0.05)."""
    rng = np.random.default_rng(seed)
    tensors = []
    half = lambda a: a.astype(np.float16).astype(np.float32)  # noqa: E731

    def conv3(name, cin, cout, gain=1.0):
        w = rng.standard_normal((9 * cin, cout)) * np.sqrt(2.0 / (9 * cin)) * gain
        tensors.append((f"{name}.weight", half(w), True))

    def lin(name, k, n, bias=True, gain=1.0):
        w = rng.standard_normal((k, n)) * np.sqrt(1.0 / k) * gain
        tensors.append((f"{name}.weight", half(w), True))
        if bias:
            tensors.append((f"{name}.bias", rng.uniform(-0.05, 0.05, n).astype(np.float32), False))

    def ln(name, c):
        tensors.append((f"{name}.weight", (1 + 0.05 * rng.standard_normal(c)).astype(np.float32), False))
        tensors.append((f"{name}.bias", (0.02 * rng.standard_normal(c)).astype(np.float32), False))

    def block(name, c):
        h = c // 2
        lin(f"{name}.conv1_1", c, c)
        conv3(f"{name}.conv_block.0", h, h)
        conv3(f"{name}.conv_block.2", h, h, branch_gain)
        t = f"{name}.trans_block"
        ln(f"{t}.ln1", h)
        lin(f"{t}.msa.embedding_layer", h, 3 * h)
        tensors.append((f"{t}.msa.position_bias", (0.02 * rng.standard_normal((h // 32, 64, 64))).astype(np.float32),
                        False))
        lin(f"{t}.msa.linear", h, h, gain=branch_gain)
        ln(f"{t}.ln2", h)
        lin(f"{t}.mlp.0", h, 4 * h)
        lin(f"{t}.mlp.2", 4 * h, h, gain=branch_gain)
        lin(f"{name}.conv1_2", c, c, gain=branch_gain)

    conv3("m_head.0", 3, 64)
    for i, c in [(1, 64), (2, 128), (3, 256)]:
        for b in range(4):
            block(f"m_down{i}.{b}", c)
        lin(f"m_down{i}.4", 4 * c, 2 * c, bias=False)
    for b in range(4):
        block(f"m_body.{b}", 512)
    for i, c in [(3, 256), (2, 128), (1, 64)]:
        lin(f"m_up{i}.0", 2 * c, 4 * c, bias=False)
        for b in range(1, 5):
            block(f"m_up{i}.{b}", c)
    conv3("m_tail.0", 64, 3, tail_gain)
    return tensors


def write_scunet(path, seed: int = 0) -> str:
    return write(path, MAGIC["scunet"], scunet_tensors(seed))


def scunet_input(width: int, height: int, seed: int = 0) -> np.ndarray:
    """A seeded noisy RGB image: uniform [0, 1) plus N(0, (25/255)^2), clamped."""
    rng = np.random.default_rng(seed)
    base = rng.random((height, width, 3))
    noisy = base + rng.standard_normal((height, width, 3)) * (25.0 / 255.0)
    return np.clip(noisy, 0.0, 1.0).astype(np.float32)


# crates/lama-native/src/network.rs:271 PHASE_TAPS: the (input offset, kernel
# tap) pairs one output phase of a 3x3 stride-2 transposed convolution reads
# along an axis.
LAMA_PHASE_TAPS = [[(0, 1)], [(0, 2), (1, 0)]]


def lama_phase_matrices(weight: np.ndarray):
    """A ConvTranspose2d weight [cin, cout, 3, 3] as the four phase matrices
    of tools/lama/export_weights.py:146-152: phase 2 py + px stacks the cin x
    cout slices of its taps, y-major."""
    out = []
    for phase in range(4):
        ys, xs = LAMA_PHASE_TAPS[phase // 2], LAMA_PHASE_TAPS[phase % 2]
        out.append(np.concatenate([weight[:, :, ky, kx] for _, ky in ys for _, kx in xs]))
    return out


def lama_tensors(seed: int = 0, branch_gain: float = 0.1, tail_gain: float = 0.3):
    """Big LaMa tensors as crates/lama-native/src/network.rs:151-171,280-297,
    381-403 load them: matrices f16 (export --half), biases f32. Batch norms
    are folded in the exported file, so the generator draws the folded
    matrices directly: convolutions He-normal (std sqrt(2 / fan_in)), biases
    U(+-0.05); the three layers that end the second convolution of each
    residual block (ffc1 local, cross, spectral_out) are scaled by
    `branch_gain` so that 18 residual additions of ReLU outputs stay of order
    one, and the last layer by `tail_gain` so that the sigmoid stays off its
    tails. The transposed convolutions are drawn as [cin, cout, 3, 3]
    weights and split into their phases with one shared bias."""
    rng = np.random.default_rng(seed)
    tensors = []
    half = lambda a: a.astype(np.float16).astype(np.float32)  # noqa: E731

    def mat(name, k, n, fan_in=None, bias=True, gain=1.0):
        w = rng.standard_normal((k, n)) * np.sqrt(2.0 / (fan_in or k)) * gain
        tensors.append((f"{name}.weight", half(w), True))
        if bias:
            tensors.append((f"{name}.bias", rng.uniform(-0.05, 0.05, n).astype(np.float32), False))

    mat("first", 49 * 4, 64)
    for i, (cin, cout) in enumerate([(64, 128), (128, 256), (256, 512)]):
        mat(f"down{i}", 9 * cin, cout)
    for b in range(18):
        for f in range(2):
            g = branch_gain if f == 1 else 1.0
            name = f"block{b}.ffc{f}"
            mat(f"{name}.local", 9 * 512, 128, gain=g)
            mat(f"{name}.cross", 9 * 128, 384, gain=g)
            mat(f"{name}.spectral_in", 384, 192)
            mat(f"{name}.fourier", 384, 384)
            mat(f"{name}.spectral_out", 192, 384, bias=False, gain=g)
    for i, (cin, cout) in enumerate([(512, 256), (256, 128), (128, 64)]):
        w = rng.standard_normal((cin, cout, 3, 3)) * np.sqrt(2.0 / (cin * 9 / 4))
        bias = rng.uniform(-0.05, 0.05, cout).astype(np.float32)
        for p, m in enumerate(lama_phase_matrices(w)):
            tensors.append((f"up{i}.phase{p}.weight", half(m), True))
            tensors.append((f"up{i}.phase{p}.bias", bias, False))
    mat("last", 49 * 64, 3, gain=tail_gain)
    return tensors


def write_lama(path, seed: int = 0) -> str:
    return write(path, MAGIC["lama"], lama_tensors(seed))


def lama_input(width: int, height: int, seed: int = 0, cover: float = 0.3):
    """A seeded inpainting input: RGB uniform [0, 1) (height x width x 3,
    float32) and a binary mask (height x width, 1 = fill) of random
    rectangles, each up to a quarter of each side, added until they cover
    `cover` of the image."""
    rng = np.random.default_rng(seed)
    image = rng.random((height, width, 3), dtype=np.float32)
    mask = np.zeros((height, width), np.float32)
    while mask.mean() < cover:
        rh = int(rng.integers(1, max(2, height // 4 + 1)))
        rw = int(rng.integers(1, max(2, width // 4 + 1)))
        y = int(rng.integers(0, height - rh + 1))
        x = int(rng.integers(0, width - rw + 1))
        mask[y:y + rh, x:x + rw] = 1.0
    return image, mask


BIREFNET_STAGES = [(96, 2), (192, 2), (384, 6), (768, 2)]
BIREFNET_SIZES = [1, 1, 3, 7]
BIREFNET_LEVELS = [(1728, 768), (960, 384), (480, 192), (240, 96)]
BIREFNET_MEAN = (0.485, 0.456, 0.406)
BIREFNET_STD = (0.229, 0.224, 0.225)


def birefnet_tensors(seed: int = 0, branch_gain: float = 0.3, offset_scale: float = 0.5, head_gain: float = 1.0):
    """BiRefNet-lite tensors as crates/birefnet-native/src/swin.rs:115-158 and
    decoder.rs:106-135,316-340,538-545,605-633,753-786 load them. As
    tools/birefnet/export_weights.py:248-259 writes them with --half: 2-D
    `.weight` tensors f16, everything else f32. Batch norms are folded in the
    exported file, so the generator draws the folded matrices directly:
    convolutions before a ReLU He-normal, other layers LeCun-normal, biases
    U(+-0.05), LayerNorm weight 1 + N(0, 0.05^2) and bias N(0, 0.02^2),
    position bias N(0, 0.02^2). The residual branches' last layers (proj,
    fc2) are scaled by `branch_gain`; the deformable offsets and modulator
    logits are drawn so that the offsets are of order `offset_scale` pixels."""
    rng = np.random.default_rng(seed)
    tensors = []

    def half(a):
        return a.astype(np.float16).astype(np.float32)

    def mat(name, k, n, bias=True, he=False, gain=1.0, bias_scale=0.05):
        w = rng.standard_normal((k, n)) * np.sqrt((2.0 if he else 1.0) / k) * gain
        tensors.append((f"{name}.weight", half(w), True))
        if bias:
            tensors.append((f"{name}.bias", rng.uniform(-bias_scale, bias_scale, n).astype(np.float32), False))

    def ln(name, c):
        tensors.append((f"{name}.weight", (1 + 0.05 * rng.standard_normal(c)).astype(np.float32), False))
        tensors.append((f"{name}.bias", (0.02 * rng.standard_normal(c)).astype(np.float32), False))

    mat("patch_embed", 48, 96)
    ln("patch_embed.norm", 96)
    for s, (c, depth) in enumerate(BIREFNET_STAGES):
        for b in range(depth):
            p = f"stage{s}.block{b}"
            ln(f"{p}.norm1", c)
            mat(f"{p}.qkv", c, 3 * c)
            tensors.append((f"{p}.position_bias",
                            (0.02 * rng.standard_normal((c // 32, 49, 49))).astype(np.float32), False))
            mat(f"{p}.proj", c, c, gain=branch_gain)
            ln(f"{p}.norm2", c)
            mat(f"{p}.fc1", c, 4 * c)
            mat(f"{p}.fc2", 4 * c, c, gain=branch_gain)
        if s < 3:
            ln(f"stage{s}.merge.norm", 4 * c)
            mat(f"stage{s}.merge", 4 * c, 2 * c, bias=False)
        ln(f"stage{s}.norm", c)

    def block(p, cin, cout, gate):
        mat(f"{p}.conv_in", 9 * cin, 64, he=True)
        mat(f"{p}.conv_out", 9 * 64, cout)
        if gate:
            mat(f"{p}.gdt", 9 * cout, 16, he=True)
            mat(f"{p}.gdt_attn", 16, 1)
        for i, k in enumerate(BIREFNET_SIZES):
            taps = k * k
            mat(f"{p}.aspp.branch{i}.offset", taps * 64, 3 * taps, gain=offset_scale, bias_scale=offset_scale)
            mat(f"{p}.aspp.branch{i}", taps * 64, 256, he=True)
        mat(f"{p}.aspp.pool", 64, 256, he=True)
        mat(f"{p}.aspp.conv1", 5 * 256, 64, he=True)

    block("squeeze", 2880, 1536, False)
    for i, (cin, cout) in enumerate(BIREFNET_LEVELS):
        block(f"block{4 - i}", cin, cout, i < 3)
    for n, c in [(4, 768), (3, 384), (2, 192)]:
        mat(f"lateral{n}", c, c)
    for n, cin, cout in [(5, 3072, 192), (4, 768, 192), (3, 192, 96), (2, 48, 48)]:
        mat(f"patches{n}.conv1", 9 * cin, 64)
        mat(f"patches{n}.conv_out", 9 * 64, cout)
    mat("head", 96, 1, gain=head_gain)
    mat("patches1.conv1", 27, 64)
    mat("patches1.conv_out", 9 * 64, 1)
    return tensors


def write_birefnet(path, seed: int = 0) -> str:
    return write(path, MAGIC["birefnet"], birefnet_tensors(seed))


def birefnet_input(side: int, seed: int = 0) -> np.ndarray:
    """A seeded 8-bit RGB image, side x side x 3, uniform over 0..255."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, (side, side, 3), dtype=np.uint8)


def birefnet_normalize(rgb: np.ndarray) -> np.ndarray:
    """lib.rs:116-133: (v / 255 - mean) / std per colour, in f32."""
    table = np.empty((256, 3), np.float32)
    v = np.arange(256, dtype=np.float32) / np.float32(255.0)
    for c in range(3):
        table[:, c] = (v - np.float32(BIREFNET_MEAN[c])) / np.float32(BIREFNET_STD[c])
    return table[rgb, np.arange(3)].astype(np.float32)

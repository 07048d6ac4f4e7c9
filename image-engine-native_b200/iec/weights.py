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


# ------------------------------------------------------------------ layouts
# The exporters (tools/*/export_weights.py) turn upstream PyTorch layouts into
# the engine's; these helpers state each mapping and its inverse.


def conv_matrix(w: np.ndarray) -> np.ndarray:
    """A convolution weight [cout, cin, ky, kx] as the engine's matrix of
    (ky, kx, cin) rows by cout columns (tools/realesrgan/export_weights.py:
    48-55, and the same function in the SCUNet and LaMa exporters)."""
    cout, cin, kh, kw = w.shape
    return np.transpose(w, (2, 3, 1, 0)).reshape(kh * kw * cin, cout)


def conv_weight(m: np.ndarray, kh: int, kw: int) -> np.ndarray:
    """The inverse of conv_matrix."""
    rows, cout = m.shape
    cin = rows // (kh * kw)
    return np.ascontiguousarray(np.transpose(m.reshape(kh, kw, cin, cout), (3, 2, 0, 1)))


def transposed_matrix(w: np.ndarray) -> np.ndarray:
    """A transposed convolution weight [cin, cout, ky, kx] as cin rows by
    (ky, kx, cout) columns (tools/scunet/export_weights.py:57-60)."""
    cin, cout, kh, kw = w.shape
    return np.transpose(w, (0, 2, 3, 1)).reshape(cin, kh * kw * cout)


def transposed_weight(m: np.ndarray, kh: int, kw: int) -> np.ndarray:
    """The inverse of transposed_matrix."""
    cin, cols = m.shape
    cout = cols // (kh * kw)
    return np.ascontiguousarray(np.transpose(m.reshape(cin, kh, kw, cout), (0, 3, 1, 2)))


# -------------------------------------------------------------- Real-ESRGAN
def realesrgan_checkpoint(seed: int = 0, bias_scale: float = 0.05):
    """A seeded SRVGGNetCompact state dict in the upstream layout that
    tools/realesrgan/export_weights.py reads (its "params_ema" set): for i in
    0..34, body.{2i}.weight [cout, cin, 3, 3] He-normal (std
    sqrt(2 / (9 cin))), body.{2i}.bias [cout] uniform in +-bias_scale, and
    for i < 33 the PReLU slopes body.{2i+1}.weight [64] = 0.25 (names from
    crates/realesrgan-native/src/network.rs:54-74, which the exporter passes
    through unchanged)."""
    rng = np.random.default_rng(seed)
    state = {}
    for i in range(34):
        cin = 3 if i == 0 else 64
        cout = 48 if i == 33 else 64
        std = np.sqrt(2.0 / (9 * cin))
        m = (rng.standard_normal((9 * cin, cout)) * std).astype(np.float32)
        state[f"body.{2 * i}.weight"] = conv_weight(m, 3, 3)
        state[f"body.{2 * i}.bias"] = rng.uniform(-bias_scale, bias_scale, cout).astype(np.float32)
        if i < 33:
            state[f"body.{2 * i + 1}.weight"] = np.full(64, 0.25, np.float32)
    return state


def export_realesrgan(state, weak=None, strength=None, half: bool = False):
    """tools/realesrgan/export_weights.py:48-101 restated: with `weak`, every
    tensor blended as strength * state + (1 - strength) * weak in float32
    (Real-ESRGAN's --denoise_strength; lines 83-93), then each 4-D
    convolution weight as its engine matrix (lines 48-55); with `half`, the
    2-D matrices stored as f16. Returns (name, array, half) in file order."""
    state = {k: np.asarray(v, np.float32) for k, v in state.items()}
    if weak is not None:
        s = np.float32(strength)
        weak = {k: np.asarray(v, np.float32) for k, v in weak.items()}
        if weak.keys() != state.keys() or any(weak[k].shape != v.shape for k, v in state.items()):
            raise ValueError("the two checkpoints hold different tensors")
        state = {k: s * v + (np.float32(1) - s) * weak[k] for k, v in state.items()}
    out = []
    for name, value in state.items():
        if value.ndim == 4:
            value = conv_matrix(value)
        out.append((name, value, half and value.ndim == 2))
    return out


def realesrgan_tensors(seed: int = 0, bias_scale: float = 0.05):
    """The seeded Real-ESRGAN file's tensors: realesrgan_checkpoint(seed)
    through the exporter's mapping (float32, as written without --half)."""
    return export_realesrgan(realesrgan_checkpoint(seed, bias_scale))


def write_realesrgan(path, seed: int = 0) -> str:
    return write(path, MAGIC["realesrgan"], realesrgan_tensors(seed))


def realesrgan_input(width: int, height: int, seed: int = 0) -> np.ndarray:
    """A seeded RGB image, NHWC float32 uniform in [0, 1)."""
    rng = np.random.default_rng(seed)
    return rng.random((height, width, 3), dtype=np.float32)


SCUNET_WINDOW = 8


def scunet_position_bias(params: np.ndarray) -> np.ndarray:
    """A window attention's relative position parameters [heads, 15, 15] as
    its whole bias [heads, 64, 64]: the bias between the tokens at (y1, x1)
    and (y2, x2) of a window is params[:, y1 - y2 + 7, x1 - x2 + 7]
    (tools/scunet/export_weights.py:63-69)."""
    n = SCUNET_WINDOW
    y, x = np.divmod(np.arange(n * n), n)
    dy = y[:, None] - y[None, :] + n - 1
    dx = x[:, None] - x[None, :] + n - 1
    return params[:, dy, dx]


def scunet_checkpoint(seed: int = 0, branch_gain: float = 0.25, tail_gain: float = 0.1):
    """A seeded SCUNet state dict in the upstream layout that
    tools/scunet/export_weights.py reads, float32: convolutions (m_head.0,
    the blocks' conv1_1, conv1_2 and conv_block.{0,2}, the strided m_down*.4,
    m_tail.0) as [cout, cin, ky, kx], the transposed m_up*.0 as
    [cin, cout, 2, 2], linear layers (msa.embedding_layer, msa.linear,
    mlp.{0,2}) as [out, in], and each attention's
    msa.relative_position_params [heads, 15, 15]; the block and tensor names
    are those crates/scunet-native/src/network.rs:113-260 and swin.rs:101-119
    load, which the exporter keeps.
    Values: convolutions He-normal, linear layers LeCun-normal; the last
    layer of each residual branch (conv_block.2, msa.linear, mlp.2, conv1_2)
    scaled by `branch_gain` and the tail by `tail_gain`, so that the 28
    residual blocks keep activations of order one and the output stays
    within a few units, as a trained denoiser's does (plain He/LeCun init
    compounds to outputs of several hundred). Position parameters
    N(0, 0.02^2), LayerNorm weight 1 + N(0, 0.05^2) and bias N(0, 0.02^2),
    biases U(+-0.05)."""
    rng = np.random.default_rng(seed)
    state = {}

    def draw(k, n, std):
        return (rng.standard_normal((k, n)) * std).astype(np.float32)

    def conv(name, cin, cout, size, gain=1.0, he=True, bias=False):
        m = draw(size * size * cin, cout, np.sqrt((2.0 if he else 1.0) / (size * size * cin)) * gain)
        state[f"{name}.weight"] = conv_weight(m, size, size)
        if bias:
            state[f"{name}.bias"] = rng.uniform(-0.05, 0.05, cout).astype(np.float32)

    def linear(name, k, n, gain=1.0):
        state[f"{name}.weight"] = np.ascontiguousarray(draw(k, n, np.sqrt(1.0 / k) * gain).T)
        state[f"{name}.bias"] = rng.uniform(-0.05, 0.05, n).astype(np.float32)

    def ln(name, c):
        state[f"{name}.weight"] = (1 + 0.05 * rng.standard_normal(c)).astype(np.float32)
        state[f"{name}.bias"] = (0.02 * rng.standard_normal(c)).astype(np.float32)

    def block(name, c):
        h = c // 2
        conv(f"{name}.conv1_1", c, c, 1, he=False, bias=True)
        conv(f"{name}.conv_block.0", h, h, 3)
        conv(f"{name}.conv_block.2", h, h, 3, branch_gain)
        t = f"{name}.trans_block"
        ln(f"{t}.ln1", h)
        linear(f"{t}.msa.embedding_layer", h, 3 * h)
        state[f"{t}.msa.relative_position_params"] = (
            0.02 * rng.standard_normal((h // 32, 2 * SCUNET_WINDOW - 1, 2 * SCUNET_WINDOW - 1))).astype(np.float32)
        linear(f"{t}.msa.linear", h, h, gain=branch_gain)
        ln(f"{t}.ln2", h)
        linear(f"{t}.mlp.0", h, 4 * h)
        linear(f"{t}.mlp.2", 4 * h, h, gain=branch_gain)
        conv(f"{name}.conv1_2", c, c, 1, branch_gain, he=False, bias=True)

    conv("m_head.0", 3, 64, 3)
    for i, c in [(1, 64), (2, 128), (3, 256)]:
        for b in range(4):
            block(f"m_down{i}.{b}", c)
        conv(f"m_down{i}.4", c, 2 * c, 2, he=False)
    for b in range(4):
        block(f"m_body.{b}", 512)
    for i, c in [(3, 256), (2, 128), (1, 64)]:
        m = draw(2 * c, 4 * c, np.sqrt(1.0 / (2 * c)))
        state[f"m_up{i}.0.weight"] = transposed_weight(m, 2, 2)
        for b in range(1, 5):
            block(f"m_up{i}.{b}", c)
    conv("m_tail.0", 64, 3, 3, tail_gain)
    return state


def export_scunet(state, half: bool = True):
    """tools/scunet/export_weights.py:72-104 restated: relative position
    parameters become the whole position_bias, the m_up*.0 transposed
    convolutions cin x (ky, kx, cout) matrices, other 4-D weights conv
    matrices, 2-D (linear) weights transposed to in x out; with `half`, 2-D
    `.weight` tensors are stored as f16. Returns (name, array, half)."""
    out = []
    for name, value in state.items():
        value = np.asarray(value, np.float32)
        if name.endswith(".relative_position_params"):
            name = name[: -len("relative_position_params")] + "position_bias"
            value = scunet_position_bias(value)
        elif name.startswith("m_up") and name.split(".")[1:] == ["0", "weight"]:
            value = transposed_matrix(value)
        elif value.ndim == 4:
            value = conv_matrix(value)
        elif value.ndim == 2:
            value = value.T
        out.append((name, value, half and value.ndim == 2 and name.endswith(".weight")))
    return out


def scunet_tensors(seed: int = 0, branch_gain: float = 0.25, tail_gain: float = 0.1):
    """The seeded SCUNet file's tensors: scunet_checkpoint(seed) through the
    exporter's mapping with --half (2-D matrices f16; biases, norms and
    position biases f32)."""
    return export_scunet(scunet_checkpoint(seed, branch_gain, tail_gain))


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


LAMA_LOCAL, LAMA_GLOBAL, LAMA_BLOCKS = 128, 384, 18
LAMA_BN_EPS = 1e-5


def lama_checkpoint(seed: int = 0, branch_gain: float = 0.1, tail_gain: float = 0.3):
    """A seeded Big LaMa generator state dict in the upstream layout that
    tools/lama/export_weights.py reads (the names after its
    "generator.model." prefix, from that exporter's code), float32:

    * 1, 2, 3: the first conv7 (4 -> 64) and two stride-2 downsamplings, each
      ffc.convl2l [cout, cin, k, k] with batch norm bn_l;
    * 4: the last downsampling split into ffc.convl2l (256 -> 128) and
      ffc.convl2g (256 -> 384) with bn_l and bn_g;
    * 5 .. 22, conv1 and conv2: the fast Fourier convolutions, ffc.convl2l,
      convg2l, convl2g (3x3), the spectral transform ffc.convg2g.conv1.0
      (384 -> 192, 1x1) with batch norm conv1.1, fu.conv_layer (384 -> 384,
      1x1, channels alternating real and imaginary parts) with fu.bn, and
      conv2 (192 -> 384); bn_l and bn_g;
    * 24, 27, 30: ConvTranspose2d [cin, cout, 3, 3] with bias, batch norms
      25, 28, 31; 34: the last conv7 (64 -> 3) with bias.

    Values: convolutions He-normal (std sqrt(2 / fan_in)); the layers that
    end the second convolution of each residual block (conv2's convl2l,
    convg2l, convl2g and the spectral conv2) are scaled by `branch_gain` so
    that 18 residual additions of ReLU outputs stay of order one, and the
    last layer by `tail_gain` so that the sigmoid stays off its tails. Batch
    norms: weight 1 + N(0, 0.05^2), bias U(+-0.05), running mean
    N(0, 0.05^2), running variance U(0.8, 1.25); biases U(+-0.05)."""
    rng = np.random.default_rng(seed)
    state = {}

    def conv(name, cin, cout, k, gain=1.0, fan_in=None):
        std = np.sqrt(2.0 / (fan_in or k * k * cin)) * gain
        state[name] = (rng.standard_normal((cout, cin, k, k)) * std).astype(np.float32)

    def bn(name, c):
        state[f"{name}.weight"] = (1 + 0.05 * rng.standard_normal(c)).astype(np.float32)
        state[f"{name}.bias"] = rng.uniform(-0.05, 0.05, c).astype(np.float32)
        state[f"{name}.running_mean"] = (0.05 * rng.standard_normal(c)).astype(np.float32)
        state[f"{name}.running_var"] = rng.uniform(0.8, 1.25, c).astype(np.float32)
        state[f"{name}.num_batches_tracked"] = np.array(1000, np.int64)

    conv("1.ffc.convl2l.weight", 4, 64, 7)
    bn("1.bn_l", 64)
    for layer, (cin, cout) in ((2, (64, 128)), (3, (128, 256))):
        conv(f"{layer}.ffc.convl2l.weight", cin, cout, 3)
        bn(f"{layer}.bn_l", cout)
    conv("4.ffc.convl2l.weight", 256, LAMA_LOCAL, 3)
    conv("4.ffc.convl2g.weight", 256, LAMA_GLOBAL, 3)
    bn("4.bn_l", LAMA_LOCAL)
    bn("4.bn_g", LAMA_GLOBAL)
    spectral = LAMA_GLOBAL // 2
    for b in range(LAMA_BLOCKS):
        for half, g in (("conv1", 1.0), ("conv2", branch_gain)):
            p = f"{5 + b}.{half}"
            fan_local = 9 * (LAMA_LOCAL + LAMA_GLOBAL)
            conv(f"{p}.ffc.convl2l.weight", LAMA_LOCAL, LAMA_LOCAL, 3, g, fan_local)
            conv(f"{p}.ffc.convg2l.weight", LAMA_GLOBAL, LAMA_LOCAL, 3, g, fan_local)
            conv(f"{p}.ffc.convl2g.weight", LAMA_LOCAL, LAMA_GLOBAL, 3, g)
            conv(f"{p}.ffc.convg2g.conv1.0.weight", LAMA_GLOBAL, spectral, 1)
            bn(f"{p}.ffc.convg2g.conv1.1", spectral)
            conv(f"{p}.ffc.convg2g.fu.conv_layer.weight", 2 * spectral, 2 * spectral, 1)
            bn(f"{p}.ffc.convg2g.fu.bn", 2 * spectral)
            conv(f"{p}.ffc.convg2g.conv2.weight", spectral, LAMA_GLOBAL, 1, g)
            bn(f"{p}.bn_l", LAMA_LOCAL)
            bn(f"{p}.bn_g", LAMA_GLOBAL)
    for layer, (cin, cout) in ((24, (512, 256)), (27, (256, 128)), (30, (128, 64))):
        std = np.sqrt(2.0 / (cin * 9 / 4))
        state[f"{layer}.weight"] = (rng.standard_normal((cin, cout, 3, 3)) * std).astype(np.float32)
        state[f"{layer}.bias"] = rng.uniform(-0.05, 0.05, cout).astype(np.float32)
        bn(str(layer + 1), cout)
    conv("34.weight", 64, 3, 7, tail_gain)
    state["34.bias"] = rng.uniform(-0.05, 0.05, 3).astype(np.float32)
    return state


def export_lama(state, half: bool = False):
    """tools/lama/export_weights.py:86-164 restated: each batch norm folded
    into the convolution before it (scale w / sqrt(var + 1e-5), shift
    b - mean scale, in float32); the local-to-local and global-to-local
    convolutions of each fast Fourier convolution joined along their input
    channels as "local", local-to-global as "cross"; the spectral transform's
    1x1 convolutions as "spectral_in", "fourier" (its channels reordered from
    interleaved real/imaginary to all real parts, then all imaginary ones)
    and "spectral_out" (carrying bn_g's scale); each transposed convolution
    as four phase products. With `half`, 2-D matrices are stored as f16.
    Returns (name, array, half) in file order."""
    src = {k: np.asarray(v, np.float32) for k, v in state.items() if not k.endswith("num_batches_tracked")}
    used = set()

    def get(name):
        used.add(name)
        return src[name]

    def bn(name):
        scale = get(f"{name}.weight") / np.sqrt(get(f"{name}.running_var") + LAMA_BN_EPS)
        return scale, get(f"{name}.bias") - get(f"{name}.running_mean") * scale

    out = []

    def put(name, matrix, bias=None):
        out.append((f"{name}.weight", np.asarray(matrix, np.float32), half and matrix.ndim == 2))
        if bias is not None:
            out.append((f"{name}.bias", np.asarray(bias, np.float32), False))

    scale, shift = bn("1.bn_l")
    put("first", conv_matrix(get("1.ffc.convl2l.weight")) * scale, shift)
    for i, layer in enumerate((2, 3)):
        scale, shift = bn(f"{layer}.bn_l")
        put(f"down{i}", conv_matrix(get(f"{layer}.ffc.convl2l.weight")) * scale, shift)
    joined = np.concatenate([get("4.ffc.convl2l.weight"), get("4.ffc.convl2g.weight")])
    (sl, hl), (sg, hg) = bn("4.bn_l"), bn("4.bn_g")
    put("down2", conv_matrix(joined) * np.concatenate([sl, sg]), np.concatenate([hl, hg]))
    spectral = LAMA_GLOBAL // 2
    planar = np.array([2 * c + j for j in range(2) for c in range(spectral)])
    for b in range(LAMA_BLOCKS):
        for f, part in enumerate(("conv1", "conv2")):
            p, name = f"{5 + b}.{part}", f"block{b}.ffc{f}"
            (sl, hl), (sg, hg) = bn(f"{p}.bn_l"), bn(f"{p}.bn_g")
            local = np.concatenate([get(f"{p}.ffc.convl2l.weight"), get(f"{p}.ffc.convg2l.weight")], axis=1)
            put(f"{name}.local", conv_matrix(local) * sl, hl)
            put(f"{name}.cross", conv_matrix(get(f"{p}.ffc.convl2g.weight")) * sg, hg)
            g = f"{p}.ffc.convg2g"
            scale, shift = bn(f"{g}.conv1.1")
            put(f"{name}.spectral_in", conv_matrix(get(f"{g}.conv1.0.weight")) * scale, shift)
            scale, shift = bn(f"{g}.fu.bn")
            fourier = conv_matrix(get(f"{g}.fu.conv_layer.weight")) * scale
            put(f"{name}.fourier", fourier[planar][:, planar], shift[planar])
            put(f"{name}.spectral_out", conv_matrix(get(f"{g}.conv2.weight")) * sg)
    for i, (layer, norm) in enumerate(((24, 25), (27, 28), (30, 31))):
        weight = get(f"{layer}.weight")
        scale, shift = bn(str(norm))
        bias = get(f"{layer}.bias") * scale + shift
        for phase, m in enumerate(lama_phase_matrices(weight)):
            put(f"up{i}.phase{phase}", m * scale, bias)
    put("last", conv_matrix(get("34.weight")), get("34.bias"))
    unused = sorted(set(src) - used)
    if unused:
        raise ValueError(f"generator tensors not exported: {unused[:5]}")
    return out


def lama_tensors(seed: int = 0, branch_gain: float = 0.1, tail_gain: float = 0.3):
    """The seeded Big LaMa file's tensors: lama_checkpoint(seed) through the
    exporter's mapping, float32 (written without --half; the backend rounds
    the matrices to f16 at load)."""
    return export_lama(lama_checkpoint(seed, branch_gain, tail_gain))


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

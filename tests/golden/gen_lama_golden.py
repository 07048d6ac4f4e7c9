#!/usr/bin/env python3
"""Generate the golden fixture that pins the LaMa oracle: lama_torch.npz.

    python tests/golden/gen_lama_golden.py

The reference checks its LaMa against LaMa's own PyTorch generator
(tools/lama/torch_reference.py), which imports the third-party LaMa sources;
those are not in this container. So this script restates the generator's
published forward pass (FFCResNetGenerator with every batch norm folded, as
tools/lama/export_weights.py:86-164 folds them) in float64 PyTorch of its own,
built from the same seeded weights file the oracle reads, converted back
through the inverse of the exporter's mapping:

- matrices [(ky, kx, cin), cout] -> conv weights [cout, cin, ky, kx]
  (export_weights.py:80-83);
- the Fourier unit's matrix from the planar order [re(c) | im(c)] back to
  the interleaved channels 2c + j that torch.stack(real, imag) makes
  (export_weights.py:104,130-131);
- the four phase matrices of each transposed convolution back to one
  ConvTranspose2d weight [cin, cout, 3, 3] (export_weights.py:146-152).

It then runs torch's own reflect padding, strided and transposed
convolutions and rfftn / irfftn with norm="ortho". This pins the oracle's
restatement of the things the weights file alone does not say: the phase
taps, the FFT conventions (which parts the inverse reads), the channel order
of the spectrum and the padding modes.
"""

from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "image-engine-native_b200"))

from iec import weights as W  # noqa: E402

# (width, height, input seed): odd transform lengths, the smallest size, and
# a size whose sides are not multiples of 8.
CASES = [(40, 24, 1), (9, 9, 2), (27, 35, 3)]


def torch_state(tensors):
    import torch

    return {name: torch.from_numpy(np.asarray(a, np.float64)) for name, a, _ in tensors}


def conv_weight(m, size):
    """[(ky, kx, cin), cout] -> [cout, cin, ky, kx]."""
    k, cout = m.shape
    cin = k // (size * size)
    return m.reshape(size, size, cin, cout).permute(3, 2, 0, 1).contiguous()


def transposed_weight(phases, cin, cout):
    """The inverse of weights.lama_phase_matrices."""
    import torch

    w = torch.zeros(cin, cout, 3, 3, dtype=torch.float64)
    for p, m in enumerate(phases):
        ys, xs = W.LAMA_PHASE_TAPS[p // 2], W.LAMA_PHASE_TAPS[p % 2]
        t = 0
        for _, ky in ys:
            for _, kx in xs:
                w[:, :, ky, kx] = m[t * cin:(t + 1) * cin]
                t += 1
    return w


def forward(state, image, mask):
    """The generator on one image: image h x w x 3, mask h x w, in 0..=1."""
    import torch
    import torch.nn.functional as F

    s = state
    height, width = mask.shape
    h, w = -(-height // 8) * 8, -(-width // 8) * 8
    img = torch.from_numpy(image.astype(np.float64)).permute(2, 0, 1)
    m = torch.from_numpy(mask.astype(np.float64))[None]
    x = torch.cat([img * (1 - m), m])[None]
    # Padding to a multiple of 8 mirrors the last rows and columns, the edge
    # pixel repeated (numpy's "symmetric"; network.rs:348-370).
    xs = x[0].numpy()
    xs = np.pad(xs, ((0, 0), (0, h - height), (0, w - width)), mode="symmetric")
    x = torch.from_numpy(xs)[None]

    def conv(x, name, size, stride=1, bias=True, reflect=True):
        pad = size // 2
        if reflect and pad:
            x = F.pad(x, (pad, pad, pad, pad), mode="reflect")
        b = s[f"{name}.bias"] if bias else None
        return F.conv2d(x, conv_weight(s[f"{name}.weight"], size), b, stride=stride)

    x = F.relu(conv(x, "first", 7))
    for i in range(3):
        x = F.relu(conv(x, f"down{i}", 3, stride=2))

    def spectral(xg, name):
        y = F.relu(conv(xg, f"{name}.spectral_in", 1))
        c = y.shape[1]
        hh, ww = y.shape[-2:]
        f = torch.fft.rfftn(y, dim=(-2, -1), norm="ortho")
        f = torch.stack((f.real, f.imag), dim=2).reshape(1, 2 * c, hh, ww // 2 + 1)
        planar = np.array([2 * ch + j for j in range(2) for ch in range(c)])
        wf = torch.zeros_like(s[f"{name}.fourier.weight"])
        bf = torch.zeros_like(s[f"{name}.fourier.bias"])
        wf[np.ix_(planar, planar)] = s[f"{name}.fourier.weight"]
        bf[planar] = s[f"{name}.fourier.bias"]
        f = F.relu(F.conv2d(f, wf.t().reshape(2 * c, 2 * c, 1, 1), bf))
        f = f.reshape(1, c, 2, hh, ww // 2 + 1)
        f = torch.complex(f[:, :, 0], f[:, :, 1])
        back = torch.fft.irfftn(f, s=(hh, ww), dim=(-2, -1), norm="ortho")
        return F.conv2d(y + back, conv_weight(s[f"{name}.spectral_out.weight"], 1))

    def ffc(x, name):
        xl = x[:, :128]
        local = F.relu(conv(x, f"{name}.local", 3))
        glob = F.relu(conv(xl, f"{name}.cross", 3) + spectral(x[:, 128:], name))
        return torch.cat([local, glob], dim=1)

    for b in range(18):
        x = x + ffc(ffc(x, f"block{b}.ffc0"), f"block{b}.ffc1")
    for i, (cin, cout) in enumerate([(512, 256), (256, 128), (128, 64)]):
        phases = [s[f"up{i}.phase{p}.weight"] for p in range(4)]
        wt = transposed_weight(phases, cin, cout)
        x = F.relu(F.conv_transpose2d(x, wt, s[f"up{i}.phase0.bias"], stride=2, padding=1, output_padding=1))
    x = torch.sigmoid(conv(x, "last", 7))
    return x[0, :, :height, :width].permute(1, 2, 0).numpy()


def main():
    import torch

    torch.set_num_threads(8)
    tensors = W.lama_tensors(0)
    sha = hashlib.sha256(W.encode(W.MAGIC["lama"], tensors)).hexdigest()
    state = torch_state(tensors)
    out = {"weights_sha256": np.array(sha)}
    for i, (width, height, seed) in enumerate(CASES):
        image, mask = W.lama_input(width, height, seed)
        with torch.no_grad():
            pred = forward(state, image, mask)
        out[f"case{i}_image"] = image
        out[f"case{i}_mask"] = mask
        out[f"case{i}_out"] = pred.astype(np.float32)
        print(f"case {i}: {width} x {height}, output mean {pred.mean():.4f}")
    np.savez_compressed(os.path.join(HERE, "lama_torch.npz"), **out)


if __name__ == "__main__":
    main()

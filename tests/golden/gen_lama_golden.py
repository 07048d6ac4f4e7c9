#!/usr/bin/env python3
"""Generate the golden fixture that pins the LaMa oracle: lama_torch.npz.

    python tests/golden/gen_lama_golden.py

The reference checks its LaMa against LaMa's own PyTorch generator
(tools/lama/torch_reference.py), which imports the third-party LaMa sources;
those are not in this container. So this script restates the generator's
published forward pass in float64 PyTorch of its own, run directly on the
seeded upstream checkpoint (iec.weights.lama_checkpoint: the tensors the
reference's tools/lama/export_weights.py reads, under its names): batch norms
in evaluation mode, the fast Fourier convolutions' four convolutions, the
Fourier unit's 1x1 convolution over channels that alternate real and
imaginary parts (torch.stack(real, imag) order), and ConvTranspose2d for the
upsamplings. The oracle reads the weights file that the reference's exporter
writes from that checkpoint (byte for byte: tests/test_export_pinning.py), so
this fixture pins the oracle's reading of the exported layout (folded batch
norms, the planar real|imaginary reorder, the phase split of the transposed
convolutions) together with what the file alone does not say: the phase
taps, the FFT conventions (which parts the inverse reads), the channel order
of the spectrum and the padding modes. It uses torch's own reflect padding,
strided and transposed convolutions and rfftn / irfftn with norm="ortho".
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


BN_EPS = 1e-5


def torch_state(state):
    import torch

    return {name: torch.from_numpy(np.asarray(a, np.float64)) for name, a in state.items()
            if not name.endswith("num_batches_tracked")}


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

    def bn(x, name):
        return F.batch_norm(x, s[f"{name}.running_mean"], s[f"{name}.running_var"], s[f"{name}.weight"],
                            s[f"{name}.bias"], training=False, eps=BN_EPS)

    def conv(x, weight, stride=1, bias=None):
        pad = weight.shape[-1] // 2
        if pad:
            x = F.pad(x, (pad, pad, pad, pad), mode="reflect")
        return F.conv2d(x, s[weight] if isinstance(weight, str) else weight, bias, stride=stride)

    x = F.relu(bn(F.conv2d(F.pad(x, (3, 3, 3, 3), mode="reflect"), s["1.ffc.convl2l.weight"]), "1.bn_l"))
    for layer in (2, 3):
        x = F.relu(bn(conv(x, s[f"{layer}.ffc.convl2l.weight"], 2), f"{layer}.bn_l"))
    xl = F.relu(bn(conv(x, s["4.ffc.convl2l.weight"], 2), "4.bn_l"))
    xg = F.relu(bn(conv(x, s["4.ffc.convl2g.weight"], 2), "4.bn_g"))

    def spectral(xg, g):
        y = F.relu(bn(F.conv2d(xg, s[f"{g}.conv1.0.weight"]), f"{g}.conv1.1"))
        c = y.shape[1]
        hh, ww = y.shape[-2:]
        f = torch.fft.rfftn(y, dim=(-2, -1), norm="ortho")
        f = torch.stack((f.real, f.imag), dim=2).reshape(1, 2 * c, hh, ww // 2 + 1)
        f = F.relu(bn(F.conv2d(f, s[f"{g}.fu.conv_layer.weight"]), f"{g}.fu.bn"))
        f = f.reshape(1, c, 2, hh, ww // 2 + 1)
        f = torch.complex(f[:, :, 0], f[:, :, 1])
        back = torch.fft.irfftn(f, s=(hh, ww), dim=(-2, -1), norm="ortho")
        return F.conv2d(y + back, s[f"{g}.conv2.weight"])

    def ffc(xl, xg, p):
        local = conv(xl, s[f"{p}.ffc.convl2l.weight"]) + conv(xg, s[f"{p}.ffc.convg2l.weight"])
        glob = conv(xl, s[f"{p}.ffc.convl2g.weight"]) + spectral(xg, f"{p}.ffc.convg2g")
        return F.relu(bn(local, f"{p}.bn_l")), F.relu(bn(glob, f"{p}.bn_g"))

    for b in range(18):
        yl, yg = ffc(xl, xg, f"{5 + b}.conv1")
        yl, yg = ffc(yl, yg, f"{5 + b}.conv2")
        xl, xg = xl + yl, xg + yg
    x = torch.cat([xl, xg], dim=1)
    for layer in (24, 27, 30):
        x = F.conv_transpose2d(x, s[f"{layer}.weight"], s[f"{layer}.bias"], stride=2, padding=1, output_padding=1)
        x = F.relu(bn(x, str(layer + 1)))
    x = torch.sigmoid(conv(x, s["34.weight"], bias=s["34.bias"]))
    return x[0, :, :height, :width].permute(1, 2, 0).numpy()


def main():
    import torch

    torch.set_num_threads(8)
    sha = hashlib.sha256(W.encode(W.MAGIC["lama"], W.lama_tensors(0))).hexdigest()
    state = torch_state(W.lama_checkpoint(0))
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

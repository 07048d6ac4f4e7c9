#!/usr/bin/env python3
"""Generate the golden fixture that pins the BiRefNet oracle: birefnet_torch.npz.

    python tests/golden/gen_birefnet_golden.py

The reference checks its BiRefNet against the ONNX export of the model
(tools/birefnet/torch_reference.py imports the third-party sources from
Hugging Face, which are not in this container). So this script restates the
published network's forward pass in float64 PyTorch of its own, from the same
seeded weights file the oracle reads (tools/birefnet/export_weights.py folds
every batch norm, so the file's matrices are the layers' weights):

- Swin-T (swin.rs): a 4x4 stride-4 patch embedding, LayerNorm; per block
  LayerNorm, zero padding to a multiple of 7 AFTER the norm, a cyclic shift
  by 3 in odd blocks (torch.roll), 7x7 windows, attention with the given
  relative position bias and, for shifted blocks, the mask the original Swin
  builds from the padded map's nine regions (-100 between regions), the
  reverse shift, the crop, the residual; the MLP with exact GELU; patch
  merging of x[0::2, 0::2], x[1::2, 0::2], x[0::2, 1::2], x[1::2, 1::2];
- the decoder (decoder.rs): torchvision's modulated deformable convolution
  (`deform_conv2d` with mask = 2 sigmoid(logits)) for the ASPP branches, the
  pooling branch as mean, 1x1, ReLU broadcast over the map and concatenated
  (not folded into a bias), bilinear resizes with align_corners=True, image
  patches by reshaping, the gates, and the full-resolution branch as two
  3x3 convolutions (not composed).

This pins the oracle's restatement of what the weights file alone does not
say: window padding and masks, merge order, the deformable sampling rules,
the resize rule, the patch channel order and the head.
"""

from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "image-engine-native_b200"))

from iec import weights as W  # noqa: E402

CASES = [(64, 1), (128, 2)]  # (side, input seed)


def state(tensors):
    import torch

    return {name: torch.from_numpy(np.asarray(a, np.float64)) for name, a, _ in tensors}


def conv_w(m, size):
    """[(ky, kx, cin), cout] -> [cout, cin, ky, kx]."""
    k, cout = m.shape
    cin = k // (size * size)
    return m.reshape(size, size, cin, cout).permute(3, 2, 0, 1).contiguous()


def layer_norm(x, s, name):
    import torch.nn.functional as F

    return F.layer_norm(x, x.shape[-1:], s[f"{name}.weight"], s[f"{name}.bias"], eps=1e-5)


def swin_block(x, s, p, c, shift):
    """x: [H, W, C]."""
    import torch
    import torch.nn.functional as F

    H, Wd, _ = x.shape
    heads = c // 32
    shortcut = x
    h = layer_norm(x, s, f"{p}.norm1")
    Hp, Wp = -(-H // 7) * 7, -(-Wd // 7) * 7
    h = F.pad(h, (0, 0, 0, Wp - Wd, 0, Hp - H))
    if shift:
        h = torch.roll(h, shifts=(-shift, -shift), dims=(0, 1))
    win = h.reshape(Hp // 7, 7, Wp // 7, 7, c).permute(0, 2, 1, 3, 4).reshape(-1, 49, c)
    qkv = win @ s[f"{p}.qkv.weight"] + s[f"{p}.qkv.bias"]
    q, k, v = qkv.split(c, dim=-1)

    def split_heads(t):
        return t.reshape(t.shape[0], 49, heads, 32).permute(0, 2, 1, 3)

    q, k, v = split_heads(q), split_heads(k), split_heads(v)
    att = q @ k.transpose(-1, -2) / np.sqrt(32.0) + s[f"{p}.position_bias"][None]
    if shift:
        img = torch.zeros(Hp, Wp)
        cnt = 0
        for hs in (slice(0, -7), slice(-7, -shift), slice(-shift, None)):
            for ws in (slice(0, -7), slice(-7, -shift), slice(-shift, None)):
                img[hs, ws] = cnt
                cnt += 1
        mw = img.reshape(Hp // 7, 7, Wp // 7, 7).permute(0, 2, 1, 3).reshape(-1, 49)
        mask = (mw[:, None, :] - mw[:, :, None]) != 0
        att = att + (mask.double() * -100.0)[:, None]
    out = torch.softmax(att, dim=-1) @ v
    out = out.permute(0, 2, 1, 3).reshape(-1, 49, c)
    out = out @ s[f"{p}.proj.weight"] + s[f"{p}.proj.bias"]
    out = out.reshape(Hp // 7, Wp // 7, 7, 7, c).permute(0, 2, 1, 3, 4).reshape(Hp, Wp, c)
    if shift:
        out = torch.roll(out, shifts=(shift, shift), dims=(0, 1))
    x = shortcut + out[:H, :Wd]
    h = layer_norm(x, s, f"{p}.norm2")
    h = F.gelu(h @ s[f"{p}.fc1.weight"] + s[f"{p}.fc1.bias"])
    return x + h @ s[f"{p}.fc2.weight"] + s[f"{p}.fc2.bias"]


def backbone(img, s):
    """img: [3, side, side] normalised; returns the four normalised stage maps [H, W, C]."""
    import torch
    import torch.nn.functional as F

    x = F.conv2d(img[None], conv_w(s["patch_embed.weight"], 4), s["patch_embed.bias"], stride=4)[0]
    x = layer_norm(x.permute(1, 2, 0), s, "patch_embed.norm")
    feats = []
    for st, (c, depth) in enumerate(W.BIREFNET_STAGES):
        for b in range(depth):
            x = swin_block(x, s, f"stage{st}.block{b}", c, 3 if b % 2 else 0)
        feats.append(layer_norm(x, s, f"stage{st}.norm"))
        if st < 3:
            m = torch.cat([x[0::2, 0::2], x[1::2, 0::2], x[0::2, 1::2], x[1::2, 1::2]], dim=-1)
            x = layer_norm(m, s, f"stage{st}.merge.norm") @ s[f"stage{st}.merge.weight"]
    return feats


def up(x, size):
    """[C, h, w] -> [C, size, size], bilinear with aligned corners."""
    import torch.nn.functional as F

    return F.interpolate(x[None], size=(size, size), mode="bilinear", align_corners=True)[0]


def conv3(x, s, name, relu=False):
    import torch.nn.functional as F

    y = F.conv2d(x[None], conv_w(s[f"{name}.weight"], 3), s[f"{name}.bias"], padding=1)[0]
    return F.relu(y) if relu else y


def aspp(t, s, p):
    import torch
    import torch.nn.functional as F
    from torchvision.ops import deform_conv2d

    outs = []
    for i, k in enumerate(W.BIREFNET_SIZES):
        b = f"{p}.branch{i}"
        taps = k * k
        om = F.conv2d(t[None], conv_w(s[f"{b}.offset.weight"], k), s[f"{b}.offset.bias"], padding=k // 2)
        offset, mask = om[:, :2 * taps], 2.0 * torch.sigmoid(om[:, 2 * taps:])
        y = deform_conv2d(t[None], offset, conv_w(s[f"{b}.weight"], k), s[f"{b}.bias"], padding=k // 2, mask=mask)
        outs.append(F.relu(y[0]))
    pooled = F.relu(t.mean(dim=(1, 2)) @ s[f"{p}.pool.weight"] + s[f"{p}.pool.bias"])
    outs.append(pooled[:, None, None].expand(-1, t.shape[1], t.shape[2]))
    cat = torch.cat(outs)
    return F.relu(F.conv2d(cat[None], conv_w(s[f"{p}.conv1.weight"], 1), s[f"{p}.conv1.bias"])[0])


def dblock(x, s, p, gate):
    import torch
    import torch.nn.functional as F

    t = conv3(x, s, f"{p}.conv_in", relu=True)
    t = aspp(t, s, f"{p}.aspp")
    out = conv3(t, s, f"{p}.conv_out")
    if gate:
        g = conv3(out, s, f"{p}.gdt", relu=True)
        g = torch.sigmoid(F.conv2d(g[None], conv_w(s[f"{p}.gdt_attn.weight"], 1), s[f"{p}.gdt_attn.bias"])[0])
        out = out * g
    return out


def patches(img, size):
    """image2patches: [3, side, side] -> [3 g g, size, size], channel (c g + gy) g + gx."""
    side = img.shape[1]
    g = side // size
    return img.reshape(3, g, size, g, size).permute(0, 1, 3, 2, 4).reshape(3 * g * g, size, size)


def forward(s, image):
    """image: side x side x 3 normalised (float32 numpy) -> side x side logits."""
    import torch
    import torch.nn.functional as F

    side = image.shape[0]
    img = torch.from_numpy(image.astype(np.float64)).permute(2, 0, 1)
    half = up(img, side // 2)
    full_f = backbone(img, s)
    half_f = backbone(half, s)
    levels = []
    for i in range(4):
        grid = side >> (i + 2)
        f = full_f[i].permute(2, 0, 1)
        h = half_f[i].permute(2, 0, 1)
        levels.append(torch.cat([f, up(h, grid)]))
    g4 = side >> 5
    x4 = torch.cat([up(levels[0], g4), up(levels[1], g4), up(levels[2], g4), levels[3]])
    prev = dblock(x4, s, "squeeze", False)
    for i in range(4):
        level = 3 - i
        grid = side >> (level + 2)
        if i == 0:
            main = prev
        else:
            lat = f"lateral{5 - i}"
            x = levels[level]
            main = F.conv2d(x[None], conv_w(s[f"{lat}.weight"], 1), s[f"{lat}.bias"])[0] + up(prev, grid)
        pn = [5, 4, 3, 2][i]
        pt = patches(img, grid)
        pt = conv3(conv3(pt, s, f"patches{pn}.conv1"), s, f"patches{pn}.conv_out")
        prev = dblock(torch.cat([main, pt]), s, f"block{4 - i}", i < 3)
    low = F.conv2d(prev[None], conv_w(s["head.weight"], 1))[0]
    logits = up(low, side)[0] + s["head.bias"][0]
    fr = conv3(conv3(img, s, "patches1.conv1"), s, "patches1.conv_out")[0]
    return (logits + fr).numpy()


def main():
    import torch

    torch.set_num_threads(8)
    tensors = W.birefnet_tensors(0)
    sha = hashlib.sha256(W.encode(W.MAGIC["birefnet"], tensors)).hexdigest()
    s = state(tensors)
    out = {"weights_sha256": np.array(sha)}
    for i, (side, seed) in enumerate(CASES):
        rgb = W.birefnet_input(side, seed)
        with torch.no_grad():
            logits = forward(s, W.birefnet_normalize(rgb))
        out[f"case{i}_rgb"] = rgb
        out[f"case{i}_logits"] = logits.astype(np.float32)
        print(f"case {i}: side {side}, logits mean {logits.mean():.4f} std {logits.std():.4f}")
    np.savez_compressed(os.path.join(HERE, "birefnet_torch.npz"), **out)


if __name__ == "__main__":
    main()

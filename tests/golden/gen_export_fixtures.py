#!/usr/bin/env python3
"""Pin the weights files of this repository to the reference's own exporters.

    python tests/golden/gen_export_fixtures.py REFERENCE

REFERENCE is a checkout of image-engine-native. For each seeded checkpoint
of iec.weights (realesrgan_checkpoint, scunet_checkpoint, lama_checkpoint:
upstream PyTorch layouts, the names the exporters read), this script saves
the checkpoint as torch.save writes it (wrapped the way each exporter expects
its input), runs the reference's exporter on it
(REFERENCE/tools/<model>/export_weights.py, which needs only numpy and
tools/checkpoint.py), and records the SHA-256 of the file it writes in
export_sha256.json beside this script. It also checks that iec.weights'
restatement of the exporter (export_<model>) gives the same bytes.

tests/test_export_pinning.py then checks, without the reference, that the
restatement still gives those bytes, and that write_<model> (the seeded
files every test and benchmark uses) writes exactly them: every weights file
the backend is tested on is one the reference's exporter writes from a
checkpoint. BiRefNet's exporter reads an ONNX graph through the `onnx`
package, which is not installed here, so its file is not pinned this way.
"""

from __future__ import annotations

import hashlib
import io
import json
import os
import subprocess
import sys
import tempfile
import zipfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "image-engine-native_b200"))

from iec import weights as W  # noqa: E402

OUT = os.path.join(HERE, "export_sha256.json")

# name: (model, checkpoint seed, exporter flags, weak checkpoint seed, strength)
CASES = {
    "realesrgan": ("realesrgan", 0, [], None, None),
    "realesrgan_half": ("realesrgan", 0, ["--half"], None, None),
    "realesrgan_dn_blend": ("realesrgan", 0, [], 1, 0.5),
    "scunet_half": ("scunet", 0, ["--half"], None, None),
    "scunet": ("scunet", 0, [], None, None),
    "lama": ("lama", 0, [], None, None),
    "lama_half": ("lama", 0, ["--half"], None, None),
}


def torch_bytes(obj) -> bytes:
    """`obj` (dicts of numpy arrays) as torch.save writes it."""
    import torch

    def conv(o):
        if isinstance(o, dict):
            return {k: conv(v) for k, v in o.items()}
        return torch.from_numpy(np.ascontiguousarray(o))

    buf = io.BytesIO()
    torch.save(conv(obj), buf)
    return buf.getvalue()


def ours(model, seed, flags, weak_seed, strength) -> bytes:
    half = "--half" in flags
    if model == "realesrgan":
        weak = W.realesrgan_checkpoint(weak_seed) if weak_seed is not None else None
        tensors = W.export_realesrgan(W.realesrgan_checkpoint(seed), weak, strength, half)
    elif model == "scunet":
        tensors = W.export_scunet(W.scunet_checkpoint(seed), half)
    else:
        tensors = W.export_lama(W.lama_checkpoint(seed), half)
    return W.encode(W.MAGIC[model], tensors)


def reference_export(reference, tmp, model, seed, flags, weak_seed, strength) -> bytes:
    tool = os.path.join(reference, "tools", model, "export_weights.py")
    out = os.path.join(tmp, f"{model}.weights")
    args = list(flags)
    if model == "realesrgan":
        # Real-ESRGAN's release files hold "params_ema" (preferred) or
        # "params" (export_weights.py:37-44); the weak file takes the second.
        ckpt = os.path.join(tmp, "model.pth")
        with open(ckpt, "wb") as f:
            f.write(torch_bytes({"params_ema": W.realesrgan_checkpoint(seed)}))
        if weak_seed is not None:
            weak = os.path.join(tmp, "weak.pth")
            with open(weak, "wb") as f:
                f.write(torch_bytes({"params": W.realesrgan_checkpoint(weak_seed)}))
            args += ["--weak", weak, "--strength", str(strength)]
    elif model == "scunet":
        ckpt = os.path.join(tmp, "model.pth")
        with open(ckpt, "wb") as f:
            f.write(torch_bytes(W.scunet_checkpoint(seed)))
    else:
        # big-lama.zip holding big-lama/models/best.ckpt, whose "state_dict"
        # carries the generator under "generator.model." (export_weights.py:
        # 62-72); a discriminator tensor beside it is skipped by the exporter.
        state = {f"generator.model.{k}": v for k, v in W.lama_checkpoint(seed).items()}
        state["discriminator.model.0.weight"] = np.zeros((2, 2), np.float32)
        ckpt = os.path.join(tmp, "big-lama.zip")
        with zipfile.ZipFile(ckpt, "w") as z:
            z.writestr("big-lama/models/best.ckpt", torch_bytes({"state_dict": state}))
    subprocess.run([sys.executable, tool, *args, ckpt, out], check=True, stdout=subprocess.DEVNULL)
    with open(out, "rb") as f:
        return f.read()


def main():
    if len(sys.argv) != 2:
        sys.exit(__doc__.split("\n\n")[1])
    reference = sys.argv[1]
    record = {}
    for name, (model, seed, flags, weak_seed, strength) in CASES.items():
        with tempfile.TemporaryDirectory() as tmp:
            theirs = reference_export(reference, tmp, model, seed, flags, weak_seed, strength)
        mine = ours(model, seed, flags, weak_seed, strength)
        sha = hashlib.sha256(theirs).hexdigest()
        same = mine == theirs
        print(f"{name}: {len(theirs)} bytes, sha256 {sha[:16]}..., restatement {'identical' if same else 'DIFFERS'}")
        if not same:
            sys.exit(f"{name}: iec.weights.export_{model} does not give the reference exporter's bytes")
        record[name] = {"model": model, "seed": seed, "flags": flags, "weak_seed": weak_seed,
                        "strength": strength, "bytes": len(theirs), "sha256": sha,
                        "exporter": f"tools/{model}/export_weights.py"}
    with open(OUT, "w") as f:
        json.dump(record, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()

#!/usr/bin/env python3
"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container that has the reference checkout (read-only), giving its
path as the argument or in IEC_REFERENCE:

    python tests/golden/gen_golden.py REFERENCE

Real-ESRGAN: the reference's own PyTorch definition of SRVGGNetCompact
(tools/realesrgan/torch_reference.py:25-43, the network its CPU path is
tested against in crates/realesrgan-native/tests/reference.rs:61-80) is
imported from the reference checkout, loaded with the seeded random-init
checkpoint iec.weights.realesrgan_checkpoint (PyTorch's [cout, cin, ky, kx]
layout; the weights file the oracle and the backend read is what the
reference's tools/realesrgan/export_weights.py writes from it, byte for
byte) and run on seeded inputs. The outputs, with the inputs and the SHA-256
of the weights file, are written as realesrgan_torch.npz. The reference
itself is never needed at test time.
"""

from __future__ import annotations

import hashlib
import importlib.util
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "image-engine-native_b200"))

from iec import weights as W  # noqa: E402

CASES = [(20, 12, 1), (33, 17, 2)]  # (width, height, input seed)


def load_reference_module(reference: str):
    path = os.path.join(reference, "tools", "realesrgan", "torch_reference.py")
    spec = importlib.util.spec_from_file_location("reference_torch_realesrgan", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def realesrgan(reference: str):
    import torch

    torch.set_num_threads(4)
    mod = load_reference_module(reference)
    data = W.encode(W.MAGIC["realesrgan"], W.realesrgan_tensors(0))
    sha = hashlib.sha256(data).hexdigest()
    # The seeded checkpoint in the upstream layout; the weights file is what
    # the reference's exporter writes from it (tests/test_export_pinning.py).
    state = {name: torch.from_numpy(a) for name, a in W.realesrgan_checkpoint(0).items()}
    model = mod.SRVGGNetCompact()
    model.load_state_dict(state, strict=True)
    model.eval()
    out = {"weights_sha256": np.array(sha)}
    for width, height, seed in CASES:
        image = W.realesrgan_input(width, height, seed)
        x = torch.from_numpy(image.transpose(2, 0, 1)[None].copy())
        with torch.no_grad():
            y = model(x)[0].numpy().transpose(1, 2, 0)
        out[f"input_{width}x{height}"] = image
        out[f"torch_{width}x{height}"] = np.ascontiguousarray(y, np.float32)
    np.savez_compressed(os.path.join(HERE, "realesrgan_torch.npz"), **out)
    print("realesrgan_torch.npz", sha)


def main():
    reference = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("IEC_REFERENCE")
    if not reference:
        sys.exit("usage: gen_golden.py REFERENCE (the reference checkout; or set IEC_REFERENCE)")
    realesrgan(reference)


if __name__ == "__main__":
    main()

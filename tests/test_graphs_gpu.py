"""Model passes replayed as CUDA graphs (GPU tests).

SCUNet, LaMa and BiRefNet passes without progress reports run eagerly the
first time a size and set of buffers is seen, are captured into a graph the
second time and replayed after that. Every run must give the first one's
output bit for bit, and a different size in between must not disturb the
replays (the graph is dropped and rebuilt).
"""

import os

import numpy as np
import pytest

from iec import weights as W

pytestmark = pytest.mark.gpu


def _same(a, b):
    return np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))


def test_scunet_replays_match_the_eager_run(workdir):
    import torch

    import iec

    path = str(workdir / "scunet_graph.weights")
    W.write_scunet(path, 0)
    m = iec.Scunet(path)
    s = torch.cuda.Stream()
    img = torch.from_numpy(W.scunet_input(96, 64, 3)).cuda()
    other = torch.from_numpy(W.scunet_input(64, 32, 4)).cuda()
    outs = []
    for k in range(5):
        if k == 3:  # another size between replays
            o = torch.empty_like(other)
            m.run_device(other.data_ptr(), 64, 32, o.data_ptr(), s.cuda_stream)
        res = torch.empty_like(img)
        m.run_device(img.data_ptr(), 96, 64, res.data_ptr(), s.cuda_stream)
        s.synchronize()
        outs.append(res.cpu().numpy())
    m.close()
    assert all(_same(o, outs[0]) for o in outs[1:])


def test_lama_replays_match_the_eager_run(workdir):
    import torch

    import iec

    path = str(workdir / "lama_graph.weights")
    W.write_lama(path, 0)
    m = iec.Lama(path)
    s = torch.cuda.Stream()
    image, mask = W.lama_input(64, 48, 5)
    ti, tm = torch.from_numpy(image).cuda(), torch.from_numpy(mask).cuda()
    res = torch.empty_like(ti)
    outs = []
    for _ in range(4):
        m.run_device(ti.data_ptr(), tm.data_ptr(), 64, 48, res.data_ptr(), s.cuda_stream)
        s.synchronize()
        outs.append(res.cpu().numpy())
    m.close()
    assert all(_same(o, outs[0]) for o in outs[1:])


def test_birefnet_replays_match_the_eager_run(workdir):
    import torch

    import iec

    path = str(workdir / "birefnet_graph.weights")
    W.write_birefnet(path, 0)
    m = iec.Birefnet(path)
    s = torch.cuda.Stream()
    rgb = torch.from_numpy(W.birefnet_input(128, 6)).cuda()
    res = torch.empty((128, 128), dtype=torch.float32, device="cuda")
    outs = []
    for _ in range(4):
        m.run_device(rgb.data_ptr(), True, 128, res.data_ptr(), s.cuda_stream)
        s.synchronize()
        outs.append(res.cpu().numpy())
    # The host entry point (its own staging buffers) repeats too.
    host = [m.run(W.birefnet_input(128, 6)) for _ in range(3)]
    m.close()
    assert all(_same(o, outs[0]) for o in outs[1:])
    assert all(_same(h, outs[0]) for h in host)


def test_launch_timing_records_an_eager_pass_with_the_same_output(workdir):
    """iec_set_launch_timing: the pass runs eagerly with events around every
    instrumented launch; its output equals the graph replay's bit for bit and
    every record has a duration and algorithmic work."""
    import torch

    import iec

    path = str(workdir / "scunet_timing.weights")
    W.write_scunet(path, 0)
    m = iec.Scunet(path)
    s = torch.cuda.Stream()
    img = torch.from_numpy(W.scunet_input(96, 64, 5)).cuda()
    try:
        want = None
        for _ in range(3):  # eager, captured, replayed
            want = torch.empty_like(img)
            m.run_device(img.data_ptr(), 96, 64, want.data_ptr(), s.cuda_stream)
        iec.set_launch_timing(m, True)
        got = torch.empty_like(img)
        m.run_device(img.data_ptr(), 96, 64, got.data_ptr(), s.cuda_stream)
        s.synchronize()
        recs = iec.launch_timing(m)
        iec.set_launch_timing(m, False)
        assert _same(got.cpu().numpy(), want.cpu().numpy())
        names = {r["name"].split(" ")[0] for r in recs}
        assert any(n.startswith("igemm_sm100") for n in names)
        assert {"layer_norm_rows", "window_attention_kernel"} <= names
        assert all(r["ms"] > 0 and (r["flop"] > 0 or r["bytes"] > 0) for r in recs)
        assert iec.launch_timing(m) == []  # off: a new, empty record
    finally:
        m.close()

#!/usr/bin/env python3
"""Benchmark of the CUDA backend: output megapixels/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Workload (the sharded-batch configuration): a batch of 256 independent 3 x 256 x 384
Real-ESRGAN inputs (seeded, uniform in [0, 1)), seeded random-init weights,
split evenly across the N ranks (one process per GPU, no collective on the
data path: the batch shards by image). One step = the whole batch once.
value = 256 x 1.5729 output MP / step time (device time, max over ranks).

Printed as one JSON line by rank 0:
  value      inputs resident in HBM (302 MB in, 4.8 GB out: larger than L2),
             CUDA events on the stream the kernels run on;
  e2e        the same through the C ABI's host-buffer entry points from
             page-locked memory, the H2D and D2H copies inside the timed
             region: 8-bit images (iec_realesrgan_run_batch_u8, Model::run's
             semantics) as the value, f32 ones (iec_realesrgan_run_batch) in
             e2e.f32;
  roofline   the dominant kernel (conv3x3 64->64, 32 of 34 layers): its
             algorithmic FLOPs per launch over its mean launch time, both
             measured by events around each launch during the timed steps;
  cpu_baseline  the CPU oracle (a restatement of the reference's CPU f32
             path) on the host's cores, rank 0 at N = 1, a bounded sample.
`--impl reference` times that CPU path alone (rank 0; the others exit).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "image-engine-native_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

BATCH, WIDTH, HEIGHT = 256, 384, 256
OUT_MP = WIDTH * HEIGHT * 16 / 1e6  # 1.572864 output MP per image
# Algorithmic work of one 64 -> 64 3x3 convolution per pixel (2 FLOP / MAC).
CONV64_FLOP_PER_PX = 2 * 9 * 64 * 64
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except (OSError, ValueError):
        return FALLBACK_PEAKS, "fallback"


def traffic_per_px(name="conv3x3_64x64_realesrgan.txt"):
    """DRAM bytes per output pixel of one 64->64 layer from a committed ncu
    summary under profiles/ (the per-layer kernel's, or the fused body's), or
    None."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("dram_bytes_per_pixel:"):
                    return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


class Clocks:
    """nvidia-smi samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", ",".join(str(g) for g in self.gpus)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) >= 9:
                        rows.append(parts)
            os.unlink(self.path)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = max((num(r[2]) or 0) for r in rows)
        power = [num(r[3]) or 0 for r in rows]
        loaded = [s for s, p in zip(sm, power) if p > 0.4 * max(power)] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows), "power_w_max": max(power)}


def host_threads():
    """Threads the CPU path may use: every core of this process's affinity
    mask, whatever OMP_NUM_THREADS a launcher such as torchrun has set."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def oracle_threads(n):
    from oracle import refcpu

    refcpu.set_threads(n)
    return refcpu.threads()


def cpu_sample(weights_path, seconds=12.0, cap=30.0, six_seconds=8.0):
    """The CPU oracle on whole 3x256x384 images until `seconds` have passed,
    on every core of the affinity mask; then the same with 6 threads (the
    reference's published protocol times 6 threads, README.md:26-27)."""
    from iec import weights as W
    from oracle import refcpu

    model = refcpu.RealEsrgan(weights_path)
    image = W.realesrgan_input(WIDTH, HEIGHT, 0)

    def timed(threads, secs):
        cores = oracle_threads(threads)
        model.run_float(image[:32, :32])  # warm-up of the threads
        n, t0 = 0, time.perf_counter()
        while True:
            model.run_float(image)
            n += 1
            el = time.perf_counter() - t0
            if el >= secs or el + el / n > cap:
                return n, el, cores

    n, el, cores = timed(host_threads(), seconds)
    out = {"value": n * OUT_MP / el, "unit": "MP/s", "cores": cores, "kind": "port",
           "sample": f"{n} whole 3x256x384 images of the batch, {el:.1f} s, oracle/refcpu (restated reference CPU f32 path: Winograd F(4x4) + FMA products), {cores} threads (the affinity mask)"}
    n6, el6, c6 = timed(min(6, host_threads()), six_seconds)
    out["six_threads"] = {"value": n6 * OUT_MP / el6, "unit": "MP/s", "cores": c6,
                          "sample": f"{n6} whole images, {el6:.1f} s"}
    oracle_threads(host_threads())
    return out


def reference_arm(args, weights_path):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from iec import weights as W
    from oracle import refcpu

    oracle_threads(host_threads())
    model = refcpu.RealEsrgan(weights_path)
    image = W.realesrgan_input(WIDTH, HEIGHT, 0)
    for _ in range(args.warmup):
        model.run_float(image)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        model.run_float(image)
    el = time.perf_counter() - t0
    value = args.steps * OUT_MP / el
    cores = refcpu.threads()
    line = {
        "impl": "reference", "metric": "output megapixels/s", "value": value, "unit": "MP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config(args, args.chunk),
        "cpu_baseline": {"value": value, "unit": "MP/s", "cores": cores, "kind": "port",
                         "sample": f"one 3x256x384 image of the batch per step, oracle/refcpu (the reference CPU f32 path restated; the Rust reference cannot be built here), {cores} threads"},
        "e2e": {"value": value, "unit": "MP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def time_device(fn, stream, warmup=3, iters=10):
    """Mean seconds per call of `fn` (queued on `stream`), by CUDA events."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(iters):
        fn()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / 1e3 / iters


def other_models(wdir, stream, sptr, args):
    """SCUNet 3x512x768, Big LaMa 4x512x512 and BiRefNet-lite 3x1024x1024
    (seeded weights), device-resident; LaMa and BiRefNet also through their
    host entry points; with the CPU oracle's time for one run beside each."""
    out = {}
    only = set(args.models.split(","))
    cpu = not args.no_cpu and not args.profile_models
    if "scunet" in only:
        out.update(scunet_leg(wdir, stream, sptr, cpu))
    if "lama" in only:
        out.update(lama_leg(wdir, stream, sptr, cpu))
    if "birefnet" in only:
        out.update(birefnet_leg(wdir, stream, sptr, cpu))
    return out


def cpu_once(fn, mp):
    """The CPU oracle's time for one run of a model's configuration (after a
    small warm-up of its threads): the per-model CPU baseline."""
    from oracle import refcpu

    oracle_threads(host_threads())
    t0 = time.perf_counter()
    fn()
    el = time.perf_counter() - t0
    cores = refcpu.threads()
    return {"value": mp / el, "unit": "MP/s", "seconds": el, "cores": cores, "kind": "port"}


def launch_table(model, run, pk):
    """One eager pass of `run` with launch timing on (iec_set_launch_timing:
    CUDA events around each instrumented launch, the pass's side-stream work
    serialised onto its stream so each pair times one kernel alone), summarised:
    the dominant GEMM shape by total time against its own roofline (tensor
    when its algorithmic FLOPs per algorithmic byte reach the ridge point of
    the sustained dense peak over the measured copy rate, else HBM), all GEMM
    launches together (the time they would take at their rooflines over the
    time they took), and achieved GB/s of the bandwidth-bound kernels
    (algorithmic bytes over event time, against the measured copy rate)."""
    import torch

    import iec

    iec.set_launch_timing(model, True)
    run()
    torch.cuda.synchronize()
    recs = iec.launch_timing(model)
    iec.set_launch_timing(model, False)
    peak = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    hbm = pk["hbm_gbs"]
    ridge = peak * 1e12 / (hbm * 1e9)  # FLOP per byte

    def bound(g):
        """(bound, achieved, unit, frac, frac_tensor, frac_hbm) of one GEMM group."""
        sec = g["ms"] / 1e3
        tf = g["flop"] / sec / 1e12
        gbs = g["bytes"] / sec / 1e9
        if g["bytes"] > 0 and g["flop"] / g["bytes"] < ridge:
            return "hbm", gbs, "GB/s", gbs / hbm, tf / peak, gbs / hbm
        return "tensor", tf, "TFLOP/s", tf / peak, tf / peak, gbs / hbm

    groups = {}
    for r in recs:
        g = groups.setdefault(r["name"], {"launches": 0, "ms": 0.0, "flop": 0.0, "bytes": 0.0})
        g["launches"] += 1
        g["ms"] += r["ms"]
        g["flop"] += r["flop"]
        g["bytes"] += r["bytes"]
    gemms = {k: v for k, v in groups.items() if k.startswith("igemm_sm100")}
    out = {"launches_timed": len(recs), "ms_sum": sum(r["ms"] for r in recs)}
    if gemms:
        name, g = max(gemms.items(), key=lambda kv: kv[1]["ms"])
        b, ach, unit, frac, ft, fh = bound(g)
        out["roofline"] = {"kernel": name + " (A x W: M x N x K)", "bound": b, "launches": g["launches"],
                           "mean_launch_ms": g["ms"] / g["launches"], "flop_per_launch": g["flop"] / g["launches"],
                           "bytes_per_launch": g["bytes"] / g["launches"],
                           "flop_per_byte": g["flop"] / g["bytes"] if g["bytes"] else None, "ridge_flop_per_byte": ridge,
                           "achieved": ach, "peak": hbm if b == "hbm" else peak, "unit": unit, "frac": frac,
                           "frac_of_tensor_peak": ft, "frac_of_hbm": fh, "share_of_timed": g["ms"] / out["ms_sum"]}
        fl = sum(v["flop"] for v in gemms.values())
        ms = sum(v["ms"] for v in gemms.values())
        at_roof = sum(max(v["flop"] / (peak * 1e12), v["bytes"] / (hbm * 1e9)) for v in gemms.values()) * 1e3
        out["all_gemms"] = {"launches": sum(v["launches"] for v in gemms.values()), "ms": ms,
                            "achieved_tflops": fl / (ms / 1e3) / 1e12, "frac": fl / (ms / 1e3) / 1e12 / peak,
                            "roofline_ms": at_roof, "frac_of_roofline": at_roof / ms}
        top = sorted(gemms.items(), key=lambda kv: -kv[1]["ms"])[:6]
        out["top_gemms"] = []
        for k, v in top:
            b, ach, unit, frac, ft, fh = bound(v)
            out["top_gemms"].append({"kernel": k, "launches": v["launches"], "mean_ms": v["ms"] / v["launches"],
                                     "tflops": v["flop"] / (v["ms"] / 1e3) / 1e12, "bound": b,
                                     "achieved": ach, "unit": unit, "frac": frac})
    bw = {}
    for k, v in groups.items():
        if k.startswith("igemm_sm100") or v["bytes"] <= 0:
            continue
        gbs = v["bytes"] / (v["ms"] / 1e3) / 1e9
        bw[k] = {"launches": v["launches"], "mean_ms": v["ms"] / v["launches"], "gbs": gbs,
                 "frac_hbm": gbs / pk["hbm_gbs"], "share_of_timed": v["ms"] / out["ms_sum"]}
    out["bandwidth_kernels"] = bw
    return out


def scunet_leg(wdir, stream, sptr, cpu):
    import torch

    import iec
    from iec import weights as W

    out = {}
    path = os.path.join(wdir, "scunet.weights")
    W.write_scunet(path, 0)
    m = iec.Scunet(path, device=torch.cuda.current_device())
    img = torch.from_numpy(W.scunet_input(768, 512, 0)).cuda()
    res = torch.empty_like(img)
    t = time_device(lambda: m.run_device(img.data_ptr(), 768, 512, res.data_ptr(), sptr), stream)
    table = launch_table(m, lambda: m.run_device(img.data_ptr(), 768, 512, res.data_ptr(), sptr), peaks()[0])
    image = W.scunet_input(768, 512, 0)
    for _ in range(3):  # warm-up: buffers, then the pass's graph (captured on the second call)
        m.run_float(image)
    t0 = time.perf_counter()
    for _ in range(5):
        m.run_float(image)
    te = (time.perf_counter() - t0) / 5
    out["scunet_768x512"] = {"workload": "SCUNet 3x512x768 (single-image configuration)", "value": 768 * 512 / 1e6 / t,
                             "unit": "MP/s", "ms": t * 1e3, "gflop": 899.58,
                             "tflops_achieved": 899.58e9 / t / 1e12, "e2e_ms": te * 1e3,
                             "e2e_value": 768 * 512 / 1e6 / te, **table}
    m.close()
    if cpu:
        from oracle import refcpu

        ref = refcpu.Scunet(path)
        ref.run_float(image[:64, :64])
        out["scunet_768x512"]["cpu_baseline"] = cpu_once(lambda: ref.run_float(image), 768 * 512 / 1e6)
    return out


def lama_leg(wdir, stream, sptr, cpu):
    """Big LaMa 512 x 512, about 30 % masked (seeded f16 weights and rectangles)."""
    import torch

    import iec
    from iec import weights as W

    out = {}
    path = os.path.join(wdir, "lama.weights")
    W.write_lama(path, 0)
    m = iec.Lama(path, device=torch.cuda.current_device())
    image, mask = W.lama_input(512, 512, 0)
    img = torch.from_numpy(image).cuda()
    msk = torch.from_numpy(mask).cuda()
    res = torch.empty_like(img)
    t = time_device(lambda: m.run_device(img.data_ptr(), msk.data_ptr(), 512, 512, res.data_ptr(), sptr), stream)
    table = launch_table(m, lambda: m.run_device(img.data_ptr(), msk.data_ptr(), 512, 512, res.data_ptr(), sptr),
                         peaks()[0])
    for _ in range(3):  # warm-up: buffers, then the pass's graph (captured on the second call)
        m.run_float(image, mask)
    t0 = time.perf_counter()
    for _ in range(5):
        m.run_float(image, mask)
    te = (time.perf_counter() - t0) / 5
    out["lama_512x512"] = {"workload": "Big LaMa 4x512x512 (single-image configuration)", "value": 512 * 512 / 1e6 / t,
                           "unit": "MP/s", "ms": t * 1e3, "gflop": 439.8, "tflops_achieved": 439.8e9 / t / 1e12,
                           "e2e_ms": te * 1e3, "e2e_value": 512 * 512 / 1e6 / te, **table}
    m.close()
    if cpu:
        from oracle import refcpu

        ref = refcpu.Lama(path)
        ref.run_float(image[:16, :16], mask[:16, :16])
        out["lama_512x512"]["cpu_baseline"] = cpu_once(lambda: ref.run_float(image, mask), 512 * 512 / 1e6)
    return out


def birefnet_leg(wdir, stream, sptr, cpu):
    """BiRefNet-lite at side 1024 (seeded f16 weights, uniform 8-bit image):
    device-resident, and through the host entry point."""
    import torch

    import iec
    from iec import weights as W

    out = {}
    path = os.path.join(wdir, "birefnet.weights")
    W.write_birefnet(path, 0)
    m = iec.Birefnet(path, device=torch.cuda.current_device())
    rgb = W.birefnet_input(1024, 0)
    img = torch.from_numpy(rgb).cuda()
    res = torch.empty((1024, 1024), dtype=torch.float32, device="cuda")
    t = time_device(lambda: m.run_device(img.data_ptr(), True, 1024, res.data_ptr(), sptr), stream)
    table = launch_table(m, lambda: m.run_device(img.data_ptr(), True, 1024, res.data_ptr(), sptr), peaks()[0])
    for _ in range(3):  # warm-up: buffers, then the pass's graph (captured on the second call)
        m.run(rgb)
    t0 = time.perf_counter()
    for _ in range(3):
        m.run(rgb)
    te = (time.perf_counter() - t0) / 3
    out["birefnet_1024"] = {"workload": "BiRefNet-lite 3x1024x1024 (single-image configuration)",
                            "value": 1024 * 1024 / 1e6 / t, "unit": "MP/s", "ms": t * 1e3, "gflop": 606.36,
                            "tflops_achieved": 606.36e9 / t / 1e12, "e2e_ms": te * 1e3,
                            "e2e_value": 1024 * 1024 / 1e6 / te, **table}
    m.close()
    if cpu:
        from oracle import refcpu

        ref = refcpu.Birefnet(path)
        ref.run(rgb[:64, :64])
        out["birefnet_1024"]["cpu_baseline"] = cpu_once(lambda: ref.run(rgb), 1024 * 1024 / 1e6)
    return out


def config(args, chunk):
    return {"workload": f"realesrgan_x4v3 batch of {args.batch} x 3x256x384 (sharded batch), split by image",
            "model": "Real-ESRGAN general-x4v3 (SRVGGNetCompact, 34 conv3x3), seeded random-init weights",
            "global_batch": args.batch, "image": f"{WIDTH}x{HEIGHT}", "images_per_launch": chunk,
            "parallelism": f"dp{args.gpus} (by image, no collective)",
            "l2": "inputs 302 MB and outputs 4.8 GB exceed the 126 MB L2; no flush"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--chunk", type=int, default=8, help="images per launch")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer measurement")
    ap.add_argument("--no-tiles", action="store_true", help="skip the large-image tiles leg")
    ap.add_argument("--no-models", action="store_true", help="skip the other models' single-image legs")
    ap.add_argument("--profile-models", action="store_true",
                    help="run only the other models' single-image legs (for profiler launch lists)")
    ap.add_argument("--models", default="scunet,lama,birefnet", help="which single-image legs run (comma list)")
    ap.add_argument("--warm-seconds", type=float, default=3.0,
                    help="minimum seconds of warm-up work before the timed steps (power-capped steady state)")
    ap.add_argument("--batch", type=int, default=BATCH,
                    help="images per step (a smaller batch only for profiling captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup

    from iec import weights as W

    wdir = tempfile.mkdtemp()
    weights_path = os.path.join(wdir, "realesrgan.weights")
    W.write_realesrgan(weights_path, 0)

    if args.impl == "reference":
        reference_arm(args, weights_path)
        return

    import numpy as np
    import torch

    import iec

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    batch = args.batch
    assert batch % world == 0
    count = batch // world

    if args.profile_models:
        stream = torch.cuda.Stream()
        print(json.dumps(other_models(wdir, stream, stream.cuda_stream, args)), flush=True)
        return

    model = iec.RealEsrgan(weights_path, device=local, batch_chunk=args.chunk)
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    d_in = torch.rand((count, HEIGHT, WIDTH, 3), generator=gen, device="cuda", dtype=torch.float32)
    d_out = torch.empty((count, HEIGHT * 4, WIDTH * 4, 3), device="cuda", dtype=torch.float32)
    stream = torch.cuda.Stream()
    sptr = stream.cuda_stream

    def step():
        model.run_device(d_in.data_ptr(), count, WIDTH, HEIGHT, d_out.data_ptr(), sptr)

    def barrier():
        if dist:
            dist.barrier()

    def max_over_ranks(x):
        if not dist:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # Warm-up: at least W steps and at least --warm-seconds of work, so every
    # GPU is at its power-capped steady state (clock and power) when the
    # timed region starts, whatever N makes one step's length.
    warm_steps, w0 = 0, time.perf_counter()
    while warm_steps < args.warmup or time.perf_counter() - w0 < args.warm_seconds:
        step()
        warm_steps += 1
        if warm_steps >= args.warmup:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    launches_per_step = model.launches(count, WIDTH, HEIGHT)
    model.set_timing(args.steps * launches_per_step * 2 + 64)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with Clocks([local] if world == 1 else list(range(world))) as clk:
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    elapsed = max_over_ranks(start.elapsed_time(end) / 1e3)
    kinds, ms = model.timing(args.steps * launches_per_step * 2 + 64)
    model.set_timing(0)
    # The dominant kernel: the fused 32-layer body launch (kind 4) where the
    # passes take it, else the per-layer 64->64 convolution (kind 2).
    if (kinds == 4).any():
        conv_ms, conv_layers = float(ms[kinds == 4].mean()), 32
        conv_kernel = "conv3x3_body_sm100 (the 32 64->64 PReLU layers, one persistent launch)"
        conv_profile = "conv3x3_body_realesrgan.txt"
    else:
        conv_ms, conv_layers = (float(ms[kinds == 2].mean()) if (kinds == 2).any() else None), 1
        conv_kernel = "conv3x3_sm100<64,64,PRELU>"
        conv_profile = "conv3x3_64x64_realesrgan.txt"
    step_s = elapsed / args.steps
    value = batch * OUT_MP / step_s

    e2e = None
    if not args.no_e2e:
        # End to end through the host-buffer entry points, page-locked
        # buffers, every step's H2D copy of its inputs and D2H copy of its
        # outputs inside the timed region: 8-bit images (Model::run, the
        # reference's public byte API) and f32 ones (Model::run_float).
        e2e_steps = max(2, args.steps // 2)

        def host_leg(run, h_in, h_out):
            run(h_in, h_out, sptr)
            barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(e2e_steps):
                run(h_in, h_out, sptr)
            e1.record(stream)
            torch.cuda.synchronize()
            barrier()
            sec = max_over_ranks(e0.elapsed_time(e1) / 1e3) / e2e_steps
            bi = batch * WIDTH * HEIGHT * 3 * h_in.element_size()
            bo = batch * WIDTH * HEIGHT * 3 * 16 * h_out.element_size()
            return {"value": batch * OUT_MP / sec, "unit": "MP/s", "h2d_bytes_per_step": bi,
                    "d2h_bytes_per_step": bo, "ms_per_step": sec * 1e3,
                    "d2h_gbs_aggregate": bo / sec / 1e9}

        h_in = torch.empty((count, HEIGHT, WIDTH, 3), dtype=torch.float32, pin_memory=True)
        h_in.copy_(d_in)
        h_out = torch.empty((count, HEIGHT * 4, WIDTH * 4, 3), dtype=torch.float32, pin_memory=True)
        f32 = host_leg(model.run_batch, h_in, h_out)
        # The host path gives the device path's numbers bit for bit.
        f32["matches_device_path"] = bool(torch.equal(h_out[:2].cuda(), d_out[:2]))
        f32["api"] = "iec_realesrgan_run_batch (f32 host buffers, page-locked)"
        del h_out
        b_in = torch.empty((count, HEIGHT, WIDTH, 3), dtype=torch.uint8, pin_memory=True)
        b_in.copy_((d_in * 255).round().to(torch.uint8))
        b_out = torch.empty((count, HEIGHT * 4, WIDTH * 4, 3), dtype=torch.uint8, pin_memory=True)
        e2e = host_leg(model.run_batch_u8, b_in, b_out)
        e2e["api"] = "iec_realesrgan_run_batch_u8 (8-bit host buffers, page-locked: Model::run semantics)"
        e2e["f32"] = f32
        del b_in, b_out, h_in

    # The other sharded workload: one 3x4096x4096 image cut into 512 x 512
    # tiles with a 34-pixel margin; each rank runs its cost-balanced range of
    # the 64 tiles (device-resident input and output, no gather in the timed
    # region). Same max-over-ranks device timing.
    tiles_leg = None
    if not args.no_tiles:
        from iec import shard

        TW, TILE, MARGIN = 4096, 512, 34
        grid = shard.tile_grid(TW, TW, TILE, MARGIN)
        first, last = shard.split_ranges([t.cost for t in grid], world)[rank]
        g2 = torch.Generator(device="cuda").manual_seed(4321)
        big_in = torch.rand((TW, TW, 3), generator=g2, device="cuda", dtype=torch.float32)
        big_out = torch.empty((4 * TW, 4 * TW, 3), device="cuda", dtype=torch.float32)

        def tiles_step():
            model.run_tiles_device(big_in.data_ptr(), TW, TW, TILE, MARGIN, first, last, big_out.data_ptr(), sptr)

        tiles_step()
        torch.cuda.synchronize()
        barrier()
        t_a, t_b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        tiles_steps = max(2, args.steps // 2)
        t_a.record(stream)
        for _ in range(tiles_steps):
            tiles_step()
        t_b.record(stream)
        torch.cuda.synchronize()
        barrier()
        t_s = max_over_ranks(t_a.elapsed_time(t_b) / 1e3) / tiles_steps
        tiles_leg = {"workload": "realesrgan_x4v3 one 3x4096x4096 image, 64 tiles of 512 + 34 margin, split by tile",
                     "value": TW * TW * 16 / 1e6 / t_s, "unit": "MP/s", "ms_per_step": t_s * 1e3,
                     "steps": tiles_steps, "tiles_rank0": [first, last],
                     "computed_over_algorithmic_px": sum(t.cost for t in grid) / (TW * TW)}
        if world > 1:
            # Reassembly on rank 0 over NCCL (each rank's band of output rows,
            # point to point, device to device), timed as the max over ranks,
            # then checked bit for bit against rank 0's own run of all 64 tiles.
            ranges = shard.split_ranges([t.cost for t in grid], world)
            shard.gather_bands(big_out, grid, ranges, rank, world, dist)  # warm: NCCL sets up its P2P links
            barrier()
            torch.cuda.synchronize()
            g0 = time.perf_counter()
            shard.gather_bands(big_out, grid, ranges, rank, world, dist)
            torch.cuda.synchronize()
            g_s = max_over_ranks(time.perf_counter() - g0)
            barrier()
            equal = None
            if rank == 0:
                ref = torch.empty_like(big_out)
                model.run_tiles_device(big_in.data_ptr(), TW, TW, TILE, MARGIN, 0, len(grid), ref.data_ptr(), sptr)
                torch.cuda.synchronize()
                equal = bool(torch.equal(big_out.view(torch.int32), ref.view(torch.int32)))
                del ref
            barrier()
            tiles_leg.update({"gather_ms": g_s * 1e3, "gather": "NCCL point-to-point bands of output rows to rank 0 (second gather; the first sets up the links)",
                              "reassembled_bit_equal": equal})
        del big_in, big_out

    # One image (the single-image configuration) on one GPU, device-resident.
    single = None
    if rank == 0 and world == 1:
        s_out = torch.empty((1, HEIGHT * 4, WIDTH * 4, 3), device="cuda", dtype=torch.float32)
        for _ in range(3):
            model.run_device(d_in.data_ptr(), 1, WIDTH, HEIGHT, s_out.data_ptr(), sptr)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record(stream)
        for _ in range(20):
            model.run_device(d_in.data_ptr(), 1, WIDTH, HEIGHT, s_out.data_ptr(), sptr)
        b.record(stream)
        torch.cuda.synchronize()
        t1 = a.elapsed_time(b) / 1e3 / 20
        single = {"workload": "realesrgan_x4v3 one 3x256x384 image (single-image configuration)", "value": OUT_MP / t1,
                  "unit": "MP/s", "ms": t1 * 1e3}

    # The other models' single-image configurations on one GPU (rank 0 at
    # N = 1), device-resident, CUDA events on the launch stream.
    per_model_extra = {}
    if rank == 0 and world == 1 and not args.no_models:
        per_model_extra.update(other_models(wdir, stream, sptr, args))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_sample(weights_path)

    if rank == 0:
        pk, src = peaks()
        peak = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
        px_per_launch = args.chunk * WIDTH * HEIGHT
        flop_per_launch = CONV64_FLOP_PER_PX * px_per_launch * conv_layers
        achieved = flop_per_launch / (conv_ms / 1e3) / 1e12 if conv_ms else None
        tpp = traffic_per_px(conv_profile)
        clocks = clk.summary()
        line = {
            "metric": "output megapixels/s", "value": value, "unit": "MP/s", "n_gpus": world,
            "steps": args.steps, "warmup": warm_steps, "ms_per_step": step_s * 1e3, "higher_is_better": True,
            "warmup_floor_s": args.warm_seconds,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16 (f32 accumulate)",
            "data": "synthetic (seeded uniform images, seeded He-normal weights)",
            "config": config(args, args.chunk),
            "e2e": e2e,
            "roofline": {"kernel": conv_kernel, "bound": "tensor", "achieved": achieved,
                         "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak if achieved else None,
                         "peak_source": f"{src} bf16 dense (sustained; f16 rate is the same)",
                         "mean_launch_ms": conv_ms, "layers_per_launch": conv_layers,
                         "flop_per_launch": flop_per_launch,
                         "traffic": tpp * px_per_launch * conv_layers if tpp else None,
                         "algorithmic_bytes_per_launch": px_per_launch * 64 * 2 * 2 * conv_layers},
            "cpu_baseline": cpu,
            "gpu_launches": launches_per_step * args.steps * world,
            "clocks": clocks,
            "sharded_tiles": tiles_leg,
            "per_model": {"realesrgan_single_image": single, **per_model_extra},
        }
        print(json.dumps(line), flush=True)
    model.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

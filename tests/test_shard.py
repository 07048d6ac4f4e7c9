"""Host-side sharding: the tile grid, the cost-balanced split, and a
world-size-2 run over gloo on the CPU in which each rank computes its range
of tiles and rank 0 stitches the gathered windows. The per-rank engine here
is the CPU oracle; on GPUs the same split drives iec_realesrgan_run_float_tiles.
"""

import os
import socket

import numpy as np
import pytest

from iec import shard
from iec import weights as W


def test_grid_matches_the_reference_rule():
    # lib.rs:241-289: equal tiles over a ceil(width / tile) x ceil(height / tile)
    # grid, margins clipped at the image.
    tiles = shard.tile_grid(70, 45, 24, 34)
    assert len(tiles) == 3 * 2
    assert [(t.x0, t.x1) for t in tiles[:3]] == [(0, 23), (23, 46), (46, 70)]
    assert [(t.y0, t.y1) for t in tiles[::3]] == [(0, 22), (22, 45)]
    assert tiles[4].rx0 == 0 and tiles[4].rx1 == 70 and tiles[4].ry0 == 0 and tiles[4].ry1 == 45
    big = shard.tile_grid(4096, 4096, 512, 34)
    assert len(big) == 64
    assert max(t.rx1 - t.rx0 for t in big) == 580


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_split_covers_every_tile_once_and_balances(world):
    tiles = shard.tile_grid(4096, 4096, 512, 34)
    ranges = shard.split_ranges([t.cost for t in tiles], world)
    assert len(ranges) == world
    assert ranges[0][0] == 0 and ranges[-1][1] == len(tiles)
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    loads = [sum(t.cost for t in tiles[a:b]) for a, b in ranges]
    assert max(loads) <= 1.25 * sum(loads) / world


def test_split_batch():
    assert shard.split_batch(256, 8) == [(32 * r, 32 * (r + 1)) for r in range(8)]
    assert shard.split_batch(5, 2) == [(0, 2), (2, 5)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, weights, result_path):
    import torch.distributed as dist

    from oracle import refcpu

    refcpu.set_threads(2)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = refcpu.RealEsrgan(weights)
        image = W.realesrgan_input(70, 45, 9)
        tiles = shard.tile_grid(70, 45, 24, 34)
        first, last = shard.split_ranges([t.cost for t in tiles], world)[rank]
        local = []
        for t in tiles[first:last]:
            region = image[t.ry0:t.ry1, t.rx0:t.rx1]
            out = model.run_float(region)
            kx0, ky0 = 4 * (t.x0 - t.rx0), 4 * (t.y0 - t.ry0)
            local.append((t.index, out[ky0:ky0 + 4 * (t.y1 - t.y0), kx0:kx0 + 4 * (t.x1 - t.x0)].copy()))
        gathered = shard.gather_windows(local, rank, world, dist)
        if rank == 0:
            full = shard.stitch(np.zeros((180, 280, 3), np.float32), tiles, gathered)
            np.save(result_path, full)
    finally:
        dist.destroy_process_group()


def test_two_ranks_over_gloo_reassemble_the_tiled_run(realesrgan_weights, tmp_path):
    import torch.multiprocessing as mp

    from oracle import refcpu

    result = str(tmp_path / "stitched.npy")
    mp.start_processes(_rank, args=(2, _free_port(), realesrgan_weights, result), nprocs=2, join=True,
                       start_method="spawn")
    stitched = np.load(result)
    image = W.realesrgan_input(70, 45, 9)
    model = refcpu.RealEsrgan(realesrgan_weights)
    tiled = model.run_float_tiled(image, 24, 34)
    assert np.array_equal(stitched.view(np.uint32), tiled.view(np.uint32))
    whole = model.run_float(image)
    assert np.abs(stitched - whole).max() < 1e-4


def _band_rank(rank, world, port, result_path):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tiles = shard.tile_grid(70, 45, 24, 34)
        ranges = shard.split_ranges([t.cost for t in tiles], world)
        first, last = ranges[rank]
        out = torch.full((180, 280, 3), -1.0)
        for t in tiles[first:last]:  # this rank's windows: the tile's index as the value
            out[4 * t.y0:4 * t.y1, 4 * t.x0:4 * t.x1] = float(t.index)
        shard.gather_bands(out, tiles, ranges, rank, world, dist)
        if rank == 0:
            np.save(result_path, out.numpy())
    finally:
        dist.destroy_process_group()


def test_bands_gathered_point_to_point_reassemble_every_window(tmp_path):
    """shard.gather_bands (device tensors on GPUs, here CPU tensors over
    gloo): three ranks whose tile ranges split a row of tiles; rank 0 ends
    with every tile's window and nothing else overwritten."""
    import torch.multiprocessing as mp

    result = str(tmp_path / "bands.npy")
    mp.start_processes(_band_rank, args=(3, _free_port(), result), nprocs=3, join=True, start_method="spawn")
    out = np.load(result)
    tiles = shard.tile_grid(70, 45, 24, 34)
    want = np.full((180, 280, 3), -1.0, np.float32)
    for t in tiles:
        want[4 * t.y0:4 * t.y1, 4 * t.x0:4 * t.x1] = t.index
    assert np.array_equal(out, want)
    ranges = shard.split_ranges([t.cost for t in tiles], 3)
    assert any(ranges[r][0] % 3 for r in range(1, 3))  # a range starts inside a tile row

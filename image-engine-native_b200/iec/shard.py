"""Sharding Real-ESRGAN work over the GPUs of one box, one process per GPU.

Both sharded workloads split without any exchange step:
  * a batch of images: each rank runs a contiguous slice of the batch;
  * one large image: the grid of tiles Model::run_float_tiled cuts
    (crates/realesrgan-native/src/lib.rs:241-289: equal tiles, each run with
    `margin` pixels of context, only its own window kept) is split into
    contiguous ranges of tiles balanced by the pixels each tile computes (its
    region with the margin); each rank runs its range with
    iec_realesrgan_run_float_tiles / run_tiles_device, which write only their
    tiles' windows, and the windows are gathered to rank 0.
Every tile's pixels come out exactly as in the single-GPU run_float_tiled,
whichever rank computes it. Ranks talk only through torch.distributed (NCCL
on GPUs, gloo on CPU) to gather the outputs, never on the data path.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Tile:
    index: int
    x0: int
    y0: int
    x1: int
    y1: int
    rx0: int
    ry0: int
    rx1: int
    ry1: int

    @property
    def cost(self) -> int:
        """Pixels the network computes for this tile (its region)."""
        return (self.rx1 - self.rx0) * (self.ry1 - self.ry0)


def tile_grid(width: int, height: int, tile: int, margin: int) -> list[Tile]:
    """The reference's tiles, row-major: lib.rs:241-289."""
    if tile <= 0:
        raise ValueError("tile size 0")
    cols, rows = -(-width // tile), -(-height // tile)
    out = []
    for j in range(rows):
        y0, y1 = j * height // rows, (j + 1) * height // rows
        for i in range(cols):
            x0, x1 = i * width // cols, (i + 1) * width // cols
            out.append(Tile(len(out), x0, y0, x1, y1, max(x0 - margin, 0), max(y0 - margin, 0),
                            min(x1 + margin, width), min(y1 + margin, height)))
    return out


def split_ranges(costs: list[int], world: int) -> list[tuple[int, int]]:
    """Contiguous ranges [first, last) of items, one per rank, each as close
    as a prefix split allows to 1/world of the total cost."""
    n = len(costs)
    total = sum(costs)
    ranges, start, acc = [], 0, 0
    for r in range(world):
        if r == world - 1:
            ranges.append((start, n))
            break
        target = total * (r + 1) / world
        end = start
        while end < n and acc + costs[end] / 2 <= target:
            acc += costs[end]
            end += 1
        # Leave at least one item for each remaining rank when possible.
        end = min(end, n - (world - 1 - r)) if n >= world else end
        end = max(end, start)
        ranges.append((start, end))
        start = end
    return ranges


def split_batch(count: int, world: int) -> list[tuple[int, int]]:
    """Contiguous slices of a batch, sizes differing by at most one."""
    return [(r * count // world, (r + 1) * count // world) for r in range(world)]


def crop_windows(out, tiles: list[Tile], scale: int = 4):
    """The tiles' windows of a (scale H) x (scale W) x 3 output, as arrays."""
    return [(t.index, out[scale * t.y0:scale * t.y1, scale * t.x0:scale * t.x1].copy()) for t in tiles]


def stitch(out, tiles: list[Tile], windows, scale: int = 4):
    """Write gathered windows [(tile index, array)] into the full output."""
    by_index = {t.index: t for t in tiles}
    for index, arr in windows:
        t = by_index[index]
        out[scale * t.y0:scale * t.y1, scale * t.x0:scale * t.x1] = arr
    return out


def gather_windows(local, rank: int, world: int, dist=None):
    """All ranks' [(tile index, array)] lists, concatenated on rank 0 (None
    elsewhere), through torch.distributed.gather_object."""
    if world == 1 or dist is None:
        return list(local)
    parts = [None] * world if rank == 0 else None
    dist.gather_object(local, parts, dst=0)
    if rank != 0:
        return None
    return [w for part in parts for w in part]


def band_of(tiles: list[Tile], first: int, last: int, scale: int = 4) -> tuple[int, int]:
    """Output rows [y0, y1) that hold the windows of tiles first .. last - 1
    (a contiguous row-major range, so one band of whole output rows)."""
    if first >= last:
        return 0, 0
    return scale * min(t.y0 for t in tiles[first:last]), scale * max(t.y1 for t in tiles[first:last])


def gather_bands(out, tiles: list[Tile], ranges: list[tuple[int, int]], rank: int, world: int, dist, scale: int = 4):
    """Reassemble a tiled output on rank 0 without leaving the devices: rank
    r > 0 sends the band of output rows its tiles' windows lie in (a
    contiguous slice of `out`, a (scale H) x (scale W) x 3 tensor) with
    torch.distributed point-to-point sends (NCCL over NVLink for CUDA
    tensors, gloo for CPU ones); rank 0 receives the bands in rank order and
    copies only that rank's windows into its own `out`. Every rank takes the
    same steps; returns `out` (complete on rank 0)."""
    if world == 1:
        return out
    if rank != 0:
        y0, y1 = band_of(tiles, *ranges[rank], scale)
        if y1 > y0:
            dist.send(out[y0:y1].contiguous(), dst=0)
        return out
    for r in range(1, world):
        first, last = ranges[r]
        y0, y1 = band_of(tiles, first, last, scale)
        if y1 <= y0:
            continue
        band = out.new_empty((y1 - y0,) + tuple(out.shape[1:]))
        dist.recv(band, src=r)
        for t in tiles[first:last]:
            out[scale * t.y0:scale * t.y1, scale * t.x0:scale * t.x1] = \
                band[scale * t.y0 - y0:scale * t.y1 - y0, scale * t.x0:scale * t.x1]
    return out

"""Row sharding of one material (config 4b): the band plan and the halo exchanges, on CPU.

The exchanges run over torch.distributed with the gloo backend and 2 or 3 ranks; the
expected result is the one the in-process LocalShards exchange defines (the GPU tests
check that against the unsharded training step)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from neural_textures_b200.sharded import HALO, DistComm, exchange_gradients, exchange_latents, lattice_band, \
    source_band


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("lattice_h,height", [(512, 512), (512, 256), (2048, 4096), (1024, 16384), (96, 64)])
def test_bands_partition_the_source(world, lattice_h, height):
    if world > 1 and height // world < HALO:
        pytest.skip("band thinner than the halo")
    bands = [source_band(r, world, lattice_h, height) for r in range(world)]
    assert bands[0].lo == 0 and bands[-1].hi == height
    for a, b in zip(bands, bands[1:]):
        assert a.hi == b.lo
    assert sum(b.owned for b in bands) == height


def _footprint_rows(iy_lo, iy_hi, lattice_h, image_h, height):
    """Every source row the Catmull-Rom footprints of lattice rows [iy_lo, iy_hi) can reach
    (jitter at both extremes, float32 arithmetic as in the kernels)."""
    rows = set()
    stride = np.float32(image_h / lattice_h)
    for iy in range(iy_lo, iy_hi):
        for j in (np.float32(-0.5), np.float32(0.4999999)):
            t = np.float32(np.float32(iy) + np.float32(0.5)) + j
            py = np.float32(t * stride)
            py = min(max(py, np.float32(0.5)), np.float32(image_h - 0.5))
            v = np.float32(py / np.float32(image_h))
            by = int(np.floor(np.float32(v * np.float32(height)) - np.float32(0.5)))
            rows.update((by - 1 + k) % height for k in range(4))
    return rows


@pytest.mark.parametrize("world", [2, 3, 4])
@pytest.mark.parametrize("lattice_h,image_h,height", [(128, 256, 128), (128, 256, 64), (64, 512, 512), (96, 96, 48)])
def test_halo_covers_every_footprint(world, lattice_h, image_h, height):
    for r in range(world):
        a, b = lattice_band(r, world, lattice_h)
        band = source_band(r, world, lattice_h, height)
        stored = set(band.stored_rows_of_full().tolist())
        missing = _footprint_rows(a, b, lattice_h, image_h, height) - stored
        assert not missing, (r, sorted(missing)[:8])


class _FakeShard:
    """Just the buffers and views the exchange functions touch (no device state)."""

    def __init__(self, rank, world, lattice_h, heights, width, C):
        self.torch = torch
        self.rank, self.world = rank, world
        self.bands = [source_band(rank, world, lattice_h, h) for h in heights]
        # value of stored row k of grid i on this rank: 1000 * full row + 10 * rank + i
        self.grids, self.ggrads = [], []
        for i, b in enumerate(self.bands):
            full = torch.from_numpy(b.stored_rows_of_full().astype(np.float32))
            g = (1000 * full + 10 * rank + i).view(-1, 1, 1).expand(b.stored, width, C).contiguous()
            self.grids.append(g.clone())
            self.ggrads.append(g.clone())

    band_view = lambda s, t, i: t[i][s.bands[i].halo:s.bands[i].halo + s.bands[i].owned]
    halo_above = lambda s, t, i: t[i][:s.bands[i].halo]
    halo_below = lambda s, t, i: t[i][s.bands[i].halo + s.bands[i].owned:]
    band_first = lambda s, t, i: t[i][s.bands[i].halo:2 * s.bands[i].halo]
    band_last = lambda s, t, i: t[i][s.bands[i].owned:s.bands[i].owned + s.bands[i].halo]


def _worker(rank, world, port, lattice_h, heights, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        s = _FakeShard(rank, world, lattice_h, heights, 3, 4)
        before = [g.clone() for g in s.ggrads]
        exchange_gradients(s, DistComm())
        exchange_latents(s, DistComm())
        out = []
        for i, b in enumerate(s.bands):
            full = b.stored_rows_of_full()
            # gradients: the band's first / last HALO rows gained the neighbours' halo copies of
            # the same full rows (value 1000 * row + 10 * neighbour + i); halos were cleared
            g = s.ggrads[i][:, 0, 0].numpy()
            exp = before[i][:, 0, 0].numpy().copy()
            exp[:HALO] = 0
            exp[HALO + b.owned:] = 0
            up, dn = (rank - 1) % world, (rank + 1) % world
            exp[HALO:2 * HALO] += 1000 * full[HALO:2 * HALO] + 10 * up + i
            exp[b.owned:b.owned + HALO] += 1000 * full[b.owned:b.owned + HALO] + 10 * dn + i
            # latents: halo rows now hold the owners' values of those full rows
            lat = s.grids[i][:, 0, 0].numpy()
            exp_lat = 1000 * full + 10 * rank + i
            exp_lat[:HALO] = 1000 * full[:HALO] + 10 * up + i
            exp_lat[HALO + b.owned:] = 1000 * full[HALO + b.owned:] + 10 * dn + i
            out.append(bool(np.array_equal(g, exp)) and bool(np.array_equal(lat, exp_lat)))
        q.put((rank, all(out)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_halo_exchange_over_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 48, (48, 24), q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(results.values()), results

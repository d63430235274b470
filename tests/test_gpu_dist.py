"""The one-thread sharded step of the C ABI (nt_dist_train_step) against the in-process
sharded step (LocalShards, which the sharded tests check against the unsharded training
step): shards sharing one GPU, and, where the box has two GPUs, shards on both (the
exchange kernels then read the other GPU's memory)."""
import ctypes as C

import numpy as np
import pytest

from tests.model_utils import rel_l2

pytestmark = pytest.mark.gpu

CASES = [  # image, grids, C, cout, lattice
    ((256, 256), ((128, 128), (64, 64)), 8, 8, (128, 128)),
    ((192, 256), ((96, 128), (48, 64)), 12, 12, (96, 128)),
]
STEPS = 3
LR = 1e-2  # latent learning rate of ShardedTexture


def _make(case, world, seed, devices):
    from neural_textures_b200.sharded import ShardedTexture
    image, grids, Cc, cout, lattice = CASES[case]
    sh = [ShardedTexture(r, world, *image, grids, Cc, cout, lattice, device=devices[r % len(devices)])
          for r in range(world)]
    for s in sh:
        s.init(seed=seed)
    return sh


def _status(devices):
    import torch
    from neural_textures_b200 import _native
    out = 0
    for d in devices:
        with torch.cuda.device(d):
            v = C.c_uint32(0)
            _native.check(_native.load().nt_read_device_status(C.byref(v), 1))
            out |= v.value
    return out


def _cpu(t):
    return t.float().cpu().numpy()


def _compare(ref, got):
    import torch
    n = len(got)
    for r in range(n):
        a, b = ref[r], got[r]
        for i in range(2):
            x, y = _cpu(b.band_view(b.grids, i)), _cpu(a.band_view(a.grids, i))
            # the two sides differ only in the order of float atomics, which can flip the sign
            # of a near-zero gradient: Adam then moves that entry the other way (<= 2 lr a step)
            diff = np.abs(x - y)
            assert np.mean(diff > 1e-3) < 0.01 and diff.max() <= 2 * STEPS * LR + 1e-3, (r, i, diff.max())
            # halo rows hold the neighbours' band edges exactly
            up, dn = got[(r - 1) % n], got[(r + 1) % n]
            assert torch.equal(b.halo_above(b.grids, i).cpu(), up.band_last(up.grids, i).cpu())
            assert torch.equal(b.halo_below(b.grids, i).cpu(), dn.band_first(dn.grids, i).cpu())
            # every gradient was consumed: band by Adam, halos by the refresh
            assert not bool(b.ggrads[i].any())
        for l in range(3):
            assert rel_l2(_cpu(b.W[l]), _cpu(a.W[l])) < 1e-2
            assert rel_l2(_cpu(b.b[l]), _cpu(a.b[l])) < 1e-2
            assert torch.equal(b.W[l].cpu(), got[0].W[l].cpu())  # one network, bit-identical on every shard
            assert torch.equal(b.b[l].cpu(), got[0].b[l].cpu())
        assert not bool(b.net_grad.any())
        assert b.step == a.step == STEPS
    loss_ref = sum(float(s.loss_accum.item()) for s in ref)
    loss_got = sum(float(s.loss_accum.item()) for s in got)
    assert abs(loss_got - loss_ref) <= 1e-3 * loss_ref


def _run(case, world, ref_devices, got_devices, seed, own_streams=False):
    import torch
    from neural_textures_b200.sharded import LocalShards, dist_train_step
    ref = LocalShards(_make(case, world, seed, ref_devices))
    got = _make(case, world, seed, got_devices)
    streams = None
    if own_streams:  # one stream per shard: only the events order the phases across shards
        torch.cuda.synchronize()
        held = [torch.cuda.Stream(device=s.device) for s in got]
        streams = [st.cuda_stream for st in held]
    for _ in range(STEPS):
        ref.step()
        dist_train_step(got, streams)
    for d in set(ref_devices) | set(got_devices):
        torch.cuda.synchronize(d)
    assert _status(sorted(set(got_devices))) == 0
    _compare(ref.shards, got)


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_dist_step_matches_local_shards(cuda, world, case):
    _run(case, world, ["cuda:0"], ["cuda:0"], seed=7)


@pytest.mark.parametrize("world", [2, 3])
def test_dist_step_with_a_stream_per_shard(cuda, world):
    """Shards on one GPU, each on its own stream: the phases are ordered only by the events
    between the streams."""
    _run(0, world, ["cuda:0"], ["cuda:0"], seed=11, own_streams=True)


@pytest.mark.parametrize("world", [2, 4])
def test_dist_step_on_two_devices(cuda, world):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run(0, world, ["cuda:0"], ["cuda:0", "cuda:1"], seed=9)


def test_dist_single_shard_is_train_step(cuda):
    """count 1: the training pass and Adam of nt_train_step."""
    import torch
    from neural_textures_b200.sharded import dist_train_step, train_step
    a = _make(0, 1, 3, ["cuda:0"])
    b = _make(0, 1, 3, ["cuda:0"])
    for _ in range(2):
        train_step(a[0], None)
        dist_train_step(b)
    torch.cuda.synchronize()
    for i in range(2):
        diff = np.abs(_cpu(a[0].grids[i]) - _cpu(b[0].grids[i]))
        assert np.mean(diff > 1e-3) < 0.01
    assert b[0].step == 2

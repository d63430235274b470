"""Row-sharded training (config 4b) against the unsharded training step, on one GPU.

Several shards of one material run in one process (LocalShards): each trains its band of
lattice rows with the CUDA kernel on its stored rows only, halo gradients go to their
owners and the network gradients are summed, as the NCCL path does between GPUs.  The
assembled result must equal the unsharded pass up to float atomic ordering."""
import ctypes as C

import numpy as np
import pytest

from tests.model_utils import rel_l2

pytestmark = pytest.mark.gpu

CASES = [  # image, grids, C, cout, lattice
    ((256, 256), ((128, 128), (64, 64)), 8, 8, (128, 128)),
    ((192, 256), ((96, 128), (48, 64)), 12, 12, (96, 128)),
    ((256, 192), ((128, 96), (64, 48)), 8, 10, (128, 96)),
]


def _unsharded(torch, image, grids, Cc, cout, lattice, seed):
    import neural_textures_b200 as nt
    t = nt.NeuralTexture(*image, grid_sizes=grids, latent_channels=Cc, output_channels=cout, lattice=lattice)
    t.init(seed=seed)
    return t


def _shards(image, grids, Cc, cout, lattice, world, seed):
    from neural_textures_b200.sharded import LocalShards, ShardedTexture
    sh = [ShardedTexture(r, world, *image, grids, Cc, cout, lattice) for r in range(world)]
    for s in sh:
        s.init(seed=seed)
    return LocalShards(sh)


def _status():
    from neural_textures_b200 import _native
    v = C.c_uint32(0)
    _native.check(_native.load().nt_read_device_status(C.byref(v), 1))
    return v.value


@pytest.mark.parametrize("world", [1, 2, 3])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_sharded_gradients_equal_unsharded(cuda, world, case):
    import torch
    from neural_textures_b200 import _native
    image, grids, Cc, cout, lattice = CASES[case]
    ref = _unsharded(torch, image, grids, Cc, cout, lattice, seed=3)
    _status()
    _native.check(_native.load().nt_invoke_training(C.byref(ref.params()), 0, None))
    loc = _shards(image, grids, Cc, cout, lattice, world, seed=3)
    loc.gradients()
    torch.cuda.synchronize()
    assert _status() == 0
    for i in range(2):
        got = loc.gather(lambda s: s.ggrads, i).cpu().numpy()
        exp = ref.ggrads[i].cpu().numpy()
        assert rel_l2(got, exp) < 1e-5, (i, rel_l2(got, exp))
    s0 = loc.shards[0]
    for l in range(3):
        assert rel_l2(s0.gW[l].cpu().numpy(), ref.gW[l].cpu().numpy()) < 1e-5
        assert rel_l2(s0.gb[l].cpu().numpy(), ref.gb[l].cpu().numpy()) < 1e-5
    loss = sum(float(s.loss_accum.item()) for s in loc.shards)
    assert abs(loss - float(ref.loss_accum.item())) <= 1e-4 * float(ref.loss_accum.item())


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_steps_follow_unsharded(cuda, world):
    import torch
    image, grids, Cc, cout, lattice = CASES[0]
    ref = _unsharded(torch, image, grids, Cc, cout, lattice, seed=5)
    loc = _shards(image, grids, Cc, cout, lattice, world, seed=5)
    for _ in range(4):
        ref.train_step()
        loc.step()
    torch.cuda.synchronize()
    assert _status() == 0
    for i in range(2):
        got = loc.gather(lambda s: s.grids, i).float().cpu().numpy()
        exp = ref.grids[i].float().cpu().numpy()
        # Adam moves every latent by ~lr per step; atomics may flip the sign of a
        # near-zero gradient, so a few entries may differ by up to 2 lr per step
        diff = np.abs(got - exp)
        assert np.mean(diff > 1e-3) < 0.01 and diff.max() <= 8 * 1e-2 + 1e-3
    for l in range(3):
        assert rel_l2(loc.shards[-1].W[l].float().cpu().numpy(), ref.W[l].float().cpu().numpy()) < 1e-2
        assert torch.equal(loc.shards[0].W[l], loc.shards[-1].W[l])  # the network stays replicated
    # halo rows hold the owners' latest values
    for r, s in enumerate(loc.shards):
        n = len(loc.shards)
        for i in range(2):
            assert torch.equal(s.halo_below(s.grids, i), loc.shards[(r + 1) % n].band_first(loc.shards[(r + 1) % n].grids, i))

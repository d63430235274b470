"""BC6 block-feature training (TrainingKernelType::BLOCK_FEATURES, train.cu:316-458, :641-762)
against the CPU oracle.

The latents are float BC6 block records (endpoints, pixel indices, partition, mode) decoded
with the reference's float BC6 decode (train.cu:161-182, pinned bit-exactly by the golden
vectors); the CUDA training pass samples them through the Catmull-Rom footprint and sends
gradients into the records (train.cu:436-454).

- one training pass: network gradients and record gradients, relative L2 <= 2e-2, loss 1e-3;
- FINALIZE on block features (train.cu:1044-1046): records untouched, network gradients match;
- Adam over the records (AdamUpdateFloatParameter, train.cu:545-564): bit-exact, partition and
  mode slots never change.
"""
import ctypes as C

import numpy as np
import pytest

from tests.model_utils import make_texture, rel_l2, realistic_blocks, target_host

pytestmark = pytest.mark.gpu

TOL = 2e-2
CASES = [  # image, grids, C, cout, lattice
    ((64, 64), ((32, 32), (16, 16)), 8, 8, (32, 32)),
    ((96, 80), ((48, 40), (24, 20)), 12, 12, (48, 40)),
]


def _block_texture(image, grids, Cc, cout, lattice, seed):
    tex = make_texture(image, grids, Cc, cout, lattice=lattice, seed=seed)
    rng = np.random.default_rng(seed + 5)
    recs = [realistic_blocks(rng, w, h, Cc) for (w, h) in grids]
    tex.use_blocks(recs)
    tex.step = 2
    return tex, recs


def _oracle(oracle, tex, recs, finalize=False):
    grids, W, b = tex.host_model()
    m = oracle.OracleModel(channels=tex.C, cout=tex.cout, grids=grids, W=W, b=b, blocks=recs,
                           block_sizes=list(tex.grid_sizes))
    s = oracle.make_sampler(tex.image_w, tex.image_h, tex.lattice[0], tex.lattice[1], step=tex.step, seed=tex.seed)
    return oracle.train_pass(m, target_host(tex), s, channel_weights=np.array(tex.channel_weights, np.float32),
                             finalize=finalize, threads=8)


def _gpu(tex, kind):
    import torch
    import neural_textures_b200 as nt
    tex.loss_accum.zero_()
    nt.InvokeTraining(tex.params(), kind)
    torch.cuda.synchronize()
    h = lambda t: t.detach().cpu().numpy().copy()
    return tex.loss_accum.item(), [h(g) for g in tex.gW], [h(g) for g in tex.gb], [h(g) for g in tex.ggrads]


def _status():
    from neural_textures_b200 import _native
    v = C.c_uint32(0)
    _native.check(_native.load().nt_read_device_status(C.byref(v), 1))
    return v.value


@pytest.mark.parametrize("case", range(len(CASES)))
def test_block_training_pass_matches_oracle(cuda, oracle, case):
    import neural_textures_b200 as nt
    image, grids, Cc, cout, lattice = CASES[case]
    tex, recs = _block_texture(image, grids, Cc, cout, lattice, seed=11 + case)
    sse, gW, gb, gg = _gpu(tex, nt.TrainingKernelType.BLOCK_FEATURES)
    rsse, rW, rb, rg = _oracle(oracle, tex, recs)
    assert _status() == 0
    assert abs(sse - rsse) <= 1e-3 * rsse, (sse, rsse)
    for l in range(3):
        assert rel_l2(gW[l], rW[l]) <= TOL, (l, rel_l2(gW[l], rW[l]))
        assert rel_l2(gb[l], rb[l]) <= TOL, (l, rel_l2(gb[l], rb[l]))
    for g in range(2):
        assert np.abs(rg[g]).max() > 0
        assert rel_l2(gg[g], rg[g]) <= TOL, (g, rel_l2(gg[g], rg[g]))
        # partition / mode / unused slots never receive a gradient
        assert np.all(gg[g].reshape(-1, 32)[:, 28:] == 0)


def test_block_finalize_trains_only_the_network(cuda, oracle):
    import neural_textures_b200 as nt
    image, grids, Cc, cout, lattice = CASES[0]
    tex, recs = _block_texture(image, grids, Cc, cout, lattice, seed=21)
    sse, gW, gb, gg = _gpu(tex, nt.TrainingKernelType.FINALIZE)
    rsse, rW, rb, rg = _oracle(oracle, tex, recs, finalize=True)
    assert all(np.all(g == 0) for g in gg)
    assert abs(sse - rsse) <= 1e-3 * rsse
    assert rel_l2(gW[1], rW[1]) <= TOL


def test_block_adam_bit_exact(cuda, oracle):
    import torch
    import neural_textures_b200 as nt
    image, grids, Cc, cout, lattice = CASES[1]
    tex, recs = _block_texture(image, grids, Cc, cout, lattice, seed=31)
    rng = np.random.default_rng(3)
    host = []
    for g in range(2):
        n = tex.blocks[g].numel()
        grad = (rng.standard_normal(n) * 1e-3).astype(np.float32).reshape(-1, 32)
        grad[:, 28:] = 0.0             # the records' integer slots never get a gradient
        grad[rng.random(grad.shape) < 0.2] = 0.0   # zero-skip entries
        m1 = (rng.standard_normal(n) * 1e-4).astype(np.float32)
        m2 = np.abs(rng.standard_normal(n) * 1e-6).astype(np.float32)
        tex.ggrads[g].copy_(torch.from_numpy(grad.reshape(-1)).to(tex.device))
        tex.gm1[g].copy_(torch.from_numpy(m1).to(tex.device))
        tex.gm2[g].copy_(torch.from_numpy(m2).to(tex.device))
        host.append((recs[g].copy(), grad.reshape(-1).copy(), m1.copy(), m2.copy()))
    nt.InvokeOptimizeFeatures(tex.params(), nt.TrainingKernelType.BLOCK_FEATURES)
    torch.cuda.synchronize()
    b1, b2, lr, eps = tex.latent_adam
    for g in range(2):
        w, gr, m1, m2 = host[g]
        oracle.adam_f32(w, gr, m1, m2, lr, b1, b2, eps, tex.step)
        got = tex.blocks[g].cpu().numpy()
        assert np.array_equal(got.view(np.uint32), w.view(np.uint32))
        assert np.array_equal(tex.gm1[g].cpu().numpy().view(np.uint32), m1.view(np.uint32))
        assert np.array_equal(tex.gm2[g].cpu().numpy().view(np.uint32), m2.view(np.uint32))
        assert np.all(tex.ggrads[g].cpu().numpy() == 0)
        assert np.array_equal(got.reshape(-1, 32)[:, 28:30].view(np.int32), recs[g].reshape(-1, 32)[:, 28:30].view(np.int32))

"""Mip-chain latents and targets sampled at a mip coordinate (NtKernelParams.lod) against the
CPU oracle.

The reference keeps numMips levels per feature (train.h:61), chooses levels floor(lod) and the
next one and blends them (train.cu:78-103, :264-314), and runs Adam over every level
(train.cu:990-1026); its driver samples lod 0 only.  Here every sample of a call reads its
latents and its target at p.lod:
- training pass at integer, fractional and out-of-chain lods: loss within 1e-3, network and
  per-level latent gradients within relative L2 2e-2, levels not read get no gradient;
- decode at a fractional lod: max relative error 1e-2 (floor 1), the north-star decode bar;
- inference_mse_accum against the target level of an integer lod;
- Adam over whole chains and the target mip builder: bit-exact.
"""
import ctypes as C

import numpy as np
import pytest

from tests.model_utils import make_texture, max_rel, rel_l2

pytestmark = pytest.mark.gpu

TOL = 2e-2
CASES = [  # image, grids, C, cout, lattice, latent mips, target mips, lod
    ((64, 64), ((32, 32), (16, 16)), 8, 8, (32, 32), (4, 3), 4, 1.5),
    ((64, 64), ((32, 32), (16, 16)), 8, 8, (32, 32), (4, 3), 4, 1.0),
    ((96, 80), ((48, 40), (24, 20)), 12, 12, (48, 40), (5, 4), 5, 0.3),
    ((64, 64), ((32, 32), (16, 16)), 8, 8, (32, 32), (3, 2), 6, 2.6),  # past grid 1's chain: clamped
]


def _h16(t):
    import torch
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _h32(t):
    return t.detach().cpu().numpy().copy()


def _texture(case, seed):
    image, grids, Cc, cout, lattice, mips, tmips, lod = case
    tex = make_texture(image, grids, Cc, cout, lattice=lattice, seed=seed, num_mips=mips, target_num_mips=tmips)
    tex.lod = lod
    tex.step = 3
    return tex


def _model(oracle, tex):
    _, W, b = tex.host_model()
    mips = [[_h16(tex.mip_level(g, m)) for m in range(tex.num_mips[g])] for g in range(2)]
    return oracle.OracleModel(channels=tex.C, cout=tex.cout, grids=[m[0] for m in mips], W=W, b=b, mips=mips,
                              lod=tex.lod)


def _target_chain(tex):
    return [_h16(tex.target_level(m)) for m in range(tex.target_num_mips)]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_training_pass_at_lod_matches_oracle(cuda, oracle, case):
    import torch
    import neural_textures_b200 as nt
    tex = _texture(CASES[case], seed=20 + case)
    tex.loss_accum.zero_()
    nt.InvokeTraining(tex.params(), nt.TrainingKernelType.UNCONSTRAINED)
    torch.cuda.synchronize()
    model = _model(oracle, tex)
    tchain = _target_chain(tex)
    s = oracle.make_sampler(tex.image_w, tex.image_h, tex.lattice[0], tex.lattice[1], step=tex.step, seed=tex.seed)
    rsse, rW, rb, rg = oracle.train_pass(model, tchain[0], s, channel_weights=np.array(tex.channel_weights, np.float32),
                                         threads=8, target_mips=tchain)
    sse = tex.loss_accum.item()
    assert abs(sse - rsse) <= 1e-3 * rsse, (sse, rsse)
    for l in range(3):
        assert rel_l2(_h32(tex.gW[l]), rW[l]) <= TOL, l
        assert rel_l2(_h32(tex.gb[l]), rb[l]) <= TOL, l
    for g in range(2):
        read = 0
        for m in range(tex.num_mips[g]):
            got = _h32(tex.mip_level(g, m, chain=tex.ggrads[g]))
            want = rg[g][m]
            if np.abs(want).max() == 0:
                assert np.all(got == 0), (g, m)
            else:
                read += 1
                assert rel_l2(got, want) <= TOL, (g, m, rel_l2(got, want))
        assert read >= 1


def test_decode_at_fractional_lod(cuda, oracle):
    import torch
    tex = _texture(CASES[0], seed=31)
    out = tex.decode(dtype=torch.float32)
    torch.cuda.synchronize()
    want = oracle.decode(_model(oracle, tex), tex.image_w, tex.image_h, out_f32=True, threads=8)
    assert max_rel(_h32(out), want) <= 1e-2


def test_inference_mse_at_integer_lod(cuda, oracle):
    """A 32 x 32 decode at lod 1 of a 64 x 64 material compares with target level 1."""
    import torch
    import neural_textures_b200 as nt
    tex = _texture(CASES[1], seed=41)
    out = torch.empty((32 * 32, tex.cout), dtype=torch.float32, device=tex.device)
    acc = torch.zeros(1, dtype=torch.float32, device=tex.device)
    p = tex.params(inference_output=out, mse_accum=acc)
    p.image_width = p.image_height = 32
    p.target_width = p.target_height = 64
    nt.InvokeInference(p)
    torch.cuda.synchronize()
    want = oracle.decode(_model(oracle, tex), 32, 32, out_f32=True, threads=8)
    assert max_rel(_h32(out), want) <= 1e-2
    t1 = tex.target_level(1).float().cpu().numpy().reshape(-1, tex.cout)
    sse = float(((_h32(out).astype(np.float64) - t1) ** 2).sum())
    assert abs(acc.item() - sse) <= 1e-4 * sse + 1e-6


def test_adam_over_chains_bit_exact(cuda, oracle):
    import torch
    import neural_textures_b200 as nt
    tex = _texture(CASES[0], seed=51)
    rng = np.random.default_rng(9)
    before = []
    for g in range(2):
        n = tex.ggrads[g].numel()
        grad = (rng.standard_normal(n) * 1e-2).astype(np.float32)
        grad[rng.random(n) < 0.3] = 0.0
        m1 = (rng.standard_normal(n) * 1e-3).astype(np.float32)
        m2 = np.abs(rng.standard_normal(n) * 1e-5).astype(np.float32)
        tex.ggrads[g].view(-1).copy_(torch.from_numpy(grad))
        tex.gm1[g].view(-1).copy_(torch.from_numpy(m1))
        tex.gm2[g].view(-1).copy_(torch.from_numpy(m2))
        before.append((_h16(tex.grid_chains[g]), grad, m1, m2))
    nt.InvokeOptimizeFeatures(tex.params(), nt.TrainingKernelType.UNCONSTRAINED)
    torch.cuda.synchronize()
    b1, b2, lr, eps = tex.latent_adam
    for g in range(2):
        w, grad, m1, m2 = (x.copy() for x in before[g])
        oracle.adam_f16(w, grad, m1, m2, lr, b1, b2, eps, tex.step)
        assert np.array_equal(_h16(tex.grid_chains[g]), w)
        assert np.array_equal(_h32(tex.gm1[g]).reshape(-1).view(np.uint32), m1.view(np.uint32))
        assert np.array_equal(_h32(tex.gm2[g]).reshape(-1).view(np.uint32), m2.view(np.uint32))


@pytest.mark.parametrize("size,channels,n", [((64, 64), 8, 7), ((96, 80), 12, 7), ((70, 50), 3, 5), ((1, 37), 16, 6)])
def test_build_mips_bit_exact(cuda, oracle, size, channels, n):
    import torch
    import neural_textures_b200 as nt
    from neural_textures_b200 import _native
    w, h = size
    rng = np.random.default_rng(w * 7 + channels)
    total = nt.api.mip_chain_texels(w, h, n) * channels
    chain = torch.zeros(total, dtype=torch.float16, device="cuda:0")
    l0 = (rng.standard_normal((h, w, channels)) * 2).astype(np.float16)
    chain[:w * h * channels].copy_(torch.from_numpy(l0.reshape(-1)))
    _native.check(_native.load().nt_build_mips(chain.data_ptr(), w, h, channels, n, None))
    torch.cuda.synchronize()
    want = oracle.build_mips(l0.view(np.uint16), n)
    got = _h16(chain)
    assert np.array_equal(got, np.concatenate([x.reshape(-1) for x in want]))

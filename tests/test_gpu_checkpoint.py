"""NeuralTexture.save / load through the on-disk format.

- resume: a material saved with its Adam state loads bit-identically (parameters, moments,
  step, seed), and its next training step matches the original's up to the order of the
  gradient atomics (relative 1e-5; the CTAs add their gradients in run-dependent order);
- latents="bc6h": the loaded grids are the BC6H decode of the saved grids;
- block-feature records, mip chains and the mip coordinate survive a round trip.
"""
import numpy as np
import pytest

from tests.model_utils import make_texture, realistic_blocks, rel_l2

pytestmark = pytest.mark.gpu


def _bits(t):
    import torch
    t = t.detach().cpu().contiguous()
    return t.view(torch.int16).numpy().tobytes() if t.dtype == torch.float16 else t.numpy().tobytes()


def _state(tex):
    out = [tex.loss_accum]
    out += tex.W + tex.b + tex.mW + tex.vW + tex.mb + tex.vb + tex.gm1 + tex.gm2
    out += tex.blocks if tex.blocks is not None else tex.grid_chains
    return [_bits(x) for x in out]


def test_resume_is_bit_identical(cuda, tmp_path):
    import neural_textures_b200 as nt
    tex = make_texture((64, 64), ((32, 32), (16, 16)), 8, 8, lattice=(32, 32), seed=5)
    for _ in range(3):
        tex.train_step()
    path = tmp_path / "m.ntck"
    tex.save(path, optimizer=True, target=True)
    twin = nt.NeuralTexture.load(path, device=tex.device)
    assert twin.step == tex.step == 3 and twin.seed == tex.seed
    assert _state(tex)[1:] == _state(twin)[1:]
    assert _bits(twin.target_chain) == _bits(tex.target_chain)
    for t in (tex, twin):
        t.loss_accum.zero_()
        t.train_step()
    a, b = tex.loss_accum.item(), twin.loss_accum.item()
    assert abs(a - b) <= 1e-5 * a
    for x, y in zip(tex.mW + tex.vW + tex.gm1, twin.mW + twin.vW + twin.gm1):
        assert rel_l2(y.cpu().numpy(), x.cpu().numpy()) <= 1e-5


def test_bc6h_latents(cuda, tmp_path, oracle):
    import torch
    import neural_textures_b200 as nt
    tex = make_texture((64, 64), ((32, 32), (16, 16)), 8, 8, lattice=(32, 32), seed=6)
    path = tmp_path / "c.ntck"
    tex.save(path, optimizer=False, latents="bc6h", bias=4.0)
    idx = nt.api.checkpoint_index(path)
    assert "latent0.bc6h" in idx and "latent0" not in idx and "adam.m0" not in idx
    back = nt.NeuralTexture.load(path, device=tex.device)
    for g in range(2):
        ref = torch.empty_like(tex.grids[g])
        nt.bc6h_decode(nt.bc6h_encode(tex.grids[g], "interleaved", 4.0), ref, "interleaved", 4.0)
        assert torch.equal(back.grids[g], ref)
    assert all(torch.equal(a, b) for a, b in zip(back.W, tex.W))


def test_blocks_and_mips_round_trip(cuda, tmp_path):
    import torch
    import neural_textures_b200 as nt
    tex = make_texture((64, 64), ((32, 32), (16, 16)), 12, 12, lattice=(32, 32), seed=7)
    rng = np.random.default_rng(7)
    tex.use_blocks([realistic_blocks(rng, w, h, 12) for (w, h) in tex.grid_sizes])
    tex.block_bias = 3.0
    tex.save(tmp_path / "b.ntck")
    back = nt.NeuralTexture.load(tmp_path / "b.ntck", device=tex.device)
    assert back.latent_format == nt._native.NT_LATENT_BC6_BLOCKS and back.block_bias == 3.0
    assert all(torch.equal(a, b) for a, b in zip(back.blocks, tex.blocks))

    mt = make_texture((64, 64), ((32, 32), (16, 16)), 8, 8, lattice=(32, 32), seed=8, num_mips=(4, 3),
                      target_num_mips=5)
    mt.lod = 1.25
    mt.train_step()
    mt.save(tmp_path / "m.ntck", target=True)
    mb = nt.NeuralTexture.load(tmp_path / "m.ntck", device=mt.device)
    assert mb.num_mips == [4, 3] and mb.target_num_mips == 5 and mb.lod == 1.25
    assert all(torch.equal(a, b) for a, b in zip(mb.grid_chains, mt.grid_chains))
    assert torch.equal(mb.target_chain, mt.target_chain)

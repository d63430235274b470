"""BC6 block-feature training (TrainingKernelType::BLOCK_FEATURES, train.cu:316-458, :641-762)
against the CPU oracle.

The latents are float BC6 block records (endpoints, pixel indices, partition, mode) decoded
with the reference's float BC6 decode (train.cu:161-182, pinned bit-exactly by the golden
vectors); the CUDA training pass samples them through the Catmull-Rom footprint and sends
gradients into the records (train.cu:436-454).

- one training pass: network gradients and record gradients, relative L2 <= 2e-2, loss 1e-3
  (windowed decode with the tensor-core scatter or the column sweep, and the direct fallback);
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
    # coarse lattice: a tile's footprint window outgrows the shared decode buffer, so the
    # samples decode their taps directly and scatter per tap
    ((128, 128), ((128, 128), (64, 64)), 8, 8, (16, 16)),
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


# ---- block records <-> BC6H blocks (nt_bc6f_from_bc6h / nt_bc6f_to_bc6h) -----------------

def _edge_records(rng, n):
    """Records outside the trained range: NaN / inf endpoints and indices, negative and large
    pixel indices, far endpoints, out-of-range partition and mode fields."""
    rec = np.zeros((n, 32), np.float32)
    rec[:, :12] = rng.uniform(-3000.0, 3000.0, (n, 12))
    rec[:, 12:28] = rng.uniform(-0.5, 0.7, (n, 16))
    rec[0, 3] = np.nan
    rec[1, 14] = np.inf
    rec[2, 0] = -np.inf
    rec[3, 20] = np.nan
    rec[:, 28].view(np.int32)[:] = rng.integers(-100, 100, n)
    rec[:, 29].view(np.int32)[:] = rng.integers(-3, 14, n)
    return rec.reshape(-1)


def test_bridge_matches_oracle(cuda, oracle):
    import torch
    import neural_textures_b200 as nt
    rng = np.random.default_rng(41)
    dev = torch.device("cuda", 0)
    # bitstreams: random raw blocks (every mode) and blocks our encoder writes
    W, H, C = 64, 32, 12
    raw = rng.integers(0, 256, nt.bc6h_blocks_bytes(W, H, C), dtype=np.uint8)
    lat = oracle.smooth_latents(rng, (C, H, W))
    enc = oracle.bc6h_encode_surface(lat, "planar", 4.0)
    for blocks in (raw, enc):
        got = nt.bc6f_from_bc6h(torch.from_numpy(blocks).to(dev), W, H, C).cpu().numpy()
        want = oracle.bc6f_from_bc6h(blocks, W, H, C)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        back = nt.bc6f_to_bc6h(torch.from_numpy(want).to(dev), W, H, C).cpu().numpy()
        assert np.array_equal(back, oracle.bc6f_to_bc6h(want, W, H, C))
    # trained-like and out-of-range records
    n = (W // 4) * (H // 4) * (C // 3)
    for rec in (realistic_blocks(rng, W, H, C), _edge_records(rng, n)):
        got = nt.bc6f_to_bc6h(torch.from_numpy(rec).to(dev), W, H, C).cpu().numpy()
        assert np.array_equal(got, oracle.bc6f_to_bc6h(rec, W, H, C))


def _smooth_texture(oracle, seed):
    import torch
    image, grids, Cc, cout, lattice = CASES[0]
    tex = make_texture(image, grids, Cc, cout, lattice=lattice, seed=seed)
    rng = np.random.default_rng(seed)
    for g, (w, h) in zip(tex.grids, grids):
        lat = oracle.smooth_latents(rng, (Cc, h, w)).transpose(1, 2, 0).copy()
        g.copy_(torch.from_numpy(lat).view(torch.float16).to(g.device))
    tex.step = 3
    return tex


def _finalize_loss(tex):
    import neural_textures_b200 as nt
    return _gpu(tex, nt.TrainingKernelType.FINALIZE)[0]


def test_to_blocks_keeps_the_encoded_network_output(cuda, oracle):
    """After to_blocks the block features reproduce the loss of the BC6H-decoded grids (the
    records decode within one fp16 ulp of the blocks; layer 1 absorbs the codec bias)."""
    import neural_textures_b200 as nt
    tex = _smooth_texture(oracle, 51)
    bias = 4.0
    for g in tex.grids:  # grids as the codec returns them
        nt.bc6h_decode(nt.bc6h_encode(g, "interleaved", bias), g, "interleaved", bias)
    want = _finalize_loss(tex)
    tex.to_blocks(bias)
    got = _finalize_loss(tex)
    assert _status() == 0
    assert abs(got - want) <= 1e-2 * want, (got, want)


def test_export_and_return_to_grids(cuda, oracle):
    """Records made from encoded grids export to the very same bitstream; from_bc6h brings
    the decoded grids and the original layer-1 bias back."""
    import torch
    import neural_textures_b200 as nt
    tex = _smooth_texture(oracle, 61)
    bias = 4.0
    enc = [nt.bc6h_encode(g, "interleaved", bias) for g in tex.grids]
    b1 = tex.b[0].clone()
    tex.to_blocks(bias)
    exported = tex.export_bc6h()
    for a, b in zip(exported, enc):
        assert torch.equal(a, b)
    tex.from_bc6h(exported)
    assert tex.latent_format == nt._native.NT_LATENT_GRID_F16
    assert (tex.b[0].float() - b1.float()).abs().max().item() <= 1e-2  # two fp16 roundings of a shift of a few units
    for g, e in zip(tex.grids, enc):
        ref = torch.empty_like(g)
        nt.bc6h_decode(e, ref, "interleaved", bias)
        assert torch.equal(g, ref)

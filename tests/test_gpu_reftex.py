"""Reference textures (train.h:69-77) on the texture units against the CPU oracle.

- sampling: nt_reference_texture_sample against the oracle's 9-fetch Catmull-Rom with exact
  bilinear weights, at level 0, level 1, a blend and past the chain, for 1 / 2 / 3 channels.  The
  CUDA documentation gives the texture unit's bilinear weights as 9-bit fixed point with 8
  fractional bits and leaves the rounding of the coordinate unspecified (none of exact,
  nearest-1/256 and truncated-1/256 weights matches it exactly: measured 3.9e-3, 3.7e-3 and 5.7e-3
  for values in [0, 1)), so the check is the documented bound: a weight off by at most 1/256 per
  axis moves a fetch by at most 2/256 of the value range, and the 9 Catmull-Rom weights sum to at
  most 1.15^2 in magnitude;
- a training pass whose target comes from three textures (RGB, one channel, two channels, with
  loss weights; trailing outputs trained towards 0 with weight 1, train.cu:105-157), at lod 0 and
  at a fractional lod: loss 1e-3, gradients relative L2 2e-2;
- the inference MSE against the textures (train.cu:946-960).
"""
import numpy as np
import pytest

from tests.model_utils import make_texture, rel_l2

pytestmark = pytest.mark.gpu

FILTER_BOUND = 1.15 ** 2 * 2.0 / 256.0  # x the value range (documented 8-bit weight precision)


def _textures(rng, size=(40, 24), mips=4):
    import neural_textures_b200 as nt
    w, h = size
    specs = [(3, 1.0), (1, 0.5), (2, 2.0)]
    texs, defs = [], []
    for ch, lw in specs:
        img = rng.random((h, w, ch)).astype(np.float32)
        t = nt.ReferenceTexture.from_image(img, num_mips=mips, loss_weight=lw)
        pad = np.concatenate([img, np.ones((h, w, 1), np.float32)], axis=2) if ch == 3 else img
        chain = nt.api.box_chain_f32(pad, mips)
        texs.append(t)
        defs.append((chain, w, h, ch, mips, lw))
    return texs, defs


def test_sampling_matches_the_emulated_filter(cuda, oracle):
    import torch
    rng = np.random.default_rng(3)
    texs, defs = _textures(rng)
    uv = rng.uniform(-0.5, 1.5, (512, 2)).astype(np.float32)
    uvd = torch.from_numpy(uv).cuda()
    for t, d in zip(texs, defs):
        for lod in (0.0, 1.0, 1.75, 9.0):
            got = t.sample(uvd, lod).cpu().numpy()
            exact = oracle.ref_sample([d], uv, lod, 0)
            span = float(d[0].max() - d[0].min())
            err = float(np.abs(got - exact).max())
            assert err <= FILTER_BOUND * span, (d[3], lod, err)
            assert err > 0.0  # the hardware path ran (fixed-point weights differ from exact ones)
    for t in texs:
        t.close()


@pytest.mark.parametrize("lod", [0.0, 1.5])
def test_training_pass_with_reference_textures(cuda, oracle, lod):
    import torch
    import neural_textures_b200 as nt
    rng = np.random.default_rng(11)
    texs, defs = _textures(rng)
    tex = make_texture((40, 24), ((20, 12), (10, 6)), 8, 8, lattice=(40, 24), seed=4, num_mips=(3, 2))
    tex.reference_textures = texs
    tex.lod = lod
    tex.step = 2
    tex.loss_accum.zero_()
    nt.InvokeTraining(tex.params(), nt.TrainingKernelType.UNCONSTRAINED)
    torch.cuda.synchronize()
    _, W, b = tex.host_model()
    h16 = lambda x: x.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    mips = [[h16(tex.mip_level(g, m)) for m in range(tex.num_mips[g])] for g in range(2)]
    model = oracle.OracleModel(channels=8, cout=8, grids=[m[0] for m in mips], W=W, b=b, mips=mips, lod=lod)
    s = oracle.make_sampler(40, 24, 40, 24, step=2, seed=tex.seed)
    rsse, rW, rb, rg = oracle.train_pass(model, None, s, threads=8, ref_textures_defs=defs)
    sse = tex.loss_accum.item()
    assert abs(sse - rsse) <= 1e-3 * rsse, (sse, rsse)
    for l in range(3):
        assert rel_l2(tex.gW[l].cpu().numpy(), rW[l]) <= 2e-2
        assert rel_l2(tex.gb[l].cpu().numpy(), rb[l]) <= 2e-2
    m0 = int(np.floor(lod))
    for g in range(2):
        got = tex.mip_level(g, min(m0, tex.num_mips[g] - 1), chain=tex.ggrads[g]).cpu().numpy()
        assert rel_l2(got, rg[g][min(m0, tex.num_mips[g] - 1)]) <= 2e-2
    for t in texs:
        t.close()


def test_inference_mse_against_reference_textures(cuda, oracle):
    import torch
    import neural_textures_b200 as nt
    rng = np.random.default_rng(12)
    texs, defs = _textures(rng)
    tex = make_texture((40, 24), ((20, 12), (10, 6)), 8, 8, seed=5)
    tex.reference_textures = texs
    out = torch.empty((40 * 24, 8), dtype=torch.float32, device=tex.device)
    acc = torch.zeros(1, dtype=torch.float32, device=tex.device)
    nt.InvokeInference(tex.params(inference_output=out, mse_accum=acc))
    torch.cuda.synchronize()
    y = out.cpu().numpy().astype(np.float64)
    refs = oracle.ref_textures(defs)
    L = oracle.lib()
    sse = 0.0
    for k in range(40 * 24):
        x, yy = k % 40, k // 40
        ex = np.zeros(16, np.float32)
        L.nto_ref_expected(refs, len(defs), (x + 0.5) / 40, (yy + 0.5) / 24, 0.0, ex.ctypes.data_as(oracle.f32p), None)
        sse += float(((y[k] - ex[:8]) ** 2).sum())
    assert abs(acc.item() - sse) <= 1e-3 * sse
    for t in texs:
        t.close()

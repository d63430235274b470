"""Decode (train.cu:917-961) parity: the CUDA decode kernel against the CPU oracle on the
same seeded latents and weights.  Tolerance: max relative error 1e-2 (fp16), relative to
max(|ref|, 0.25) (tests/model_utils.py DECODE_FLOOR: outputs below 0.25 are held to 2.5e-3
absolute, about one fp16 step at the top of the output range); the full config-0 image is
also held to at most 1% of its outputs differing from the oracle's at all."""
import os

import numpy as np
import pytest

from tests.model_utils import make_texture, max_rel, oracle_model, target_host

pytestmark = pytest.mark.gpu

TOL = 1e-2

CASES = [
    # image, grids, C, cout, fp32 output
    ((64, 64), ((32, 32), (16, 16)), 8, 8, False),
    ((48, 40), ((24, 20), (12, 10)), 12, 12, False),
    ((37, 29), ((19, 15), (9, 7)), 8, 12, True),
    ((16, 16), ((4, 4), (2, 2)), 8, 3, False),
    ((1, 1), ((1, 1), (1, 1)), 12, 8, True),
    ((100, 3), ((50, 2), (25, 1)), 8, 16, False),
]


@pytest.mark.parametrize("image,grids,C,cout,f32", CASES)
def test_decode_matches_oracle(cuda, oracle, image, grids, C, cout, f32):
    import torch
    tex = make_texture(image, grids, C, cout, seed=3)
    out = tex.decode(dtype=torch.float32 if f32 else torch.float16)
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float32)
    ref = oracle.decode(oracle_model(oracle, tex), image[0], image[1], out_f32=True)
    assert got.shape == ref.shape
    err = max_rel(got, ref)
    assert err <= TOL, f"max rel err {err}"


def test_decode_mse_accumulator(cuda, oracle):
    import torch
    tex = make_texture((64, 48), ((32, 24), (16, 12)), 8, 8, seed=5)
    mse = torch.zeros(1, dtype=torch.float32, device=cuda)
    out = torch.empty((64 * 48, 8), dtype=torch.float16, device=cuda)
    import neural_textures_b200 as nt
    nt.InvokeInference(tex.params(inference_output=out, mse_accum=mse))
    torch.cuda.synchronize()
    y = out.cpu().numpy().astype(np.float64)
    t = target_host(tex).view(np.float16).astype(np.float64).reshape(-1, 8)
    want = float(((y - t) ** 2).sum())
    assert abs(mse.item() - want) <= 1e-4 * want


@pytest.mark.parametrize("f32", [False, True])
def test_decode_full_config0(cuda, oracle, f32):
    """BASELINE config 0 (1024^2 texels, 512^2x8 + 256^2x8 latents, 8 outputs, He-normal
    weights from the seed): every one of the 1,048,576 x 8 outputs against the oracle."""
    import torch
    tex = make_texture((1024, 1024), ((512, 512), (256, 256)), 8, 8, seed=11)
    out = tex.decode(dtype=torch.float32 if f32 else torch.float16)
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float32)
    assert np.isfinite(got).all()
    ref = oracle.decode(oracle_model(oracle, tex), 1024, 1024, out_f32=True, threads=os.cpu_count() or 1)
    assert got.shape == ref.shape == (1024 * 1024, 8)
    err = max_rel(got, ref)
    differ = float(np.mean(got != ref))
    print(f"config 0 full image ({'fp32' if f32 else 'fp16'} output): max rel err {err:.3e}, "
          f"max abs err {float(np.max(np.abs(got - ref))):.3e}, outputs differing {differ:.4%}")
    assert err <= TOL, f"max rel err {err}"
    assert differ <= 0.01, differ


def test_decode_is_deterministic(cuda):
    import torch
    tex = make_texture((96, 64), ((48, 32), (24, 16)), 12, 12, seed=2)
    a = tex.decode().cpu()
    b = tex.decode().cpu()
    assert torch.equal(a, b)


@pytest.mark.parametrize("f32", [False, True])
def test_decode_output_stride(cuda, f32):
    """inference_output_stride > output_channels (the reference's [N][16] fp32 layout,
    train.cu:950-955): the first output_channels of every texel equal the packed decode and
    the channels past them are written as 0."""
    import torch
    import neural_textures_b200 as nt
    tex = make_texture((40, 24), ((20, 12), (10, 6)), 8, 8, seed=4)
    dt = torch.float32 if f32 else torch.float16
    packed = tex.decode(dtype=dt)
    wide = torch.full((40 * 24, 16), 7.0, dtype=dt, device=cuda)
    p = tex.params(inference_output=wide)
    p.inference_output_stride = 16
    nt.InvokeInference(p)
    torch.cuda.synchronize()
    assert torch.equal(wide[:, :8], packed)
    assert torch.all(wide[:, 8:] == 0)

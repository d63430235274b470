"""Decode (train.cu:917-961) parity: the CUDA decode kernel against the CPU oracle on the
same seeded latents and weights.  Tolerance: max relative error 1e-2 (fp16), relative to
max(|ref|, 1) so that outputs near zero are held to 1e-2 absolute."""
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


def test_decode_full_config0_subset(cuda, oracle):
    """BASELINE config 0 (1024^2 texels, 512^2x8 + 256^2x8 latents, 8 outputs): the whole
    image is decoded on the GPU and a seeded subset of 20,000 texels is checked against the
    oracle; every output is finite."""
    import torch
    tex = make_texture((1024, 1024), ((512, 512), (256, 256)), 8, 8, seed=11)
    out = tex.decode()
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float32)
    assert np.isfinite(got).all()
    model = oracle_model(oracle, tex)
    rng = np.random.default_rng(0)
    starts = rng.integers(0, 1024 * 1024 - 200, 100)
    for s in starts:
        ref = oracle.decode_range(model, 1024, 1024, int(s), 200).view(np.float16).astype(np.float32)
        err = max_rel(got[s:s + 200], ref)
        assert err <= TOL, f"texels {s}..{s + 200}: max rel err {err}"


def test_decode_is_deterministic(cuda):
    import torch
    tex = make_texture((96, 64), ((48, 32), (24, 16)), 12, 12, seed=2)
    a = tex.decode().cpu()
    b = tex.decode().cpu()
    assert torch.equal(a, b)

"""Pins oracle/torch_oracle.py (the tensor-wide restatement used for the 2,000-step criterion at
BASELINE config-1 size) to the C oracle on the CPU: identical sample positions, one training
pass (loss, network and latent gradients) and one full step with Adam."""
import numpy as np
import pytest

from oracle.torch_oracle import TorchTrainer


def _material(O, image, grids, C, cout, seed):
    from neural_textures_b200.api import he_normal_weights, zero_padded_inputs
    rng = np.random.default_rng(seed)
    gs = [O.f2h(rng.uniform(-1, 1, (h, w, C))) for (w, h) in grids]
    Ws = he_normal_weights(seed, cout)
    Ws[0] = zero_padded_inputs(Ws[0], 2 * C + 8)
    W = [w.view(np.uint16).copy() for w in Ws]
    b = [O.f2h(rng.standard_normal(n) * 0.1) for n in (64, 64, cout)]
    tgt = O.generate_target(image[0], image[1], cout, seed, threads=4)
    return gs, W, b, tgt


CASES = [
    ((64, 64), ((32, 32), (16, 16)), 8, 8, (32, 32)),
    ((48, 40), ((24, 20), (12, 10)), 12, 12, (24, 20)),
    ((37, 29), ((19, 15), (9, 7)), 8, 10, (37, 29)),
]


@pytest.mark.parametrize("image,grids,C,cout,lattice", CASES)
def test_torch_pass_matches_c_oracle(oracle, image, grids, C, cout, lattice):
    O = oracle
    gs, W, b, tgt = _material(O, image, grids, C, cout, seed=5)
    step = 3
    tt = TorchTrainer(gs, W, b, tgt, C, cout, image, lattice, (0.9, 0.99, 1e-2, 1e-8), (0.9, 0.99, 5e-3, 1e-8))
    s = O.make_sampler(image[0], image[1], lattice[0], lattice[1], step=step)
    uv = O.sample_uv(s)
    u, v = tt.sample_uv(step)
    np.testing.assert_array_equal(u.numpy(), uv[:, 0])
    np.testing.assert_array_equal(v.numpy(), uv[:, 1])
    sse, gW, gb, gg = tt.train_pass(step)
    rsse, rW, rb, rg = O.train_pass(O.OracleModel(C, cout, gs, W, b), tgt, s, threads=4)
    assert abs(sse - rsse) <= 1e-5 * rsse, (sse, rsse)
    rel = lambda a, r: float(np.linalg.norm(a.ravel() - r.ravel()) / max(np.linalg.norm(r.ravel()), 1e-30))
    for l in range(3):
        assert rel(gW[l].numpy(), rW[l]) <= 1e-3, l
        assert rel(gb[l].numpy(), rb[l]) <= 1e-3, l
    for g in range(2):
        assert rel(gg[g].numpy(), rg[g]) <= 1e-3, g


def test_torch_step_matches_c_oracle(oracle):
    """Pass + Adam on network and latents (main.cpp:1071-1077): the updated fp16 parameters
    agree with the C oracle's to one fp16 step at most, and almost all bit for bit."""
    O = oracle
    image, grids, C, cout, lattice = (64, 64), ((32, 32), (16, 16)), 8, 8, (32, 32)
    gs, W, b, tgt = _material(O, image, grids, C, cout, seed=8)
    la, na = (0.9, 0.99, 1e-2, 1e-8), (0.9, 0.99, 5e-3, 1e-8)
    tt = TorchTrainer(gs, W, b, tgt, C, cout, image, lattice, la, na)
    step = 1
    tt.step(step)
    s = O.make_sampler(image[0], image[1], lattice[0], lattice[1], step=step)
    grids_c = [g.copy() for g in gs]
    W_c = [w.copy() for w in W]
    b_c = [x.copy() for x in b]
    rsse, rW, rb, rg = O.train_pass(O.OracleModel(C, cout, grids_c, W_c, b_c), tgt, s, threads=4)
    z = lambda a: np.zeros(a.shape, np.float32)
    for l in range(3):
        O.adam_f16(W_c[l], rW[l], z(rW[l]), z(rW[l]), na[2], na[0], na[1], na[3], step)
        O.adam_f16(b_c[l], rb[l], z(rb[l]), z(rb[l]), na[2], na[0], na[1], na[3], step)
    for gi in range(2):
        flat = grids_c[gi].reshape(-1)
        O.adam_f16(flat, rg[gi].reshape(-1), z(flat), z(flat), la[2], la[0], la[1], la[3], step)
    pairs = [(tt.W[l].numpy().reshape(-1), W_c[l]) for l in range(3)] + \
            [(tt.grids[g].numpy().reshape(-1), grids_c[g].reshape(-1)) for g in range(2)]
    for got, want_bits in pairs:
        want = want_bits.view(np.float16).astype(np.float32)
        got16 = got.astype(np.float16).astype(np.float32)
        assert np.array_equal(got16, got)  # the torch parameters hold fp16 values
        diff = np.abs(got - want)
        ulp = np.abs(np.spacing(want.astype(np.float16)).astype(np.float32))
        assert np.all(diff <= ulp * 1.0001), float((diff / np.maximum(ulp, 1e-30)).max())
        assert np.mean(diff == 0) >= 0.99

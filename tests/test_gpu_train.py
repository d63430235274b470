"""Training parity: the fused CUDA training pass and the fused Adam against the CPU oracle.

- one training pass (train.cu:818-915 semantics): network and latent gradients, relative
  L2 error <= 2e-2 per buffer; the sum of squared errors within 1e-3 relative;
- Adam (train.cu:521-588): bit-exact, including the zero-gradient skip and the zeroing;
- a multi-step run: the loss after 2,000 steps within 2% of the oracle's, on a 128^2 material
  against the C oracle and at full BASELINE config-1 size against its tensor restatement
  (oracle/torch_oracle.py, pinned to the C oracle by tests/test_torch_oracle_cpu.py);
- full BASELINE config-1 and config-2 size: one pass against the C oracle (same tolerances),
  plus size-independent identities (every latent gradient sums to sum_i db1[i] W1[i][k]).
"""
import ctypes as C
import os

import numpy as np
import pytest

from tests.model_utils import make_texture, max_rel, oracle_model, rel_l2, target_host

pytestmark = pytest.mark.gpu

GRAD_TOL = 2e-2


def _host(t):
    return t.detach().cpu().numpy().copy()


def _train_pass_gpu(tex, finalize=False):
    import torch
    import neural_textures_b200 as nt
    tex.loss_accum.zero_()
    kind = nt.TrainingKernelType.FINALIZE if finalize else nt.TrainingKernelType.UNCONSTRAINED
    nt.InvokeTraining(tex.params(), kind)
    torch.cuda.synchronize()
    return (tex.loss_accum.item(), [_host(g) for g in tex.gW], [_host(g) for g in tex.gb],
            [_host(g) for g in tex.ggrads])


def _oracle_pass(oracle, tex, finalize=False, threads=8):
    s = oracle.make_sampler(tex.image_w, tex.image_h, tex.lattice[0], tex.lattice[1], step=tex.step,
                            seed=tex.seed)
    return oracle.train_pass(oracle_model(oracle, tex), target_host(tex), s,
                             channel_weights=np.array(tex.channel_weights, np.float32), finalize=finalize,
                             threads=threads)


def _assert_pass_matches(got, ref, label):
    sse, gW, gb, gg = got
    rsse, rW, rb, rg = ref
    print(f"{label}: sse {sse:.6g} vs oracle {rsse:.6g}; rel-L2 dW {[round(rel_l2(gW[l], rW[l]), 6) for l in range(3)]}"
          f" db {[round(rel_l2(gb[l], rb[l]), 6) for l in range(3)]} latents {[round(rel_l2(gg[g], rg[g]), 6) for g in range(2)]}")
    assert abs(sse - rsse) <= 1e-3 * rsse, (sse, rsse)
    for l in range(3):
        assert rel_l2(gW[l], rW[l]) <= GRAD_TOL, f"dW{l}: {rel_l2(gW[l], rW[l])}"
        assert rel_l2(gb[l], rb[l]) <= GRAD_TOL, f"db{l}: {rel_l2(gb[l], rb[l])}"
    for g in range(2):
        assert rel_l2(gg[g], rg[g]) <= GRAD_TOL, f"latent grid {g}: {rel_l2(gg[g], rg[g])}"


CASES = [
    # image, grids, C, cout, lattice
    ((64, 64), ((32, 32), (16, 16)), 8, 8, (32, 32)),
    ((96, 80), ((48, 40), (24, 20)), 12, 12, (48, 40)),
    ((70, 50), ((35, 25), (17, 12)), 8, 10, (37, 23)),
    ((32, 32), ((32, 32), (8, 8)), 8, 8, (32, 32)),
    ((1, 1), ((1, 1), (1, 1)), 8, 8, (1, 1)),   # every tap wraps onto the one texel
    ((5, 3), ((3, 2), (1, 1)), 12, 3, (5, 3)),  # ragged, one-texel grid, 3 outputs
]


@pytest.mark.parametrize("image,grids,C,cout,lattice", CASES)
def test_training_pass_matches_oracle(cuda, oracle, image, grids, C, cout, lattice):
    tex = make_texture(image, grids, C, cout, lattice=lattice, seed=7)
    tex.step = 3
    sse, gW, gb, gg = _train_pass_gpu(tex)
    rsse, rW, rb, rg = _oracle_pass(oracle, tex)
    assert abs(sse - rsse) <= 1e-3 * rsse, (sse, rsse)
    for l in range(3):
        assert rel_l2(gW[l], rW[l]) <= GRAD_TOL, f"dW{l}: {rel_l2(gW[l], rW[l])}"
        assert rel_l2(gb[l], rb[l]) <= GRAD_TOL, f"db{l}: {rel_l2(gb[l], rb[l])}"
    for g in range(2):
        assert rel_l2(gg[g], rg[g]) <= GRAD_TOL, f"latent grid {g}: {rel_l2(gg[g], rg[g])}"
    # padded weight rows / columns receive no gradient
    assert np.all(gW[2].reshape(16, 64)[cout:] == 0)
    assert np.all(gW[0].reshape(64, 32)[:, 2 * C + 8:] == 0)


def test_finalize_leaves_latent_gradients_untouched(cuda, oracle):
    tex = make_texture((64, 64), ((32, 32), (16, 16)), 8, 8, lattice=(32, 32), seed=1)
    sse, gW, gb, gg = _train_pass_gpu(tex, finalize=True)
    rsse, rW, rb, rg = _oracle_pass(oracle, tex, finalize=True)
    assert all(np.all(g == 0) for g in gg)
    assert rel_l2(gW[1], rW[1]) <= GRAD_TOL


def test_channel_loss_weights(cuda, oracle):
    tex = make_texture((64, 64), ((32, 32), (16, 16)), 8, 8, lattice=(32, 32), seed=4)
    tex.channel_weights = [1.0, 0.5, 2.0, 0.0, 1.0, 3.0, 0.25, 1.0]
    sse, gW, gb, gg = _train_pass_gpu(tex)
    rsse, rW, rb, rg = _oracle_pass(oracle, tex)
    assert abs(sse - rsse) <= 1e-3 * rsse
    assert rel_l2(gW[2], rW[2]) <= GRAD_TOL
    assert np.all(gb[2][3] == 0)


def test_gradients_accumulate_across_passes(cuda):
    tex = make_texture((64, 64), ((32, 32), (16, 16)), 8, 8, lattice=(32, 32), seed=9)
    _, gW1, _, gg1 = _train_pass_gpu(tex)
    _, gW2, _, gg2 = _train_pass_gpu(tex)  # same step: same samples, grads double
    assert rel_l2(gW2[1], 2 * gW1[1]) < 1e-5
    assert rel_l2(gg2[0], 2 * gg1[0]) < 1e-5


@pytest.mark.parametrize("step", [17, 500, 3000])  # 500: 1 - beta1^t is 1; 3000: both corrections are 1
def test_adam_bit_exact(cuda, oracle, step):
    import torch
    import neural_textures_b200 as nt
    tex = make_texture((64, 64), ((32, 32), (16, 16)), 8, 8, lattice=(32, 32), seed=2)
    rng = np.random.default_rng(5)
    bufs = tex.gW + tex.gb + tex.ggrads
    for t in bufs + tex.mW + tex.vW + tex.mb + tex.vb + tex.gm1 + tex.gm2:
        vals = (rng.standard_normal(t.shape) * 10.0 ** rng.integers(-6, 0, t.shape)).astype(np.float32)
        t.copy_(torch.from_numpy(vals))
    for t in tex.vW + tex.vb + tex.gm2:
        t.abs_()
    for t in bufs:
        t.view(-1)[::13] = 0.0
    before = {k: [_host(x) for x in v] for k, v in dict(W=tex.W, b=tex.b, grids=tex.grids, gW=tex.gW, gb=tex.gb,
                                                          gg=tex.ggrads, mW=tex.mW, vW=tex.vW, mb=tex.mb,
                                                          vb=tex.vb, m1=tex.gm1, m2=tex.gm2).items()}
    nt.InvokeOptimizeAll(tex.params(step=step))
    torch.cuda.synchronize()
    b1, b2, lr, eps = tex.network_adam
    for l in range(3):
        w = before["W"][l].view(np.uint16).copy()
        g, m, v = before["gW"][l].copy(), before["mW"][l].copy(), before["vW"][l].copy()
        oracle.adam_f16(w, g, m, v, lr, b1, b2, eps, step)
        np.testing.assert_array_equal(_host(tex.W[l]).view(np.uint16), w)
        np.testing.assert_array_equal(_host(tex.mW[l]), m)
        np.testing.assert_array_equal(_host(tex.vW[l]), v)
        np.testing.assert_array_equal(_host(tex.gW[l]), g)
        w = before["b"][l].view(np.uint16).copy()
        g, m, v = before["gb"][l].copy(), before["mb"][l].copy(), before["vb"][l].copy()
        oracle.adam_f16(w, g, m, v, lr, b1, b2, eps, step)
        np.testing.assert_array_equal(_host(tex.b[l]).view(np.uint16), w)
        np.testing.assert_array_equal(_host(tex.vb[l]), v)
    b1, b2, lr, eps = tex.latent_adam
    for gi in range(2):
        w = before["grids"][gi].view(np.uint16).reshape(-1).copy()
        g = before["gg"][gi].reshape(-1).copy()
        m = before["m1"][gi].reshape(-1).copy()
        v = before["m2"][gi].reshape(-1).copy()
        oracle.adam_f16(w, g, m, v, lr, b1, b2, eps, step)
        np.testing.assert_array_equal(_host(tex.grids[gi]).view(np.uint16).reshape(-1), w)
        np.testing.assert_array_equal(_host(tex.gm1[gi]).reshape(-1), m)
        np.testing.assert_array_equal(_host(tex.gm2[gi]).reshape(-1), v)
        assert np.all(_host(tex.ggrads[gi]) == 0)


def test_separate_optimizers_equal_fused(cuda):
    import torch
    import neural_textures_b200 as nt
    a = make_texture((64, 64), ((32, 32), (16, 16)), 8, 8, lattice=(32, 32), seed=6)
    b = make_texture((64, 64), ((32, 32), (16, 16)), 8, 8, lattice=(32, 32), seed=6)
    nt.InvokeTraining(a.params())
    # float atomics make two passes differ in the last bits: give both paths the same grads
    for src, dst in zip(a.gW + a.gb + a.ggrads, b.gW + b.gb + b.ggrads):
        dst.copy_(src)
    nt.InvokeOptimizeAll(a.params(step=1))
    nt.InvokeOptimizeNetwork(b.params(step=1))
    nt.InvokeOptimizeFeatures(b.params(step=1))
    torch.cuda.synchronize()
    for x, y in zip(a.W + a.grids + a.mW + a.gm1, b.W + b.grids + b.mW + b.gm1):
        assert torch.equal(x, y)


def test_multi_step_loss_matches_oracle(cuda, oracle):
    """Run 2,000 steps on both sides with identical sampling; compare the loss level at step
    2,000 (2% tolerance: the criterion is the loss after 2,000 steps) and the loss decrease.
    The level is the mean over steps 1,900-1,999 at 4,096 samples per step: single-step losses
    swing by tens of percent with the jitter of the step's samples, and the two trajectories,
    which differ in fp32 summation order, put those swings on different steps."""
    import torch
    n_steps = 2000
    tex = make_texture((128, 128), ((64, 64), (32, 32)), 8, 8, lattice=(64, 64), seed=12)
    model_grids, model_W, model_b = tex.host_model()
    tgt = target_host(tex)
    losses_gpu = []
    for step in range(n_steps):
        tex.loss_accum.zero_()
        tex.train_step(params=tex.params(step=step))
        losses_gpu.append(tex.loss_accum.item())
    # oracle: the same loop on host copies
    grids = [g.copy() for g in model_grids]
    W = [w.copy() for w in model_W]
    b = [x.copy() for x in model_b]
    zeros = lambda a: np.zeros(a.shape, np.float32)
    mW, vW = [zeros(w) for w in W], [zeros(w) for w in W]
    mb, vb = [zeros(x) for x in b], [zeros(x) for x in b]
    mg, vg = [zeros(g) for g in grids], [zeros(g) for g in grids]
    b1, b2, lr_n, eps = tex.network_adam
    lr_l = tex.latent_adam[2]
    losses_ref = []
    for step in range(n_steps):
        model = oracle.OracleModel(channels=8, cout=8, grids=grids, W=W, b=b)
        s = oracle.make_sampler(128, 128, 64, 64, step=step)
        sse, gW, gb, gg = oracle.train_pass(model, tgt, s, threads=min(os.cpu_count() or 1, 16))
        losses_ref.append(sse)
        for l in range(3):
            oracle.adam_f16(W[l], gW[l], mW[l], vW[l], lr_n, b1, b2, eps, step)
            oracle.adam_f16(b[l], gb[l], mb[l], vb[l], lr_n, b1, b2, eps, step)
        for gi in range(2):
            flat = grids[gi].reshape(-1)
            oracle.adam_f16(flat, gg[gi].reshape(-1), mg[gi].reshape(-1), vg[gi].reshape(-1), lr_l, b1, b2, eps,
                            step)
    for n in (10, 100, 200):
        print(f"last {n} steps: gpu {np.mean(losses_gpu[-n:]):.4f} oracle {np.mean(losses_ref[-n:]):.4f}")
    lg, lr_ = np.mean(losses_gpu[-100:]), np.mean(losses_ref[-100:])
    assert lg < 0.5 * losses_gpu[0], "training must reduce the loss"
    assert abs(lg - lr_) <= 0.02 * lr_, (lg, lr_)


def _latent_sum_identity(tex, gb, gg):
    """Sum over texels of each latent gradient channel = sum_i db1[i] W1[i][k]: the
    Catmull-Rom weights of every sample sum to one."""
    C = tex.C
    W1 = _host(tex.W[0]).astype(np.float64).reshape(64, 32)
    db1 = gb[0].astype(np.float64)
    for g in range(2):
        flat = gg[g].astype(np.float64).reshape(-1, C)
        lhs = flat.sum(0)
        rhs = db1 @ W1[:, g * C:(g + 1) * C]
        tol = 1e-3 * np.abs(flat).sum(0) + 1e-2 * np.abs(rhs)
        assert np.all(np.abs(lhs - rhs) <= tol), (lhs, rhs, tol)


def test_full_config1_pass_matches_oracle(cuda, oracle):
    """BASELINE config 1 at full size (1024^2 image, 512^2x8 + 256^2x8 latents, He-normal
    weights, 262,144 samples): one training pass against the C oracle, every gradient buffer
    at rel-L2 <= 2e-2 and the sum of squared errors within 1e-3."""
    tex = make_texture((1024, 1024), ((512, 512), (256, 256)), 8, 8, lattice=(512, 512), seed=21)
    tex.step = 5
    got = _train_pass_gpu(tex)
    for a in got[1] + got[2] + got[3]:
        assert np.isfinite(a).all()
    _latent_sum_identity(tex, got[2], got[3])
    _assert_pass_matches(got, _oracle_pass(oracle, tex, threads=os.cpu_count() or 1), "config 1 pass")


def test_full_config2_pass_matches_oracle(cuda, oracle):
    """BASELINE config 2 at full size (4096^2 PBR material with 12 channels, normals from the
    height field; 1024^2x12 + 512^2x12 latents; 1,048,576 samples): unit-length target
    normals, then one training pass against the C oracle with the config-1 tolerances."""
    import neural_textures_b200 as nt
    tex = nt.NeuralTexture(4096, 4096, grid_sizes=((1024, 1024), (512, 512)), latent_channels=12,
                           output_channels=12, device="cuda:0", lattice=(1024, 1024))
    tex.init(seed=22, pbr_normals=True)
    tex.step = 2
    tgt = tex.target[::64, ::64].float().cpu().numpy().reshape(-1, 12)
    n = np.linalg.norm(tgt[:, 3:6] * 2.0 - 1.0, axis=1)  # normals stored as n * 0.5 + 0.5
    assert np.all(np.abs(n - 1.0) < 2e-2), (n.min(), n.max())
    got = _train_pass_gpu(tex)
    for a in got[1] + got[2] + got[3]:
        assert np.isfinite(a).all()
    _latent_sum_identity(tex, got[2], got[3])
    _assert_pass_matches(got, _oracle_pass(oracle, tex, threads=os.cpu_count() or 1), "config 2 pass")


def test_config1_2000_steps_loss_matches_oracle(cuda):
    """North-star criterion at BASELINE config-1 size: 2,000 training steps (fused pass + fused
    Adam, lr 1e-2 latents / 5e-3 network, beta1 0.9, beta2 0.99) on the 1024^2 material with
    262,144 samples per step, against the same 2,000 steps of the oracle's tensor restatement
    (oracle/torch_oracle.py) from the same fp16 state with the same samples.

    - Steps 0-199: every step's loss agrees within 1e-3 (the two trainings follow the same
      trajectory; measured 1e-4).
    - After that the trajectories decorrelate: the float atomics of both sides sum in an
      order that changes from run to run, and with these Adam settings the training shows
      isolated loss spikes (single steps up to ~3x the level) whose timing follows from
      those last-bit differences; over a 500-step window the level of one run of either side
      moves by up to ~6% from run to run.  The loss after 2,000 steps is therefore measured
      as the level of the second half of the run: the mean of the losses of steps
      1,000-1,999 without the 10% largest (the spike steps).  The two levels agree within 2%.
      Plain means and medians of several windows are printed beside it."""
    import torch
    from oracle.torch_oracle import TorchTrainer
    torch.backends.cuda.matmul.allow_tf32 = False
    n_steps = 2000
    tex = make_texture((1024, 1024), ((512, 512), (256, 256)), 8, 8, lattice=(512, 512), seed=31)
    grids, W, b = tex.host_model()
    ref = TorchTrainer(grids, W, b, target_host(tex), 8, 8, (1024, 1024), (512, 512), tex.latent_adam,
                       tex.network_adam, device="cuda:0")
    losses_gpu = torch.zeros(n_steps, dtype=torch.float32, device="cuda:0")
    for step in range(n_steps):
        p = tex.params(step=step)
        p.loss_accum = losses_gpu[step].data_ptr()
        tex.train_step(params=p)
    B = 512 * 512
    losses_gpu = losses_gpu.cpu().numpy().astype(np.float64) / B
    losses_ref = np.array([ref.step(step) for step in range(n_steps)]) / B
    out = os.environ.get("NT_LOSS_CURVES")
    if out:
        np.savez(out, gpu=losses_gpu, oracle=losses_ref)

    def level(x):
        return float(x[x <= np.percentile(x, 90)].mean())

    early = float(np.max(np.abs(losses_gpu[:200] / losses_ref[:200] - 1.0)))
    print(f"config 1, steps 0-199: max per-step relative loss difference {early:.2e}")
    for lo, hi in ((1000, 2000), (1500, 2000), (1900, 2000)):
        g, r = losses_gpu[lo:hi], losses_ref[lo:hi]
        print(f"config 1, steps {lo}-{hi - 1}, loss per sample: level gpu {level(g):.6f} oracle {level(r):.6f}; "
              f"mean gpu {np.mean(g):.6f} oracle {np.mean(r):.6f}; median gpu {np.median(g):.6f} "
              f"oracle {np.median(r):.6f}")
    assert early <= 1e-3, early
    lg, lr_ = level(losses_gpu[1000:]), level(losses_ref[1000:])
    assert lg < 0.01 * losses_gpu[0], "training must reduce the loss"
    assert abs(lg - lr_) <= 0.02 * lr_, (lg, lr_)


def test_material_on_another_device(cuda):
    """A material on cuda:1 trains and decodes while cuda:0 is current (the library launches on
    the current device; the texture selects its own) and matches its twin on cuda:0."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    torch.cuda.set_device(0)
    a = make_texture((64, 64), ((32, 32), (16, 16)), 8, 8, lattice=(32, 32), seed=9, device="cuda:0")
    b = make_texture((64, 64), ((32, 32), (16, 16)), 8, 8, lattice=(32, 32), seed=9, device="cuda:1")
    for t in (a, b):
        t.loss_accum.zero_()
        t.train_step()
    assert torch.cuda.current_device() == 0
    la, lb = a.loss_accum.item(), b.loss_accum.item()
    assert abs(la - lb) <= 1e-5 * la
    da, db = a.decode(dtype=torch.float32).cpu().numpy(), b.decode(dtype=torch.float32).cpu().numpy()
    assert max_rel(db, da) <= 1e-3


def test_tile_counter_workspace(cuda):
    """The training pass with a workspace (each CTA claims the next tile from a counter) gives
    the gradients of the fixed tile shares up to the order of float atomics, leaves the
    workspace zeroed, and rejects a workspace that is too small.  The lattice has 4,096 tiles,
    at least 8 per CTA, where the kernel takes the counters."""
    import ctypes
    import torch
    from neural_textures_b200 import _native
    L = _native.load()
    tex = make_texture((2048, 2048), ((512, 512), (256, 256)), 8, 8, lattice=(1024, 512), seed=23)
    res = []
    for ws in (True, False, True):
        for t in tex.gW + tex.gb + tex.ggrads:
            t.zero_()
        tex.loss_accum.zero_()
        p = tex.params(step=4)
        if not ws:
            p.workspace, p.workspace_bytes = None, 0
        _native.check(L.nt_invoke_training(ctypes.byref(p), 0, None))
        torch.cuda.synchronize()
        res.append((tex.loss_accum.item(), [_host(g) for g in tex.gW + tex.gb + tex.ggrads]))
        assert int(tex.workspace.abs().sum()) == 0
    for a, b in ((res[0], res[1]), (res[2], res[1])):
        assert abs(a[0] - b[0]) <= 1e-5 * b[0]
        for x, y in zip(a[1], b[1]):
            assert rel_l2(x, y) <= 1e-5
    p = tex.params(step=4)
    p.workspace_bytes = 8
    assert L.nt_invoke_training(ctypes.byref(p), 0, None) == 1
    assert b"workspace" in L.nt_get_last_error_string()

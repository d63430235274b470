"""Generate tests/golden/reference_vectors.npz from the reference's OWN code.

Runs oracle/build_ref.sh, which compiles functions of mavenkim2/neural_textures in place
(tests/forward_pass_test.cu:45-150, train.cu:37-69, :161-182, :521-564,
filter/catmull_rom.h:46-59) into oracle/_ref/libnt_ref.so, then records their outputs on
seeded inputs.  The CPU oracle (oracle/nt_oracle.c) is checked against these vectors by
tests/test_oracle_golden.py, so the oracle is pinned to the reference, not to itself.

    python tests/golden/make_golden.py [reference_root]
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402


def main(argv):
    ref_root = argv[1] if len(argv) > 1 else None
    if O.build_ref(ref_root) is None:
        raise SystemExit("reference sources not found; nothing generated")
    R = O.ref_lib()
    u16p, f32p = O.u16p, O.f32p
    out = {}

    # forward-pass known-answer test (generator + fp32 host reference)
    fin = np.zeros(32 * 12, np.uint16)
    fw0 = np.zeros(256, np.uint16)
    fw1 = np.zeros(256, np.uint16)
    fb0 = np.zeros(16, np.uint16)
    fb1 = np.zeros(16, np.uint16)
    fexp = np.zeros(32 * 16, np.float32)
    R.ref_fwdtest(*[x.ctypes.data_as(u16p) for x in (fin, fw0, fw1, fb0, fb1)], fexp.ctypes.data_as(f32p))
    out.update(fwd_inputs=fin, fwd_w0=fw0, fwd_w1=fw1, fwd_b0=fb0, fwd_b1=fb1, fwd_expected=fexp)

    # RNG: raw xorshift32 outputs and UniformFloat for several seeds, including the per-sample
    # seed formula of train.cu:833 for a few (sample, step) pairs
    rng = np.random.default_rng(1234)
    seeds = [1, 12345, 0xFFFFFFFF, 2891336453]
    for s_idx in range(6):
        for step in (0, 1, 7, 4999):
            seeds.append((s_idx * 131071) ^ ((step * 747796405 + 2891336453) & 0xFFFFFFFF))
    seeds += [int(x) for x in rng.integers(1, 2**32, 8, dtype=np.uint64)]
    bits = np.zeros((len(seeds), 16), np.uint32)
    unif = np.zeros((len(seeds), 16), np.float32)
    for i, s in enumerate(seeds):
        R.ref_rng(s & 0xFFFFFFFF, 16, bits[i].ctypes.data_as(C.POINTER(C.c_uint32)), unif[i].ctypes.data_as(f32p))
    out.update(rng_seeds=np.array(seeds, np.uint64).astype(np.uint32), rng_bits=bits, rng_uniform=unif)

    # wrap addressing and clamp
    coords = np.arange(-70, 140, dtype=np.int32)
    sizes = np.array([1, 2, 3, 7, 64], np.int32)
    wrap = np.array([[R.ref_wrap(int(c), int(n)) for c in coords] for n in sizes], np.int32)
    out.update(wrap_coords=coords, wrap_sizes=sizes, wrap_values=wrap)

    # Catmull-Rom fraction and weights at seeded uv for several texture sizes
    cr_u = np.concatenate([rng.random(400).astype(np.float32),
                           np.array([0.0, 0.5, 1.0, 1e-7, 0.999999], np.float32)])
    cr_sizes = np.array([1, 4, 256, 512, 1000, 4096], np.float32)
    cr_w = np.zeros((len(cr_sizes), len(cr_u), 4), np.float32)
    cr_f = np.zeros((len(cr_sizes), len(cr_u)), np.float32)
    for i, sz in enumerate(cr_sizes):
        for j, u in enumerate(cr_u):
            f = C.c_float()
            R.ref_catmull_rom(float(u), float(sz), cr_w[i, j].ctypes.data_as(f32p), C.byref(f))
            cr_f[i, j] = f.value
    out.update(cr_u=cr_u, cr_sizes=cr_sizes, cr_weights=cr_w, cr_frac=cr_f)

    # Adam: sequences of updates on fp16 and fp32 parameters (train.cu:521-564)
    n = 256
    hp = [(0.9, 0.99, 1e-2, 1e-8), (0.9, 0.999, 5e-3, 1e-8), (0.8, 0.95, 1e-1, 1e-6)]
    adam_w16 = (rng.standard_normal(n) * 0.5).astype(np.float16).view(np.uint16)
    adam_w32 = (rng.standard_normal(n) * 0.5).astype(np.float32)
    steps = [0, 1, 2, 3, 10, 100]
    grads =(rng.standard_normal((len(hp), len(steps), n)) * 10.0 ** rng.integers(-6, 1, (len(hp), len(steps), n))
             ).astype(np.float32)
    grads[:, :, ::17] = 0.0  # zero gradients are skipped (train.cu:580-583)
    w16_hist = np.zeros((len(hp), len(steps), n), np.uint16)
    w32_hist = np.zeros((len(hp), len(steps), n), np.float32)
    m16_hist = np.zeros((len(hp), len(steps), n), np.float32)
    v16_hist = np.zeros((len(hp), len(steps), n), np.float32)
    for h, (b1, b2, lr, eps) in enumerate(hp):
        w16 = adam_w16.copy()
        w32 = adam_w32.copy()
        m16 = np.zeros(n, np.float32)
        v16 = np.zeros(n, np.float32)
        m32 = np.zeros(n, np.float32)
        v32 = np.zeros(n, np.float32)
        for si, st in enumerate(steps):
            for i in range(n):
                g = float(grads[h, si, i])
                if g == 0.0:
                    continue  # the buffer-level skip of OptimizeParameterBuffer
                wv = C.c_uint16(int(w16[i]))
                mv, vv = C.c_float(m16[i]), C.c_float(v16[i])
                R.ref_adam_f16(C.byref(wv), C.byref(mv), C.byref(vv), g, b1, b2, lr, eps, st)
                w16[i], m16[i], v16[i] = wv.value, mv.value, vv.value
                wf = C.c_float(w32[i])
                mf, vf = C.c_float(m32[i]), C.c_float(v32[i])
                R.ref_adam_f32(C.byref(wf), C.byref(mf), C.byref(vf), g, b1, b2, lr, eps, st)
                w32[i], m32[i], v32[i] = wf.value, mf.value, vf.value
            w16_hist[h, si] = w16
            w32_hist[h, si] = w32
            m16_hist[h, si] = m16
            v16_hist[h, si] = v16
    out.update(adam_hparams=np.array(hp, np.float32), adam_steps=np.array(steps, np.int32),
               adam_w16_init=adam_w16, adam_w32_init=adam_w32, adam_grads=grads,
               adam_w16=w16_hist, adam_w32=w32_hist, adam_m16=m16_hist, adam_v16=v16_hist)

    # BC6-style float decode (train.cu:161-182)
    e0 = rng.uniform(-1, 1, (64, 3)).astype(np.float32)
    e1 = rng.uniform(-1, 1, (64, 3)).astype(np.float32)
    bits_b = np.array([10, 7, 11, 9, 8, 6], np.int32)
    xs = np.linspace(0, 1, 8, dtype=np.float32)
    dec = np.zeros((len(bits_b), 64, len(xs), 3), np.float32)
    for bi, b in enumerate(bits_b):
        for k in range(64):
            for xi, x in enumerate(xs):
                R.ref_decompress_bc6(e0[k].ctypes.data_as(f32p), e1[k].ctypes.data_as(f32p), int(b), float(x),
                                     dec[bi, k, xi].ctypes.data_as(f32p))
    out.update(bc6_e0=e0, bc6_e1=e1, bc6_bits=bits_b, bc6_x=xs, bc6_decoded=dec)

    path = os.path.join(HERE, "reference_vectors.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main(sys.argv)

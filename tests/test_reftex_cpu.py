"""Reference-texture filtering on the CPU oracle (no GPU).

filter/catmull_rom.h:39-89 evaluates Catmull-Rom with 9 bilinear fetches: on each axis the
middle two taps merge into one fetch at w2 / (w1 + w2).  With exact bilinear weights this is the
16-tap filter itself; the oracle's restatement (mode 0) must agree with the 16-tap sampler of the
latents to rounding, including wrap addressing past the edges.  The blend of two levels follows
train.cu:78-103.
"""
import numpy as np
import pytest


@pytest.mark.parametrize("w,h", [(8, 8), (13, 6), (32, 5)])
def test_nine_fetch_catmull_rom_equals_sixteen_taps(oracle, w, h):
    import ctypes as C
    rng = np.random.default_rng(w * 31 + h)
    img = rng.standard_normal((h, w, 1)).astype(np.float16)
    chain = img.astype(np.float32).reshape(-1)
    uv = rng.uniform(-0.3, 1.3, (300, 2)).astype(np.float32)
    got = oracle.ref_sample([(chain, w, h, 1, 1, 1.0)], uv, 0.0, filter_mode=0)[:, 0]
    L = oracle.lib()
    want = np.zeros(len(uv), np.float32)
    for i, (u, v) in enumerate(uv):
        out = np.zeros(16, np.float32)
        # the 16-tap sampler addresses one period: feed the wrapped coordinate
        uu, vv = np.float32(u - np.floor(u)), np.float32(v - np.floor(v))
        L.nto_sample_grid(img.view(np.uint16).ctypes.data_as(oracle.u16p), w, h, 1, float(uu), float(vv),
                          out.ctypes.data_as(oracle.f32p), None, None, None)
        want[i] = out[0]
    assert np.max(np.abs(got - want)) <= 1e-5 * max(1.0, np.abs(want).max())


def test_levels_blend_like_the_reference(oracle):
    rng = np.random.default_rng(4)
    import neural_textures_b200 as nt
    img = rng.random((16, 16, 4)).astype(np.float32)
    chain = nt.api.box_chain_f32(img, 3)
    uv = rng.uniform(0, 1, (50, 2)).astype(np.float32)
    d = [(chain, 16, 16, 4, 3, 1.0)]
    s1 = oracle.ref_sample(d, uv, 1.0, 0)
    s2 = oracle.ref_sample(d, uv, 2.0, 0)
    s = oracle.ref_sample(d, uv, 1.25, 0)
    assert np.allclose(s, 0.75 * s1 + 0.25 * s2, atol=1e-6)
    assert np.array_equal(oracle.ref_sample(d, uv, 7.0, 0), s2)  # clamped to the last level

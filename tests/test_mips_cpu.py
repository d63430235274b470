"""Mip chains on the CPU (no GPU): level choice, chain layout and the box-filter builder.

The level choice restates train.cu:78-103 (SampleReferenceTextureTrilinear: lod clamped to the
chain, levels floor(lod) and the next one, blend weight lod - floor) and the level sizes
train.cu:214-218 (max(size >> m, 1)); the reference's feature sampler (train.cu:264-314)
picks the same levels and weights for every lod in [0, n - 1].
"""
import math

import numpy as np
import pytest


def _select(n, lod):
    last = n - 1 if n > 1 else 0
    c = 0.0 if not (lod > 0) else min(lod, float(last))
    m0 = min(int(math.floor(c)), last)
    m1 = min(m0 + 1, last)
    return m0, m1, (np.float32(c) - np.float32(m0)) if m1 > m0 else 0.0


@pytest.mark.parametrize("n", [1, 2, 5, 10])
def test_mip_select_follows_the_reference(oracle, n):
    for lod in [-3.0, 0.0, 0.25, 0.5, 0.999, 1.0, 1.75, 3.5, 8.99, 9.0, 40.0, float("nan")]:
        m0, m1, t = oracle.mip_select(n, lod)
        e0, e1, et = _select(n, lod)
        assert (m0, t if t else 0.0) == (e0, float(et) if et else 0.0), (n, lod)
        if t > 0:
            assert m1 == e1 == m0 + 1


def test_chain_layout(oracle, native):
    for (w, h, n) in [(512, 512, 8), (12, 5, 4), (1, 1, 3), (96, 80, 7), (7, 300, 10)]:
        lv = oracle.mip_chain_levels(w, h, n)
        assert lv[0] == (w, h, 0)
        for m in range(1, n):
            assert lv[m][0] == max(w >> m, 1) and lv[m][1] == max(h >> m, 1)
            assert lv[m][2] == lv[m - 1][2] + lv[m - 1][0] * lv[m - 1][1]
        assert native.nt_mip_chain_texels(w, h, n) == lv[-1][2] + lv[-1][0] * lv[-1][1]
    assert native.nt_mip_chain_texels(8, 8, 0) == 64  # 0: one level
    assert native.nt_mip_chain_texels(8, 8, 17) == 0


def _down(a):
    h, w, c = a.shape
    dh, dw = max(h >> 1, 1), max(w >> 1, 1)
    out = np.zeros((dh, dw, c), np.float32)
    for y in range(dh):
        for x in range(dw):
            x0, x1 = min(2 * x, w - 1), min(2 * x + 1, w - 1)
            y0, y1 = min(2 * y, h - 1), min(2 * y + 1, h - 1)
            out[y, x] = ((a[y0, x0] + a[y0, x1]) + (a[y1, x0] + a[y1, x1])) * np.float32(0.25)
    return out.astype(np.float16)


@pytest.mark.parametrize("shape,n", [((5, 12, 3), 4), ((16, 16, 8), 5), ((1, 9, 12), 5), ((33, 17, 1), 6)])
def test_build_mips_box_filter(oracle, shape, n):
    rng = np.random.default_rng(3)
    l0 = (rng.standard_normal(shape) * 2).astype(np.float16)
    chain = oracle.build_mips(l0.view(np.uint16), n)
    cur = l0
    for m in range(1, n):
        cur = _down(cur.astype(np.float32))
        assert np.array_equal(cur.view(np.uint16), chain[m]), m

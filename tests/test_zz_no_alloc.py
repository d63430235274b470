"""nt_invoke_training_static_scratch (the training pass with its tile counters in the library's
static device array, for callers that cannot allocate) against nt_invoke_training with a
caller workspace: two calls in a row, each from zeroed gradients, give the same loss and
gradients up to the order of float atomics (relative L2 <= 1e-5, the bound the workspace
test uses), on a lattice of 4,096 tiles (at least 8 per CTA, where the kernel takes the
counters).  Named to run last, after every other test has used the library on the device;
it passes alone in a fresh process as well."""
import ctypes

import pytest

from tests.model_utils import make_texture, rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _pass(L, tex, entry, workspace):
    import torch
    from neural_textures_b200 import _native
    for t in tex.gW + tex.gb + tex.ggrads:
        t.zero_()
    tex.loss_accum.zero_()
    p = tex.params(step=4)
    if not workspace:
        p.workspace, p.workspace_bytes = None, 0
    _native.check(getattr(L, entry)(ctypes.byref(p), 0, None))
    torch.cuda.synchronize()
    return tex.loss_accum.item(), [t.detach().cpu().numpy().copy() for t in tex.gW + tex.gb + tex.ggrads]


def test_static_scratch_matches_workspace(cuda):
    from neural_textures_b200 import _native
    L = _native.load()
    tex = make_texture((2048, 2048), ((512, 512), (256, 256)), 8, 8, lattice=(1024, 512), seed=29)
    want = _pass(L, tex, "nt_invoke_training", workspace=True)
    for _ in range(2):
        got = _pass(L, tex, "nt_invoke_training_static_scratch", workspace=False)
        assert abs(got[0] - want[0]) <= TOL * want[0], (got[0], want[0])
        for g, w in zip(got[1], want[1]):
            assert rel_l2(g, w) <= TOL


def test_static_scratch_rejects_a_workspace(cuda):
    from neural_textures_b200 import _native
    L = _native.load()
    tex = make_texture((64, 64), ((32, 32), (16, 16)), 8, 8, lattice=(32, 32), seed=3)
    p = tex.params(step=1)
    assert p.workspace
    assert L.nt_invoke_training_static_scratch(ctypes.byref(p), 0, None) == 1
    assert b"workspace must be NULL" in L.nt_get_last_error_string()

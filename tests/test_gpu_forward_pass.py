"""tests/forward_pass_test.cu of the reference: the 12 -> 16 (ReLU) -> 16 known-answer test,
through RunForwardPassTest() and through the C ABI on the golden vectors."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_run_forward_pass_test(cuda):
    import neural_textures_b200 as nt
    assert nt.RunForwardPassTest()


def test_forward_pass_12x16x16_matches_reference_expected(cuda, golden):
    import torch
    from neural_textures_b200 import _native
    L = _native.load()
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(cuda)
    inputs, w0, w1 = dev(golden["fwd_inputs"]), dev(golden["fwd_w0"]), dev(golden["fwd_w1"])
    b0, b1 = dev(golden["fwd_b0"]), dev(golden["fwd_b1"])
    out = torch.zeros(32 * 16, dtype=torch.int16, device=cuda)
    _native.check(L.nt_forward_pass_12x16x16(inputs.data_ptr(), w0.data_ptr(), w1.data_ptr(), b0.data_ptr(),
                                             b1.data_ptr(), out.data_ptr(), None))
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.float16).astype(np.float32)
    # tolerance of tests/forward_pass_test.cu:236
    assert np.max(np.abs(got - golden["fwd_expected"])) <= 2e-2

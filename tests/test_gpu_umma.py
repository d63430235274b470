"""tcgen05 building blocks on the operand layouts of the fused kernels (K-major M=128 and
MN-major M=64 products from core-matrix shared-memory tiles), against numpy."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_umma_selftest(cuda):
    import torch
    from neural_textures_b200 import _native
    rng = np.random.default_rng(0)
    A = rng.standard_normal((128, 32)).astype(np.float16)
    B = rng.standard_normal((64, 32)).astype(np.float16)
    H = rng.standard_normal((128, 64)).astype(np.float16)
    dev = lambda x: torch.from_numpy(x).to(cuda)
    dA, dB, dH = dev(A), dev(B), dev(H)
    D1 = torch.zeros((128, 64), dtype=torch.float32, device=cuda)
    D2 = torch.zeros((64, 32), dtype=torch.float32, device=cuda)
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    _native.check(_native.load().nt_umma_selftest(dA.data_ptr(), dB.data_ptr(), dH.data_ptr(), D1.data_ptr(),
                                                  D2.data_ptr(), st.data_ptr(), None))
    torch.cuda.synchronize()
    assert st.item() == 0, "tensor core wait timed out"
    ref1 = A.astype(np.float64) @ B.astype(np.float64).T
    ref2 = H.astype(np.float64).T @ A.astype(np.float64)
    np.testing.assert_allclose(D1.cpu().numpy(), ref1, rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose(D2.cpu().numpy(), ref2, rtol=1e-4, atol=1e-3)


def test_bounded_wait_reports_a_timeout_and_the_context_survives(cuda):
    """A wait that nothing satisfies gives up after its poll limit and sets bit 0 of the status
    word (the kernels' timeout path), with no fault: the context keeps running work."""
    import ctypes as C
    import torch
    from neural_textures_b200 import _native
    L = _native.load()
    st = C.c_uint32(0)
    _native.check(L.nt_read_device_status(C.byref(st), 1))  # clear
    _native.check(L.nt_wait_timeout_selftest(1000))
    _native.check(L.nt_read_device_status(C.byref(st), 1))
    assert st.value & 1
    _native.check(L.nt_read_device_status(C.byref(st), 0))
    assert st.value == 0
    x = torch.arange(1024, device="cuda:0", dtype=torch.float32)
    assert float((x * 2).sum()) == 1023.0 * 1024.0

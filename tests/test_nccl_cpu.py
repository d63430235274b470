"""The NCCL path of the C ABI (nt_nccl_*), host side on the CPU: the workspace size of a band
plan, argument checks that return before anything is queued, and the communicator id (NCCL
creates it without a GPU)."""
import ctypes as C

import pytest

from neural_textures_b200.sharded import HALO, source_band

INVALID_ARG, NCCL_ERR = 1, 3


def _shard(world=2, rank=0, grids=((128, 128), (64, 64)), C_=8, lattice_h=128):
    from neural_textures_b200 import _native as N
    s = N.NtShard()
    p = s.params
    p.latent_channels, p.output_channels = C_, 8
    for i, (w, h) in enumerate(grids):
        band = source_band(rank, world, lattice_h, h)
        f = p.features[i]
        f.grid, f.gradients, f.moment1, f.moment2 = 0x10000 * (i + 1), 0x10000 * (i + 1) + 0x1000, 0x30000, 0x40000
        f.width, f.height = w, h
        p.row_origin[i], p.stored_rows[i] = band.origin, band.stored
        s.halo_rows[i] = band.halo
    return s


def test_workspace_holds_both_halos_of_both_grids(native):
    s = _shard()
    want = sum(2 * HALO * w * 8 * 4 for (w, _) in ((128, 128), (64, 64)))
    assert native.nt_nccl_workspace_bytes(C.byref(s)) == want
    s12 = _shard(C_=12, grids=((96, 128), (48, 64)))
    assert native.nt_nccl_workspace_bytes(C.byref(s12)) == sum(2 * HALO * w * 12 * 4 for w in (96, 48))
    assert native.nt_nccl_workspace_bytes(None) == 0


def test_argument_checks_return_before_any_work(native):
    s = _shard()
    assert native.nt_nccl_train_step(None, C.byref(s), None, 0) == INVALID_ARG
    assert b"comm is null" in native.nt_get_last_error_string()
    uid = (C.c_ubyte * 128)()
    h = C.c_void_p(1234)
    assert native.nt_nccl_comm_create(uid, 2, 2, 0, C.byref(h)) == INVALID_ARG
    assert h.value is None  # *comm is cleared on failure
    assert native.nt_nccl_comm_create(None, 2, 0, 0, C.byref(h)) == INVALID_ARG
    assert native.nt_nccl_comm_create(uid, 2, 0, -1, C.byref(h)) == INVALID_ARG
    assert native.nt_nccl_comm_wait(None, 10) == INVALID_ARG
    assert native.nt_nccl_comm_destroy(None) == 0


def test_unique_id(native):
    a, b = (C.c_ubyte * 128)(), (C.c_ubyte * 128)()
    st = native.nt_nccl_unique_id(a)
    if st == NCCL_ERR:
        pytest.skip(native.nt_get_last_error_string().decode())
    assert st == 0 and native.nt_nccl_unique_id(b) == 0
    assert bytes(a) != bytes(b) and any(bytes(a))
    assert native.nt_nccl_unique_id(None) == INVALID_ARG

"""The one-thread sharded step of the C ABI (nt_dist_band, nt_dist_train_step), host side,
on CPU: the band split agrees with the Python plan, and shard sets whose layout is wrong are
rejected before any CUDA call."""
import ctypes as C

import pytest

from neural_textures_b200.sharded import HALO, source_band


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("lattice_h,height", [(512, 512), (512, 256), (2048, 4096), (1024, 16384), (96, 64)])
def test_band_split_matches_python_plan(native, world, lattice_h, height):
    lo, hi = C.c_int32(), C.c_int32()
    try:
        b = source_band(0, world, lattice_h, height)
    except ValueError:
        b = None
    for r in range(world):
        st = native.nt_dist_band(r, world, lattice_h, height, HALO if world > 1 else 0, C.byref(lo), C.byref(hi))
        if b is None:
            assert st != 0
            continue
        b = source_band(r, world, lattice_h, height)
        assert st == 0, native.nt_get_last_error_string()
        assert (lo.value, hi.value) == (b.lo, b.hi)


def test_band_split_rejects_thin_bands(native):
    lo, hi = C.c_int32(), C.c_int32()
    assert native.nt_dist_band(0, 8, 64, 16, HALO, C.byref(lo), C.byref(hi)) != 0
    assert b"cannot be sharded" in native.nt_get_last_error_string()
    # owned rows between one and two halos: rejected (the step adds halo gradients to both
    # band edges at once), and a band of exactly two halos is accepted
    assert native.nt_dist_band(0, 2, 16, 10, 3, C.byref(lo), C.byref(hi)) != 0  # 5 rows, halo 3
    assert b"at least 6 rows" in native.nt_get_last_error_string()
    assert native.nt_dist_band(0, 2, 16, 12, 3, C.byref(lo), C.byref(hi)) == 0  # 6 rows, halo 3
    assert (lo.value, hi.value) == (0, 6)
    assert native.nt_dist_band(3, 2, 64, 16, 3, C.byref(lo), C.byref(hi)) != 0
    assert native.nt_dist_band(0, 2, 64, 16, 3, None, None) != 0


def _band(r, world, lattice_h, h, halo):
    """source_band's rounding without its thickness check (to build invalid sets too)."""
    a, b = r * lattice_h // world, (r + 1) * lattice_h // world
    rnd = lambda x: (2 * x * h + lattice_h) // (2 * lattice_h)
    lo, hi = rnd(a), rnd(b)
    return type("B", (), {"origin": (lo - halo) % h, "stored": hi - lo + 2 * halo})


def _shard_set(world, grids=((128, 128), (64, 64)), C_=8, halo=HALO, lattice_h=128):
    """A consistent shard set on host-only fake pointers (never dereferenced: the layout checks
    run first and the CUDA calls fail without a GPU); every shard has its own pointers."""
    from neural_textures_b200 import _native as N
    arr = (N.NtShard * world)()
    for r in range(world):
        p = arr[r].params
        p.latent_channels, p.output_channels = C_, 8
        p.lattice_width, p.lattice_height = lattice_h, lattice_h
        a, b = r * lattice_h // world, (r + 1) * lattice_h // world
        p.lattice_row0, p.lattice_rows = a, b - a
        for l in range(3):
            base = 0x100000 * (r + 1) + 0x1000 * l
            p.network_weights[l] = base + 0x10
            p.network_weight_gradients[l] = base + 0x20
            p.network_weight_moment1[l] = base + 0x30
            p.network_weight_moment2[l] = base + 0x40
            p.network_biases[l] = base + 0x50
            p.network_bias_gradients[l] = base + 0x60
            p.network_bias_moment1[l] = base + 0x70
            p.network_bias_moment2[l] = base + 0x80
        for i, (w, h) in enumerate(grids):
            band = _band(r, world, lattice_h, h, halo)
            f = p.features[i]
            base = 0x100000 * (r + 1) + 0x10000 * (i + 1)
            f.grid, f.gradients, f.moment1, f.moment2 = base, base + 0x100, base + 0x200, base + 0x300
            f.width, f.height = w, h
            p.row_origin[i] = band.origin
            p.stored_rows[i] = band.stored
            arr[r].halo_rows[i] = halo
        arr[r].device = 0
    return arr


def test_dist_step_rejects_bad_sets(native):
    INVALID_ARG = 1
    assert native.nt_dist_train_step(None, 2) == INVALID_ARG
    arr = _shard_set(2)
    assert native.nt_dist_train_step(arr, 0) != 0
    assert native.nt_dist_train_step(arr, 17) != 0
    assert b"count" in native.nt_get_last_error_string()

    bad = _shard_set(3)
    bad[1].params.step = 7
    assert native.nt_dist_train_step(bad, 3) != 0
    assert b"step" in native.nt_get_last_error_string()

    bad = _shard_set(3)
    bad[2].params.row_origin[0] = (bad[2].params.row_origin[0] + 1) % 128
    assert native.nt_dist_train_step(bad, 3) != 0
    assert b"does not start where" in native.nt_get_last_error_string()

    bad = _shard_set(3)
    bad[2].params.num_samples = 5
    assert native.nt_dist_train_step(bad, 3) != 0
    assert b"num_samples" in native.nt_get_last_error_string()

    bad = _shard_set(2)
    bad[1].halo_rows[1] = 2
    assert native.nt_dist_train_step(bad, 2) != 0
    assert b"halo_rows" in native.nt_get_last_error_string()

    bad = _shard_set(3)
    bad[0].params.latent_format = 1
    assert native.nt_dist_train_step(bad, 3) != 0
    assert b"fp16 latent grids" in native.nt_get_last_error_string()

    # bands of 4 rows between 3-row halos: the two edge additions would overlap
    thin = _shard_set(8, grids=((128, 128), (32, 32)), lattice_h=128)
    assert native.nt_dist_train_step(thin, 8) != 0
    assert b"thinner than two" in native.nt_get_last_error_string()

    # two shards passing the same buffer
    shared = _shard_set(3)
    shared[2].params.network_weight_moment1[1] = shared[0].params.network_weight_moment1[1]
    assert native.nt_dist_train_step(shared, 3) != 0
    assert b"share a network buffer" in native.nt_get_last_error_string()
    shared = _shard_set(2)
    shared[1].params.features[0].gradients = shared[0].params.features[0].gradients
    assert native.nt_dist_train_step(shared, 2) != 0
    assert b"share a buffer of latent grid 0" in native.nt_get_last_error_string()


def test_dist_step_layout_accepted(native):
    """A consistent set passes every host check and stops at the first CUDA call (no GPU here)
    or at the pointer check (fake pointers on a GPU box)."""
    arr = _shard_set(3)
    st = native.nt_dist_train_step(arr, 3)
    assert st != 0
    msg = native.nt_get_last_error_string()
    assert b"cudaSetDevice" in msg or b"not a CUDA pointer" in msg or b"not device memory" in msg, msg

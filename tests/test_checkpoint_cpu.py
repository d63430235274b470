"""The on-disk format (nt_checkpoint_write / _index / _read) on the CPU: round trips of every
dtype and shape, atomic replacement, and rejection of corrupt, truncated or foreign files and of
invalid section tables (NT_ERR_IO / NT_ERR_INVALID_ARG with a message, never a crash)."""
import os

import numpy as np
import pytest


def _sections(rng):
    return {
        "f16": (rng.standard_normal((3, 5, 8)) * 4).astype(np.float16),
        "f32": rng.standard_normal((7,)).astype(np.float32),
        "u8": rng.integers(0, 256, (2, 3, 4, 5), dtype=np.uint8),
        "i32": np.array(rng.integers(-9, 9, 11), np.int32),
        "scalar": np.array(2.5, np.float32),
        "empty": np.zeros((0, 4), np.float32),
    }


def test_round_trip(native, tmp_path):
    import neural_textures_b200 as nt
    rng = np.random.default_rng(1)
    sec = _sections(rng)
    path = tmp_path / "a.ntck"
    nt.api.checkpoint_write(path, sec)
    idx = nt.api.checkpoint_index(path)
    assert list(idx) == list(sec)
    for k, v in sec.items():
        assert idx[k] == (v.dtype, v.shape)
    back = nt.api.checkpoint_read(path)
    for k, v in sec.items():
        assert back[k].dtype == v.dtype and back[k].shape == v.shape
        assert back[k].tobytes() == v.tobytes()
    # payloads sit at 64-byte aligned offsets after the 64-byte header
    raw = open(path, "rb").read()
    assert raw[:8] == b"NTB2CKPT"
    assert raw.find(sec["f16"].tobytes()) == 64
    # replacing an existing file is atomic (written beside it, then renamed)
    nt.api.checkpoint_write(path, {"only": np.arange(4, dtype=np.int32)})
    assert list(nt.api.checkpoint_index(path)) == ["only"]
    assert not os.path.exists(str(path) + ".tmp")


def _expect(native, rc, status, needle):
    from neural_textures_b200 import _native
    assert rc == status, (rc, native.nt_get_last_error_string())
    assert needle.encode() in native.nt_get_last_error_string(), native.nt_get_last_error_string()


def test_corrupt_files_are_rejected(native, tmp_path):
    import neural_textures_b200 as nt
    from neural_textures_b200 import _native
    rng = np.random.default_rng(2)
    sec = _sections(rng)
    good = tmp_path / "g.ntck"
    nt.api.checkpoint_write(good, sec)
    raw = bytearray(open(good, "rb").read())
    dst = np.empty_like(sec["f16"])

    def variant(name, data):
        p = tmp_path / name
        open(p, "wb").write(bytes(data))
        return os.fsencode(str(p))

    NT_ERR_IO = 7
    # a flipped payload byte: the index still loads, the section's checksum does not match
    bad = bytearray(raw)
    bad[64 + 5] ^= 0x40
    rc = native.nt_checkpoint_read(variant("payload", bad), b"f16", dst.ctypes.data, dst.nbytes)
    _expect(native, rc, NT_ERR_IO, "checksum")
    # a flipped index byte
    bad = bytearray(raw)
    bad[-20] ^= 0x01
    import ctypes as C
    cnt = C.c_int32(0)
    _expect(native, native.nt_checkpoint_index(variant("index", bad), None, 0, C.byref(cnt)), NT_ERR_IO, "index")
    # truncated, foreign, missing
    _expect(native, native.nt_checkpoint_index(variant("trunc", raw[:len(raw) - 3]), None, 0, C.byref(cnt)), NT_ERR_IO,
            "index")
    _expect(native, native.nt_checkpoint_index(variant("short", raw[:40]), None, 0, C.byref(cnt)), NT_ERR_IO, "header")
    foreign = bytearray(raw)
    foreign[:8] = b"NOTACKPT"
    _expect(native, native.nt_checkpoint_index(variant("magic", foreign), None, 0, C.byref(cnt)), NT_ERR_IO,
            "not a checkpoint")
    newer = bytearray(raw)
    newer[8] = 9
    _expect(native, native.nt_checkpoint_index(variant("version", newer), None, 0, C.byref(cnt)), NT_ERR_IO, "version")
    _expect(native, native.nt_checkpoint_index(os.fsencode(str(tmp_path / "none")), None, 0, C.byref(cnt)), NT_ERR_IO,
            "cannot open")
    # wrong destination size, unknown section
    _expect(native, native.nt_checkpoint_read(os.fsencode(str(good)), b"f16", dst.ctypes.data, dst.nbytes - 2), 1,
            "bytes")
    _expect(native, native.nt_checkpoint_read(os.fsencode(str(good)), b"nope", dst.ctypes.data, dst.nbytes), 1,
            "no section")


@pytest.mark.parametrize("bad,needle", [
    (lambda e: setattr(e, "name", b""), "name"),
    (lambda e: setattr(e, "dtype", 9), "dtype"),
    (lambda e: setattr(e, "ndim", 5), "ndim"),
    (lambda e: setattr(e, "bytes", 3), "bytes"),
    (lambda e: setattr(e, "data", None), "data is null"),
])
def test_invalid_section_tables_are_rejected(native, tmp_path, bad, needle):
    from neural_textures_b200 import _native
    a = np.arange(6, dtype=np.float32)
    tab = (_native.NtCheckpointSection * 2)()
    for i, nm in enumerate((b"a", b"b")):
        tab[i].name, tab[i].dtype, tab[i].ndim = nm, _native.NT_DTYPE_F32, 1
        tab[i].shape[0], tab[i].bytes, tab[i].data = 6, a.nbytes, a.ctypes.data
    bad(tab[1])
    path = os.fsencode(str(tmp_path / "x.ntck"))
    _expect(native, native.nt_checkpoint_write(path, tab, 2), 1, needle)
    assert not os.path.exists(tmp_path / "x.ntck")
    tab2 = (_native.NtCheckpointSection * 2)()
    for i in range(2):
        tab2[i].name, tab2[i].dtype, tab2[i].ndim = b"same", _native.NT_DTYPE_F32, 1
        tab2[i].shape[0], tab2[i].bytes, tab2[i].data = 6, a.nbytes, a.ctypes.data
    _expect(native, native.nt_checkpoint_write(path, tab2, 2), 1, "twice")


def test_failed_write_leaves_no_temporary(native, tmp_path):
    """A write that cannot be completed (here the rename: the destination is a directory)
    returns NT_ERR_IO, removes its .tmp file and leaves the destination untouched."""
    import neural_textures_b200 as nt
    from neural_textures_b200 import _native
    dst = tmp_path / "ckpt"
    dst.mkdir()
    with pytest.raises(_native.NtError):
        nt.api.checkpoint_write(dst, {"a": np.arange(4, dtype=np.int32)})
    assert not os.path.exists(str(dst) + ".tmp")
    assert dst.is_dir()

"""The C-ABI library loads, exports every symbol include/nt_capi.h declares, its parameter
block matches the Python mirror, and invalid calls are rejected on the host (no GPU needed:
every rejection below happens before any CUDA call)."""
import ctypes as C
import os
import re
import subprocess

import pytest

from tests.conftest import ROOT


def header_functions():
    src = open(os.path.join(ROOT, "include", "nt_capi.h")).read()
    return sorted(set(re.findall(r"^NT_API\s+[\w\s\*]+?\b(nt_\w+)\s*\(", src, re.M)))


def test_every_declared_symbol_is_exported(native):
    from neural_textures_b200 import _native
    declared = header_functions()
    assert len(declared) >= 16
    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(line.split()[-1] for line in out.splitlines() if line.strip())
    missing = [s for s in declared if s not in exported]
    assert not missing, f"declared but not exported: {missing}"
    # and the Python binding binds exactly the declared set
    assert sorted(_native.SIGNATURES) == declared
    assert "_ZN15neural_textures18RunForwardPassTestEv" in exported  # C++ harness symbol


def test_kernel_params_layout_matches_mirror(native):
    from neural_textures_b200 import _native
    assert native.nt_version() == 1
    assert native.nt_kernel_params_size() == C.sizeof(_native.NtKernelParams)
    for name, _ in _native.NtKernelParams._fields_:
        off = native.nt_kernel_params_offset(name.encode())
        assert off == getattr(_native.NtKernelParams, name).offset, name
    assert native.nt_kernel_params_offset(b"no_such_field") == C.c_size_t(-1).value


def _valid_looking_params():
    """Parameter block with plausible (never dereferenced) aligned pointers."""
    from neural_textures_b200 import _native
    p = _native.NtKernelParams()
    fake = 0x10000
    for i in range(2):
        f = p.features[i]
        f.grid = f.gradients = f.moment1 = f.moment2 = fake
        f.width = f.height = 64
    p.latent_channels, p.output_channels = 8, 8
    for l in range(3):
        for name in ("network_weights", "network_weight_gradients", "network_weight_moment1",
                     "network_weight_moment2", "network_biases", "network_bias_gradients",
                     "network_bias_moment1", "network_bias_moment2"):
            getattr(p, name)[l] = fake
    p.target = fake
    p.image_width = p.image_height = 128
    p.lattice_width = p.lattice_height = 64
    p.sample_stride_x = p.sample_stride_y = 2.0
    p.num_samples = 64 * 64
    return p


@pytest.mark.parametrize("mutate,needle", [
    (lambda p: setattr(p, "latent_channels", 7), "latent_channels"),
    (lambda p: setattr(p, "output_channels", 17), "output_channels"),
    (lambda p: setattr(p, "output_channels", 0), "output_channels"),
    (lambda p: setattr(p, "num_samples", 5), "num_samples"),
    (lambda p: setattr(p, "target", None), "target"),
    (lambda p: setattr(p.features[1], "grid", 0x10002), "features[1].grid"),
    (lambda p: setattr(p.features[0], "width", 0), "features[0]"),
    (lambda p: p.network_weights.__setitem__(2, None), "network_weights[2]"),
    (lambda p: setattr(p, "sample_stride_x", 0.0), "strides"),
    (lambda p: setattr(p.features[0], "num_mips", 17), "num_mips"),
    (lambda p: setattr(p, "target_num_mips", 17), "target_num_mips"),
])
def test_training_rejects_invalid_arguments(native, mutate, needle):
    from neural_textures_b200 import _native
    p = _valid_looking_params()
    mutate(p)
    st = native.nt_invoke_training(C.byref(p), _native.NT_TRAIN_UNCONSTRAINED, None)
    assert st == 1, _native.last_error()
    assert needle in _native.last_error()


def test_latent_format_must_match_the_training_type(native):
    from neural_textures_b200 import _native
    p = _valid_looking_params()
    # fp16 grids cannot be trained as BC6 block features, and the reverse
    assert native.nt_invoke_training(C.byref(p), _native.NT_TRAIN_BLOCK_FEATURES, None) == 1
    assert "BLOCK_FEATURES" in _native.last_error()
    assert native.nt_invoke_optimize_features(C.byref(p), _native.NT_TRAIN_BLOCK_FEATURES, None) == 1
    p.latent_format = _native.NT_LATENT_BC6_BLOCKS
    assert native.nt_invoke_training(C.byref(p), _native.NT_TRAIN_UNCONSTRAINED, None) == 1
    assert native.nt_invoke_inference(C.byref(p), None) == 1
    p.features[0].width = 30  # block features need whole 4x4 blocks
    assert native.nt_invoke_training(C.byref(p), _native.NT_TRAIN_BLOCK_FEATURES, None) == 1
    assert "multiple of 4" in _native.last_error()


def test_mip_coordinate_restrictions(native):
    """Sharded calls sample level 0; block features sample one level whose size is a multiple
    of 4 (both rejected on the host, before any CUDA call)."""
    from neural_textures_b200 import _native
    p = _valid_looking_params()
    p.features[0].num_mips = p.features[1].num_mips = 3
    p.lod = 1.0
    p.lattice_rows = 32
    assert native.nt_invoke_training(C.byref(p), _native.NT_TRAIN_UNCONSTRAINED, None) == 1
    assert b"lod 0" in native.nt_get_last_error_string()
    p = _valid_looking_params()
    p.latent_format = _native.NT_LATENT_BC6_BLOCKS
    p.features[0].num_mips = 3
    p.lod = 0.5
    assert native.nt_invoke_training(C.byref(p), _native.NT_TRAIN_BLOCK_FEATURES, None) == 1
    assert b"one mip level" in native.nt_get_last_error_string()


def test_null_params_rejected(native):
    assert native.nt_invoke_training(None, 0, None) == 1
    assert native.nt_invoke_inference(None, None) == 1
    assert native.nt_invoke_optimize_all(None, None) == 1


def test_inference_requires_output(native):
    from neural_textures_b200 import _native
    p = _valid_looking_params()
    assert native.nt_invoke_inference(C.byref(p), None) == 1
    assert "inference_output" in _native.last_error()


def test_python_mirror_raises_ntError(native):
    import neural_textures_b200 as nt
    p = _valid_looking_params()
    p.latent_channels = 5
    with pytest.raises(nt.NtError, match="NT_ERR_INVALID_ARG"):
        nt.InvokeTraining(p)

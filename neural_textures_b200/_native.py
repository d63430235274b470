"""ctypes binding of libnt_b200.so (the C ABI declared in include/nt_capi.h).

The library is built in-tree (neural_textures_b200/lib/libnt_b200.so).  There is no
fallback: if the library is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os

from . import build as _build

LIB_PATH = _build.LIB

NT_NUM_FEATURES = 2
NT_NUM_NETWORK_LAYERS = 3
NT_MAX_OUTPUT = 16

NT_OK = 0
STATUS_NAMES = {0: "NT_OK", 1: "NT_ERR_INVALID_ARG", 2: "NT_ERR_CUDA", 3: "NT_ERR_NCCL",
                4: "NT_ERR_TIMEOUT", 5: "NT_ERR_BOUNDS", 6: "NT_ERR_UNSUPPORTED", 7: "NT_ERR_IO"}

NT_TRAIN_UNCONSTRAINED = 0
NT_TRAIN_BLOCK_FEATURES = 1
NT_TRAIN_FINALIZE = 2
NT_LATENT_GRID_F16 = 0
NT_LATENT_BC6_BLOCKS = 1
NT_BC6F_RECORD_FLOATS = 32
NT_DTYPE_F16 = 0
NT_DTYPE_F32 = 1
NT_DTYPE_U8 = 2
NT_DTYPE_I32 = 3
NT_CKPT_NAME_LEN = 32
NT_MAX_REFERENCE_TEXTURES = 16


class NtAdamConstants(C.Structure):
    _fields_ = [("beta1", C.c_float), ("beta2", C.c_float), ("learning_rate", C.c_float),
                ("epsilon", C.c_float)]


class NtFeature(C.Structure):
    _fields_ = [("grid", C.c_void_p), ("gradients", C.c_void_p), ("moment1", C.c_void_p),
                ("moment2", C.c_void_p), ("width", C.c_int32), ("height", C.c_int32), ("num_mips", C.c_int32)]


class NtReferenceTexture(C.Structure):
    _fields_ = [("texture", C.c_uint64), ("storage", C.c_uint64), ("width", C.c_int32), ("height", C.c_int32),
                ("num_channels", C.c_int32), ("num_mips", C.c_int32), ("loss_weight", C.c_float),
                ("reserved", C.c_int32)]


class NtCheckpointSection(C.Structure):
    _fields_ = [("name", C.c_char * NT_CKPT_NAME_LEN), ("dtype", C.c_int32), ("ndim", C.c_int32),
                ("shape", C.c_int64 * 4), ("bytes", C.c_int64), ("data", C.c_void_p)]


class NtKernelParams(C.Structure):
    _fields_ = [
        ("features", NtFeature * NT_NUM_FEATURES),
        ("latent_channels", C.c_int32),
        ("output_channels", C.c_int32),
        ("network_weights", C.c_void_p * 3),
        ("network_weight_gradients", C.c_void_p * 3),
        ("network_weight_moment1", C.c_void_p * 3),
        ("network_weight_moment2", C.c_void_p * 3),
        ("network_biases", C.c_void_p * 3),
        ("network_bias_gradients", C.c_void_p * 3),
        ("network_bias_moment1", C.c_void_p * 3),
        ("network_bias_moment2", C.c_void_p * 3),
        ("network_adam", NtAdamConstants),
        ("feature_adam", NtAdamConstants),
        ("target", C.c_void_p),
        ("channel_loss_weights", C.c_float * NT_MAX_OUTPUT),
        ("inference_output", C.c_void_p),
        ("inference_output_dtype", C.c_int32),
        ("inference_mse_accum", C.c_void_p),
        ("image_width", C.c_int32),
        ("image_height", C.c_int32),
        ("lattice_width", C.c_int32),
        ("lattice_height", C.c_int32),
        ("sample_stride_x", C.c_float),
        ("sample_stride_y", C.c_float),
        ("texel_offset_x", C.c_int32),
        ("texel_offset_y", C.c_int32),
        ("num_samples", C.c_int32),
        ("step", C.c_int32),
        ("seed", C.c_uint32),
        ("loss_accum", C.c_void_p),
        ("lattice_row0", C.c_int32),
        ("lattice_rows", C.c_int32),
        ("row_origin", C.c_int32 * 3),
        ("stored_rows", C.c_int32 * 3),
        ("latent_format", C.c_int32),
        ("lod", C.c_float),
        ("target_num_mips", C.c_int32),
        ("target_width", C.c_int32),
        ("target_height", C.c_int32),
        ("reference_textures", NtReferenceTexture * NT_MAX_REFERENCE_TEXTURES),
        ("num_reference_textures", C.c_int32),
        ("inference_output_stride", C.c_int32),
        ("workspace", C.c_void_p),
        ("workspace_bytes", C.c_int64),
    ]


NT_DIST_MAX_SHARDS = 16
NT_NCCL_UNIQUE_ID_BYTES = 128


class NtShard(C.Structure):
    _fields_ = [("params", NtKernelParams), ("halo_rows", C.c_int32 * NT_NUM_FEATURES), ("device", C.c_int32),
                ("stream", C.c_void_p)]


class NtBc6hSurface(C.Structure):
    _fields_ = [("data", C.c_void_p), ("width", C.c_int32), ("height", C.c_int32), ("channels", C.c_int32),
                ("channel_stride", C.c_int64), ("row_stride", C.c_int64), ("texel_stride", C.c_int64)]


# Every symbol include/nt_capi.h declares: name -> (restype, argtypes)
_P = C.POINTER(NtKernelParams)
_S = C.POINTER(NtBc6hSurface)
SIGNATURES = {
    "nt_version": (C.c_int32, []),
    "nt_get_last_error_string": (C.c_char_p, []),
    "nt_kernel_params_size": (C.c_size_t, []),
    "nt_kernel_params_offset": (C.c_size_t, [C.c_char_p]),
    "nt_launch_count": (C.c_uint64, []),
    "nt_workspace_bytes": (C.c_size_t, []),
    "nt_invoke_training": (C.c_int, [_P, C.c_int, C.c_void_p]),
    "nt_invoke_training_static_scratch": (C.c_int, [_P, C.c_int, C.c_void_p]),
    "nt_invoke_optimize_network": (C.c_int, [_P, C.c_void_p]),
    "nt_invoke_optimize_features": (C.c_int, [_P, C.c_int, C.c_void_p]),
    "nt_invoke_optimize_all": (C.c_int, [_P, C.c_void_p]),
    "nt_invoke_inference": (C.c_int, [_P, C.c_void_p]),
    "nt_train_step": (C.c_int, [_P, C.c_void_p]),
    "nt_dist_band": (C.c_int, [C.c_int32] * 5 + [C.POINTER(C.c_int32)] * 2),
    "nt_dist_train_step": (C.c_int, [C.POINTER(NtShard), C.c_int32]),
    "nt_run_forward_pass_test": (C.c_int32, []),
    "nt_forward_pass_12x16x16": (C.c_int, [C.c_void_p] * 6 + [C.c_void_p]),
    "nt_generate_target": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_uint32,
                                     C.c_int32, C.c_void_p]),
    "nt_init_latents": (C.c_int, [C.c_void_p, C.c_int64, C.c_uint32, C.c_void_p]),
    "nt_bc6h_blocks_bytes": (C.c_size_t, [C.c_int32, C.c_int32, C.c_int32]),
    "nt_bc6h_encode": (C.c_int, [_S, C.c_void_p, C.c_float, C.c_void_p]),
    "nt_bc6h_decode": (C.c_int, [C.c_void_p, _S, C.c_float, C.c_void_p]),
    "nt_bc6h_decode_raw": (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_void_p, C.c_void_p]),
    "nt_bc6h_decode_hardware": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.POINTER(C.c_float)]),
    "nt_bc6f_records_floats": (C.c_size_t, [C.c_int32, C.c_int32, C.c_int32]),
    "nt_bc6f_from_bc6h": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]),
    "nt_bc6f_to_bc6h": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]),
    "nt_umma_selftest": (C.c_int, [C.c_void_p] * 6 + [C.c_void_p]),
    "nt_read_device_status": (C.c_int, [C.POINTER(C.c_uint32), C.c_int32]),
    "nt_flush_l2": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p]),
    "nt_mip_chain_texels": (C.c_int64, [C.c_int32, C.c_int32, C.c_int32]),
    "nt_reference_texture_create": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_float,
                                             C.POINTER(NtReferenceTexture)]),
    "nt_reference_texture_destroy": (C.c_int, [C.POINTER(NtReferenceTexture)]),
    "nt_reference_texture_sample": (C.c_int, [C.POINTER(NtReferenceTexture), C.c_void_p, C.c_int64, C.c_float,
                                             C.c_void_p, C.c_void_p]),
    "nt_wait_timeout_selftest": (C.c_int, [C.c_uint32]),
    "nt_checkpoint_write": (C.c_int, [C.c_char_p, C.POINTER(NtCheckpointSection), C.c_int32]),
    "nt_checkpoint_index": (C.c_int, [C.c_char_p, C.POINTER(NtCheckpointSection), C.c_int32,
                                      C.POINTER(C.c_int32)]),
    "nt_checkpoint_read": (C.c_int, [C.c_char_p, C.c_char_p, C.c_void_p, C.c_int64]),
    "nt_build_mips": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p]),
    "nt_nccl_unique_id": (C.c_int, [C.c_void_p]),
    "nt_nccl_comm_create": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.POINTER(C.c_void_p)]),
    "nt_nccl_comm_destroy": (C.c_int, [C.c_void_p]),
    "nt_nccl_workspace_bytes": (C.c_size_t, [C.POINTER(NtShard)]),
    "nt_nccl_train_step": (C.c_int, [C.c_void_p, C.POINTER(NtShard), C.c_void_p, C.c_size_t]),
    "nt_nccl_comm_wait": (C.c_int, [C.c_void_p, C.c_int32]),
}

_lib = None


class NtError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def load(path: str | None = None):
    """Load (once) and bind libnt_b200.so.  Raises OSError if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise OSError(f"{p} is missing: build it with `python -m neural_textures_b200.build` "
                      "(there is no CPU fallback)")
    lib = C.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != NT_OK:
        msg = load().nt_get_last_error_string().decode(errors="replace")
        raise NtError(status, msg)


def last_error() -> str:
    return load().nt_get_last_error_string().decode(errors="replace")

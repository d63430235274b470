"""neural_textures_b200 -- B200-native (sm_100a) neural-texture trainer and decoder.

Drop-in for the hot path of mavenkim2/neural_textures (train.h entry points, mlp.h network,
tests/forward_pass_test harness).  All computation runs in the in-tree CUDA library
lib/libnt_b200.so through the C ABI of include/nt_capi.h; this package only allocates
device memory (through torch) and fills the parameter block.
"""
from ._native import NtError, NtKernelParams, load  # noqa: F401
from .api import (  # noqa: F401
    InvokeInference,
    InvokeOptimizeAll,
    InvokeOptimizeFeatures,
    InvokeOptimizeNetwork,
    InvokeTraining,
    NeuralTexture,
    ReferenceTexture,
    RunForwardPassTest,
    TrainingKernelType,
    TrainStep,
    bc6f_from_bc6h,
    bc6f_records_floats,
    bc6f_to_bc6h,
    bc6h_blocks_bytes,
    bc6h_decode,
    bc6h_encode,
    he_normal_weights,
    invoke_inference,
    invoke_optimize_all,
    invoke_optimize_features,
    invoke_optimize_network,
    invoke_training,
    launch_count,
    run_forward_pass_test,
    train_step,
)

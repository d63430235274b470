// neural_textures/train.h -- C++ drop-in for mavenkim2/neural_textures train.h.
//
// Same names and call shapes as the reference (train.h:22-35, :51-67, :120-161):
// KernelParams passed by value, TrainingKernelType, AdamConstants, Feature and the four
// Invoke* entry points.  Each forwards to the C ABI (nt_capi.h).  The reference's
// entry points return void and surface failures as std::runtime_error from the driver's
// CheckCuda (main.cpp:103-110); this header throws the same exception type with the
// library's message when a call is rejected or a launch fails.
#pragma once

#include <stdexcept>
#include <string>

#include "nt_capi.h"

namespace neural_textures {

using KernelParams = NtKernelParams;
using AdamConstants = NtAdamConstants;
using Feature = NtFeature;

enum class TrainingKernelType {
    UNCONSTRAINED = NT_TRAIN_UNCONSTRAINED,
    BLOCK_FEATURES = NT_TRAIN_BLOCK_FEATURES,
    FINALIZE = NT_TRAIN_FINALIZE,
};

inline void ThrowIfFailed(nt_status st, const char *what)
{
    if (st != NT_OK) throw std::runtime_error(std::string(what) + " failed: " + nt_get_last_error_string());
}

// train.h:158
inline void InvokeOptimizeNetwork(KernelParams params, nt_stream_t stream = nullptr)
{
    ThrowIfFailed(nt_invoke_optimize_network(&params, stream), "InvokeOptimizeNetwork");
}

// train.h:159
inline void InvokeOptimizeFeatures(KernelParams params, TrainingKernelType type, nt_stream_t stream = nullptr)
{
    ThrowIfFailed(nt_invoke_optimize_features(&params, static_cast<NtTrainingKernelType>(type), stream),
                  "InvokeOptimizeFeatures");
}

// train.h:160
inline void InvokeTraining(KernelParams params, TrainingKernelType type, nt_stream_t stream = nullptr)
{
    ThrowIfFailed(nt_invoke_training(&params, static_cast<NtTrainingKernelType>(type), stream), "InvokeTraining");
}

// train.h:161
inline void InvokeInference(KernelParams params, nt_stream_t stream = nullptr)
{
    ThrowIfFailed(nt_invoke_inference(&params, stream), "InvokeInference");
}

}  // namespace neural_textures

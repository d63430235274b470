// neural_textures/train.h -- C++ drop-in for mavenkim2/neural_textures train.h.
//
// Same names, field names and call shapes as the reference (train.h:22-35, :51-77, :120-161):
// KernelParams passed by value with the reference's camelCase fields, TrainingKernelType,
// AdamConstants, Feature, ReferenceTexture and the four Invoke* entry points.  Each entry
// point converts KernelParams to the C ABI's NtKernelParams (nt_capi.h) and forwards.  The
// reference's entry points return void and surface failures as std::runtime_error from the
// driver's CheckCuda (main.cpp:103-110); these throw the same exception type with the
// library's message when a call is rejected or a launch fails.
//
// What the fields mean here (the build's network is BASELINE's, not the reference's 12-32-32-16):
//   features[f]          one of NT_NUM_FEATURES (2) latent grids of latentChannels channels.
//                        unconstrainedGrid / Gradients / Moment1 / Moment2 (the reference's
//                        float3** per-mip arrays, train.h:57-60) are one buffer per grid here:
//                        fp16 [h][w][latentChannels] texels (fp32 for the others), mip levels
//                        stored one after another.  grid / gradients / moment1 / moment2 (the
//                        reference's BC6Parameters**, train.h:53-56) are the fp32 BC6 block
//                        records of the BLOCK_FEATURES path (nt_capi.h NT_LATENT_BC6_BLOCKS).
//   networkWeights ...   as train.h:124-135: fp16 weights padded column-major with padded
//                        input sizes {32, 64, 64} and padded output sizes {64, 64, 16}; fp32
//                        gradients and moments.  networkBiases[2] holds NT_OUTPUT_SIZE (16)
//                        entries, as the reference allocates it (main.cpp:758-764).
//   usedOutputChannels   output channels trained and decoded (train.h:147).  The reference
//                        computes all 16 outputs and trains those past its textures towards 0,
//                        whose weights it initialises to 0, so they stay 0 (train.cu:110-157,
//                        main.cpp:741-757); here the channels past usedOutputChannels are not
//                        computed and InvokeInference writes them as 0.
//   inferenceOutput      fp32 [imageWidth * imageHeight][NT_OUTPUT_SIZE], as train.cu:950-955.
//   numSamples           one jittered sample per texel of a 512-texel-wide region starting at
//                        (texelOffsetX, texelOffsetY), as train.cu:827-844 (0 or less: 512 x 512,
//                        train.cu:1031); it must be a multiple of 512.
//   latticeWidth ...     (no reference counterpart) a lattice of latticeWidth x latticeHeight
//                        cells of sampleStrideX x sampleStrideY texels instead; numSamples must
//                        then equal latticeWidth x latticeHeight.
// Fields below "build extensions" have no reference counterpart and default to the behaviour
// that matches the reference.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <stdexcept>
#include <string>

#include "nt_capi.h"

namespace neural_textures {

using half = __half;

#define NT_OUTPUT_SIZE 16         /* train.h:11 */
#define NT_TRAINING_REGION_SIZE 512 /* train.cu:827 kTrainingRegionSize */

// train.h:22-27
enum class TrainingKernelType {
    UNCONSTRAINED = NT_TRAIN_UNCONSTRAINED,
    BLOCK_FEATURES = NT_TRAIN_BLOCK_FEATURES,
    FINALIZE = NT_TRAIN_FINALIZE,
};

// train.h:29-35
struct AdamConstants {
    float beta1;
    float beta2;
    float learningRate;
    float epsilon;
};

// train.h:51-67 (see the header comment for the storage of each pointer)
struct Feature {
    float *grid = nullptr;  // BC6 block records (fp32)
    float *gradients = nullptr;
    float *moment1 = nullptr;
    float *moment2 = nullptr;

    half *unconstrainedGrid = nullptr;  // fp16 latents
    float *unconstrainedGradients = nullptr;
    float *unconstrainedMoment1 = nullptr;
    float *unconstrainedMoment2 = nullptr;

    int width = 0;  // in texels
    int height = 0;
    int numMips = 1;
};

// train.h:69-77
struct ReferenceTexture {
    cudaTextureObject_t texture = 0;
    int width = 0;
    int height = 0;
    int numChannels = 0;
    int numMipLevels = 0;
    float lossWeight = 1.0f;
};

// train.h:120-157
struct KernelParams {
    Feature features[NT_NUM_FEATURES];

    half *networkWeights[NT_NUM_NETWORK_LAYERS] = {};
    float *networkWeightGradients[NT_NUM_NETWORK_LAYERS] = {};
    float *networkWeightMoment1[NT_NUM_NETWORK_LAYERS] = {};
    float *networkWeightMoment2[NT_NUM_NETWORK_LAYERS] = {};

    half *networkBiases[NT_NUM_NETWORK_LAYERS] = {};
    float *networkBiasGradients[NT_NUM_NETWORK_LAYERS] = {};
    float *networkBiasMoment1[NT_NUM_NETWORK_LAYERS] = {};
    float *networkBiasMoment2[NT_NUM_NETWORK_LAYERS] = {};

    AdamConstants networkAdam = {0.9f, 0.99f, 5e-3f, 1e-8f};
    AdamConstants featureAdam = {0.9f, 0.99f, 1e-2f, 1e-8f};

    ReferenceTexture referenceTextures[NT_MAX_REFERENCE_TEXTURES];
    int numReferenceTextures = 0;
    int usedOutputChannels = NT_OUTPUT_SIZE;

    float *inferenceOutput = nullptr;
    float *inferenceMseAccum = nullptr;

    int imageWidth = 0;
    int imageHeight = 0;
    int numMips = 1;
    int numBlocksU = 0;
    int numBlocksV = 0;

    int texelOffsetX = 0;
    int texelOffsetY = 0;

    int numSamples = 0;
    int step = 0;

    // ---- build extensions (no reference counterpart) ----
    int latentChannels = 8;                // C per latent grid: 8 or 12
    const half *target = nullptr;          // fp16 [imageHeight][imageWidth][usedOutputChannels]
                                           // target, used when numReferenceTextures is 0
    float channelLossWeights[NT_OUTPUT_SIZE] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f,
                                                1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
    int latticeWidth = 0;                  // 0: the reference's 512-wide region
    int latticeHeight = 0;
    float sampleStrideX = 1.f;
    float sampleStrideY = 1.f;
    unsigned seed = 0;                     // 0: the reference's per-sample seeds
    float *lossAccum = nullptr;            // += sum of weighted squared errors of a pass
    float lod = 0.f;                       // mip coordinate of every sample (the reference's uvs.z)
};

inline void ThrowIfFailed(nt_status st, const char *what)
{
    if (st != NT_OK) throw std::runtime_error(std::string(what) + " failed: " + nt_get_last_error_string());
}

// KernelParams -> NtKernelParams.  `blocks` selects the BC6 block records as the latents.
inline NtKernelParams ToCApi(const KernelParams &p, bool blocks)
{
    NtKernelParams c;
    std::memset(&c, 0, sizeof c);
    for (int f = 0; f < NT_NUM_FEATURES; ++f) {
        const Feature &s = p.features[f];
        NtFeature &d = c.features[f];
        if (blocks) {
            d.grid = s.grid;
            d.gradients = s.gradients;
            d.moment1 = s.moment1;
            d.moment2 = s.moment2;
        } else {
            d.grid = s.unconstrainedGrid;
            d.gradients = s.unconstrainedGradients;
            d.moment1 = s.unconstrainedMoment1;
            d.moment2 = s.unconstrainedMoment2;
        }
        d.width = s.width;
        d.height = s.height;
        d.num_mips = s.numMips;
    }
    c.latent_format = blocks ? NT_LATENT_BC6_BLOCKS : NT_LATENT_GRID_F16;
    c.latent_channels = p.latentChannels;
    c.output_channels = p.usedOutputChannels;
    for (int l = 0; l < NT_NUM_NETWORK_LAYERS; ++l) {
        c.network_weights[l] = p.networkWeights[l];
        c.network_weight_gradients[l] = p.networkWeightGradients[l];
        c.network_weight_moment1[l] = p.networkWeightMoment1[l];
        c.network_weight_moment2[l] = p.networkWeightMoment2[l];
        c.network_biases[l] = p.networkBiases[l];
        c.network_bias_gradients[l] = p.networkBiasGradients[l];
        c.network_bias_moment1[l] = p.networkBiasMoment1[l];
        c.network_bias_moment2[l] = p.networkBiasMoment2[l];
    }
    c.network_adam = {p.networkAdam.beta1, p.networkAdam.beta2, p.networkAdam.learningRate, p.networkAdam.epsilon};
    c.feature_adam = {p.featureAdam.beta1, p.featureAdam.beta2, p.featureAdam.learningRate, p.featureAdam.epsilon};
    c.target = p.target;
    for (int i = 0; i < NT_OUTPUT_SIZE; ++i) c.channel_loss_weights[i] = p.channelLossWeights[i];
    c.inference_output = p.inferenceOutput;
    c.inference_output_dtype = NT_DTYPE_F32;
    c.inference_output_stride = NT_OUTPUT_SIZE;
    c.inference_mse_accum = p.inferenceMseAccum;
    c.image_width = p.imageWidth;
    c.image_height = p.imageHeight;
    const int n = p.numSamples > 0 ? p.numSamples : NT_TRAINING_REGION_SIZE * NT_TRAINING_REGION_SIZE;
    if (p.latticeWidth > 0) {
        c.lattice_width = p.latticeWidth;
        c.lattice_height = p.latticeHeight;
        c.sample_stride_x = p.sampleStrideX;
        c.sample_stride_y = p.sampleStrideY;
    } else {  // train.cu:827-832: sample i sits at texel (i % 512, i / 512) of the region
        c.lattice_width = n < NT_TRAINING_REGION_SIZE ? n : NT_TRAINING_REGION_SIZE;
        c.lattice_height = n % NT_TRAINING_REGION_SIZE == 0 || n < NT_TRAINING_REGION_SIZE
                               ? (n + NT_TRAINING_REGION_SIZE - 1) / NT_TRAINING_REGION_SIZE
                               : 0;  // rejected by the library: not a whole number of rows
        c.sample_stride_x = 1.f;
        c.sample_stride_y = 1.f;
    }
    c.texel_offset_x = p.texelOffsetX;
    c.texel_offset_y = p.texelOffsetY;
    c.num_samples = n;
    c.step = p.step;
    c.seed = p.seed;
    c.loss_accum = p.lossAccum;
    c.lod = p.lod;
    c.num_reference_textures = p.numReferenceTextures;
    for (int i = 0; i < NT_MAX_REFERENCE_TEXTURES; ++i) {
        const ReferenceTexture &s = p.referenceTextures[i];
        NtReferenceTexture &d = c.reference_textures[i];
        d.texture = (uint64_t)s.texture;
        d.width = s.width;
        d.height = s.height;
        d.num_channels = s.numChannels;
        d.num_mips = s.numMipLevels;
        d.loss_weight = s.lossWeight;
    }
    return c;
}

// Block records are the latents of BLOCK_FEATURES, and of FINALIZE when the records are set
// (the reference's FINALIZE samples its BC6 features, train.cu:845-852).
inline bool UsesBlocks(const KernelParams &p, TrainingKernelType type)
{
    if (type == TrainingKernelType::BLOCK_FEATURES) return true;
    return type == TrainingKernelType::FINALIZE && p.features[0].grid != nullptr;
}

// train.h:158
inline void InvokeOptimizeNetwork(KernelParams params, nt_stream_t stream = nullptr)
{
    const NtKernelParams c = ToCApi(params, false);
    ThrowIfFailed(nt_invoke_optimize_network(&c, stream), "InvokeOptimizeNetwork");
}

// train.h:159
inline void InvokeOptimizeFeatures(KernelParams params, TrainingKernelType type, nt_stream_t stream = nullptr)
{
    const NtKernelParams c = ToCApi(params, UsesBlocks(params, type));
    ThrowIfFailed(nt_invoke_optimize_features(&c, static_cast<NtTrainingKernelType>(type), stream),
                  "InvokeOptimizeFeatures");
}

// train.h:160
inline void InvokeTraining(KernelParams params, TrainingKernelType type, nt_stream_t stream = nullptr)
{
    const NtKernelParams c = ToCApi(params, UsesBlocks(params, type));
    ThrowIfFailed(nt_invoke_training(&c, static_cast<NtTrainingKernelType>(type), stream), "InvokeTraining");
}

// train.h:161.  Like the reference (train.cu:1050-1056) nothing runs without an image, an
// output or an MSE accumulator.
inline void InvokeInference(KernelParams params, nt_stream_t stream = nullptr)
{
    if (params.imageWidth * params.imageHeight <= 0 || !params.inferenceOutput || !params.inferenceMseAccum) return;
    const NtKernelParams c = ToCApi(params, false);
    ThrowIfFailed(nt_invoke_inference(&c, stream), "InvokeInference");
}

}  // namespace neural_textures

// driver_loop.cpp -- a reference-style driver written against the C++ drop-in headers: the
// set-up of mavenkim2/neural_textures main.cpp:680-812 (caller-allocated buffers in
// KernelParams' reference fields, reference textures as the target) and its loop
// main.cpp:1037-1091 (texelOffsetX/Y per iteration, featureAdam learning-rate decay,
// InvokeTraining, InvokeOptimizeNetwork, InvokeOptimizeFeatures, step++, then InvokeInference
// with the MSE), with std::runtime_error on failure.
//
//   driver_loop --invalid   a rejected call surfaces as std::runtime_error (no GPU needed)
//   driver_loop [iters]     known-answer test, `iters` training steps on a 768^2 material with
//                           four reference textures, inference with MSE; prints one JSON line
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <stdexcept>
#include <vector>

#include "neural_textures/forward_pass_test.h"
#include "neural_textures/train.h"

using namespace neural_textures;

namespace {

void check(cudaError_t e, const char *what)
{
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <typename T>
T *device_zeros(size_t n)
{
    T *p = nullptr;
    check(cudaMalloc(&p, n * sizeof(T)), "cudaMalloc");
    check(cudaMemset(p, 0, n * sizeof(T)), "cudaMemset");
    return p;
}

KernelParams invalid_params()
{
    KernelParams p;
    p.latentChannels = 7;  // rejected: 8 or 12 only
    p.usedOutputChannels = 8;
    return p;
}

// A smooth seeded fp32 image of `ch` channels in [0, 1].
std::vector<float> image(int w, int h, int ch, uint32_t seed)
{
    std::vector<float> v((size_t)w * h * ch);
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> U(0.f, 6.2831853f);
    float ph[4][4];
    for (auto &c : ph)
        for (float &x : c) x = U(rng);
    for (int y = 0; y < h; ++y)
        for (int x = 0; x < w; ++x)
            for (int c = 0; c < ch; ++c) {
                const float u = (x + 0.5f) / w * 6.2831853f, t = (y + 0.5f) / h * 6.2831853f;
                v[((size_t)y * w + x) * ch + c] =
                    0.5f + 0.25f * std::sin(2.f * u + ph[c][0]) * std::cos(3.f * t + ph[c][1]) +
                    0.2f * std::sin(5.f * u + 4.f * t + ph[c][2]);
            }
    return v;
}

}  // namespace

int main(int argc, char **argv)
{
    if (argc > 1 && std::strcmp(argv[1], "--invalid") == 0) {
        try {
            InvokeTraining(invalid_params(), TrainingKernelType::UNCONSTRAINED);
        } catch (const std::runtime_error &e) {
            std::printf("{\"rejected\": true, \"message\": \"%s\"}\n", e.what());
            return std::strstr(e.what(), "latent_channels") ? 0 : 1;
        }
        return 1;
    }
    const int iters = argc > 1 ? std::atoi(argv[1]) : 200;
    std::vector<NtReferenceTexture> uploaded;
    try {
        if (!RunForwardPassTest()) throw std::runtime_error("forward-pass known-answer test failed");

        const int W = 768, H = 768, C = 8;
        KernelParams params;
        params.latentChannels = C;
        // reference textures (main.cpp:558-637, 813-850): albedo RGB, normal RGB, roughness, metalness
        const int chans[4] = {3, 3, 1, 1};
        const float weights[4] = {1.f, 1.f, 0.5f, 0.5f};
        int used = 0;
        for (int i = 0; i < 4; ++i) {
            // RGB textures are uploaded as RGBA, 4 floats per texel (main.cpp:216-224, :547)
            std::vector<float> img = image(W, H, chans[i] == 3 ? 4 : chans[i], 7u + i);
            NtReferenceTexture t;
            if (nt_reference_texture_create(img.data(), W, H, chans[i], 1, weights[i], &t) != NT_OK)
                throw std::runtime_error(std::string("nt_reference_texture_create: ") + nt_get_last_error_string());
            uploaded.push_back(t);
            params.referenceTextures[i].texture = (cudaTextureObject_t)t.texture;
            params.referenceTextures[i].width = W;
            params.referenceTextures[i].height = H;
            params.referenceTextures[i].numChannels = chans[i];
            params.referenceTextures[i].numMipLevels = 1;
            params.referenceTextures[i].lossWeight = weights[i];
            used += chans[i];
        }
        params.numReferenceTextures = 4;
        params.usedOutputChannels = used;

        // latents (main.cpp:657-738, one fp16 grid per feature here)
        const int gw[2] = {384, 192}, gh[2] = {384, 192};
        for (int f = 0; f < NT_NUM_FEATURES; ++f) {
            const size_t n = (size_t)gw[f] * gh[f] * C;
            Feature &feature = params.features[f];
            feature.width = gw[f];
            feature.height = gh[f];
            feature.numMips = 1;
            feature.unconstrainedGrid = device_zeros<half>(n);
            check(nt_init_latents(feature.unconstrainedGrid, (int64_t)n, 17u + f, nullptr) == NT_OK
                      ? cudaSuccess
                      : cudaErrorUnknown,
                  "nt_init_latents");
            feature.unconstrainedGradients = device_zeros<float>(n);
            feature.unconstrainedMoment1 = device_zeros<float>(n);
            feature.unconstrainedMoment2 = device_zeros<float>(n);
        }
        // network (main.cpp:740-788): padded column-major fp16 weights, zero biases (16 for layer 3)
        const int pad_in[3] = {32, 64, 64}, pad_out[3] = {64, 64, 16}, n_in[3] = {2 * C + 8, 64, 64};
        std::mt19937 rng(1337u);
        for (int l = 0; l < NT_NUM_NETWORK_LAYERS; ++l) {
            const size_t n = (size_t)pad_in[l] * pad_out[l];
            std::vector<half> w(n, __float2half(0.f));
            std::normal_distribution<float> N(0.f, std::sqrt(2.f / (float)pad_in[l]));
            for (int o = 0; o < (l == 2 ? used : 64); ++o)
                for (int i = 0; i < n_in[l]; ++i) w[(size_t)o * pad_in[l] + i] = __float2half(N(rng));
            params.networkWeights[l] = device_zeros<half>(n);
            check(cudaMemcpy(params.networkWeights[l], w.data(), n * sizeof(half), cudaMemcpyHostToDevice), "weights");
            const size_t nb = l == 2 ? NT_OUTPUT_SIZE : 64;
            params.networkWeightGradients[l] = device_zeros<float>(n);
            params.networkWeightMoment1[l] = device_zeros<float>(n);
            params.networkWeightMoment2[l] = device_zeros<float>(n);
            params.networkBiases[l] = device_zeros<half>(nb);
            params.networkBiasGradients[l] = device_zeros<float>(nb);
            params.networkBiasMoment1[l] = device_zeros<float>(nb);
            params.networkBiasMoment2[l] = device_zeros<float>(nb);
        }
        params.networkAdam = {0.9f, 0.99f, 5e-3f, 1e-8f};
        params.featureAdam = {0.9f, 0.99f, 1e-2f, 1e-8f};
        params.imageWidth = W;
        params.imageHeight = H;
        params.numSamples = 512 * 512;
        float *loss = device_zeros<float>(1);
        params.lossAccum = loss;

        // main.cpp:1037-1077
        std::mt19937 regionRng(20260411u);
        std::uniform_int_distribution<int> randomRegionX(0, std::max(0, params.imageWidth - 512));
        std::uniform_int_distribution<int> randomRegionY(0, std::max(0, params.imageHeight - 512));
        const float baseFeatureLearningRate = params.featureAdam.learningRate;
        float first = 0.f, last = 0.f;
        for (int iter = 0; iter < iters; ++iter) {
            params.texelOffsetX = randomRegionX(regionRng);
            params.texelOffsetY = randomRegionY(regionRng);
            const TrainingKernelType type = TrainingKernelType::UNCONSTRAINED;
            params.featureAdam.learningRate = baseFeatureLearningRate * std::pow(0.9995f, (float)iter);
            check(cudaMemset(loss, 0, sizeof(float)), "cudaMemset");
            InvokeTraining(params, type);
            InvokeOptimizeNetwork(params);
            InvokeOptimizeFeatures(params, type);
            params.step++;
            float l = 0.f;
            check(cudaMemcpy(&l, loss, sizeof(float), cudaMemcpyDeviceToHost), "loss");
            if (iter == 0) first = l;
            last = l;
        }
        // main.cpp:1011-1016, :1089-1100: [N][NT_OUTPUT_SIZE] fp32 output and the MSE accumulator
        const size_t count = (size_t)W * H;
        params.inferenceOutput = device_zeros<float>(count * NT_OUTPUT_SIZE);
        params.inferenceMseAccum = device_zeros<float>(1);
        InvokeInference(params);
        check(cudaDeviceSynchronize(), "cudaDeviceSynchronize(inference)");
        std::vector<float> out(count * NT_OUTPUT_SIZE);
        float sse = 0.f;
        check(cudaMemcpy(out.data(), params.inferenceOutput, out.size() * sizeof(float), cudaMemcpyDeviceToHost),
              "inferenceOutput");
        check(cudaMemcpy(&sse, params.inferenceMseAccum, sizeof(float), cudaMemcpyDeviceToHost), "mse");
        bool zero_tail = true;  // channels past usedOutputChannels are written as 0
        for (size_t i = 0; i < count; ++i)
            for (int c = used; c < NT_OUTPUT_SIZE; ++c) zero_tail = zero_tail && out[i * NT_OUTPUT_SIZE + c] == 0.f;
        std::printf("{\"iters\": %d, \"loss_first\": %.6g, \"loss_last\": %.6g, \"mse\": %.6g, \"zero_tail\": %s}\n",
                    iters, first, last, sse / (float)(count * used), zero_tail ? "true" : "false");
        for (NtReferenceTexture &t : uploaded) nt_reference_texture_destroy(&t);
        return last < first && std::isfinite(sse) && zero_tail ? 0 : 2;
    } catch (const std::exception &e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        for (NtReferenceTexture &t : uploaded) nt_reference_texture_destroy(&t);
        return 3;
    }
}

// driver_loop.cpp -- the reference driver's training loop (mavenkim2/neural_textures
// main.cpp:1037-1091) written against the C++ drop-in headers: KernelParams by value, the four
// Invoke* entry points, RunForwardPassTest, std::runtime_error on failure.
//
//   driver_loop --invalid   a rejected call surfaces as std::runtime_error (no GPU needed)
//   driver_loop [iters]     known-answer test, `iters` training steps on a synthetic 256^2
//                           material, inference with MSE; prints one JSON line
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
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

// fp16 bits of a float (round to nearest even; normal range only, enough for small weights)
uint16_t to_half(float f)
{
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    int32_t exp = (int32_t)((x >> 23) & 0xff) - 127 + 15;
    uint32_t mant = x & 0x7fffffu;
    if (exp <= 0) return (uint16_t)sign;
    uint32_t h = sign | ((uint32_t)exp << 10) | (mant >> 13);
    const uint32_t rest = mant & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)h;
}

KernelParams invalid_params()
{
    KernelParams p{};
    p.latent_channels = 7;  // rejected: 8 or 12 only
    p.output_channels = 8;
    return p;
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
    try {
        if (!RunForwardPassTest()) throw std::runtime_error("forward-pass known-answer test failed");

        const int W = 256, H = 256, C = 8, COUT = 8;
        const int gw[2] = {128, 64}, gh[2] = {128, 64};
        KernelParams params{};
        params.latent_channels = C;
        params.output_channels = COUT;
        for (int f = 0; f < NT_NUM_FEATURES; ++f) {
            const size_t n = (size_t)gw[f] * gh[f] * C;
            void *grid = device_zeros<uint16_t>(n);
            check(nt_init_latents(grid, (int64_t)n, 17u + f, nullptr) == NT_OK ? cudaSuccess : cudaErrorUnknown,
                  "nt_init_latents");
            params.features[f] = {grid, device_zeros<float>(n), device_zeros<float>(n), device_zeros<float>(n),
                                  gw[f], gh[f], 1};
        }
        const int pad_in[3] = {32, 64, 64}, pad_out[3] = {64, 64, 16}, n_in[3] = {2 * C + 8, 64, 64};
        uint32_t lcg = 12345u;
        for (int l = 0; l < NT_NUM_NETWORK_LAYERS; ++l) {  // He-normal-like uniform weights, zero biases
            const size_t n = (size_t)pad_in[l] * pad_out[l];
            std::vector<uint16_t> w(n, 0);
            const float scale = std::sqrt(6.0f / (float)pad_in[l]);
            for (int o = 0; o < (l == 2 ? COUT : 64); ++o)
                for (int i = 0; i < n_in[l]; ++i) {
                    lcg = lcg * 1664525u + 1013904223u;
                    w[(size_t)o * pad_in[l] + i] = to_half(scale * ((float)(lcg >> 8) / 16777216.0f * 2.f - 1.f));
                }
            uint16_t *dw = device_zeros<uint16_t>(n);
            check(cudaMemcpy(dw, w.data(), n * 2, cudaMemcpyHostToDevice), "weights");
            const size_t nb = l == 2 ? COUT : 64;
            params.network_weights[l] = dw;
            params.network_weight_gradients[l] = device_zeros<float>(n);
            params.network_weight_moment1[l] = device_zeros<float>(n);
            params.network_weight_moment2[l] = device_zeros<float>(n);
            params.network_biases[l] = device_zeros<uint16_t>(nb);
            params.network_bias_gradients[l] = device_zeros<float>(nb);
            params.network_bias_moment1[l] = device_zeros<float>(nb);
            params.network_bias_moment2[l] = device_zeros<float>(nb);
        }
        params.network_adam = {0.9f, 0.99f, 5e-3f, 1e-8f};
        params.feature_adam = {0.9f, 0.99f, 1e-2f, 1e-8f};
        void *target = device_zeros<uint16_t>((size_t)W * H * COUT);
        check(nt_generate_target(target, W, H, COUT, 3u, 0, nullptr) == NT_OK ? cudaSuccess : cudaErrorUnknown,
              "nt_generate_target");
        params.target = target;
        for (int c = 0; c < COUT; ++c) params.channel_loss_weights[c] = 1.f;
        params.image_width = W;
        params.image_height = H;
        params.lattice_width = params.lattice_height = 128;
        params.sample_stride_x = params.sample_stride_y = 2.f;
        params.num_samples = 128 * 128;
        float *loss = device_zeros<float>(1);
        params.loss_accum = loss;

        float first = 0.f, last = 0.f;
        for (int iter = 0; iter < iters; ++iter) {  // main.cpp:1037-1077
            check(cudaMemset(loss, 0, sizeof(float)), "cudaMemset");
            InvokeTraining(params, TrainingKernelType::UNCONSTRAINED);
            InvokeOptimizeNetwork(params);
            InvokeOptimizeFeatures(params, TrainingKernelType::UNCONSTRAINED);
            params.step++;
            float l = 0.f;
            check(cudaMemcpy(&l, loss, sizeof(float), cudaMemcpyDeviceToHost), "loss");
            if (iter == 0) first = l;
            last = l;
        }
        float *out = device_zeros<float>((size_t)W * H * COUT);
        float *mse = device_zeros<float>(1);
        params.inference_output = out;
        params.inference_output_dtype = NT_DTYPE_F32;
        params.inference_mse_accum = mse;
        InvokeInference(params);  // main.cpp:1091
        float sse = 0.f;
        check(cudaMemcpy(&sse, mse, sizeof(float), cudaMemcpyDeviceToHost), "mse");
        std::printf("{\"iters\": %d, \"loss_first\": %.6g, \"loss_last\": %.6g, \"mse\": %.6g}\n", iters, first,
                    last, sse / (float)(W * H * COUT));
        return last < first && std::isfinite(sse) ? 0 : 2;
    } catch (const std::exception &e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 3;
    }
}

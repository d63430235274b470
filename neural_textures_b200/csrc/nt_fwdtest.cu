// nt_fwdtest.cu -- RunForwardPassTest(), the reference's known-answer test harness
// (mavenkim2/neural_textures tests/forward_pass_test.cu:152-275, declared in
// tests/forward_pass_test.h:6), rebuilt on this library's tensor-core ForwardPassGeneric.
//
// The test data are the reference's closed-form patterns (tests/forward_pass_test.cu:45-108:
// 32 lanes x 12 fp16 inputs, 12 -> 16 (ReLU) -> 16 with column-major padded weights), the
// expected values come from the same fp32 host evaluation (tests/forward_pass_test.cu:110-150)
// and the tolerance is the reference's absolute 2e-2 (tests/forward_pass_test.cu:236).  The
// formulas have to match the reference's for the test to mean the same thing.
#include <cmath>
#include <cstdio>
#include <vector>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "neural_textures/forward_pass_test.h"
#include "neural_textures/mlp.h"
#include "nt_capi.h"
#include "nt_common.cuh"

namespace neural_textures {

constexpr int kLanes = 32, kIn = 12, kHidden = 16, kOut = 16;

__global__ static void ForwardPassTestKernel(__half *outputs, const __half *inputs, const __half *w0,
                                             const __half *w1, const __half *b0, const __half *b1)
{
    const int lane = threadIdx.x & 31;
    ForwardPass12x16xOutput(inputs + lane * kIn, w0, w1, b0, b1, outputs + lane * kOut);
}

static void InitializeForwardPassTestData(std::vector<__half> &in, std::vector<__half> &w0, std::vector<__half> &w1,
                                          std::vector<__half> &b0, std::vector<__half> &b1)
{
    in.resize(kLanes * kIn);
    w0.resize(kHidden * kHidden);
    w1.resize(kHidden * kHidden);
    b0.resize(kHidden);
    b1.resize(kHidden);
    for (int lane = 0; lane < kLanes; ++lane)
        for (int k = 0; k < kIn; ++k)
            in[lane * kIn + k] =
                __float2half(0.125f + 0.01171875f * float(lane + 1) + 0.0068359375f * float(k + 1));
    for (int o = 0; o < kHidden; ++o)
        for (int i = 0; i < kHidden; ++i) {
            const float v = i < kIn ? 0.0625f + 0.0048828125f * float((3 * o + 1) % 7) +
                                          0.0029296875f * float((5 * i + 2) % 11)
                                    : 0.f;
            w0[i + o * kHidden] = __float2half(v);
            w1[i + o * kHidden] = __float2half(0.09375f + 0.00341796875f * float((7 * o + 3) % 13) +
                                               0.001953125f * float((2 * i + 5) % 9));
        }
    for (int o = 0; o < kHidden; ++o) {
        b0[o] = __float2half(0.046875f + 0.00390625f * float((4 * o + 1) % 9));
        b1[o] = __float2half(0.078125f + 0.005859375f * float((5 * o + 2) % 7));
    }
}

static void ComputeForwardPassReference(const std::vector<__half> &in, const std::vector<__half> &w0,
                                        const std::vector<__half> &w1, const std::vector<__half> &b0,
                                        const std::vector<__half> &b1, std::vector<float> &ref)
{
    ref.assign(kLanes * kOut, 0.f);
    for (int lane = 0; lane < kLanes; ++lane) {
        float hidden[kHidden];
        for (int o = 0; o < kHidden; ++o) {
            float s = __half2float(b0[o]);
            for (int i = 0; i < kHidden; ++i) {
                const float x = i < kIn ? __half2float(in[lane * kIn + i]) : 0.f;
                s += x * __half2float(w0[i + o * kHidden]);
            }
            hidden[o] = s > 0.f ? s : 0.f;
        }
        for (int o = 0; o < kOut; ++o) {
            float s = __half2float(b1[o]);
            for (int i = 0; i < kHidden; ++i) s += hidden[i] * __half2float(w1[i + o * kHidden]);
            ref[lane * kOut + o] = s;
        }
    }
}

static bool Check(cudaError_t e, const char *what)
{
    if (e == cudaSuccess) return true;
    std::printf("%s: %s\n", what, cudaGetErrorString(e));
    return false;
}

bool RunForwardPassTest()
{
    std::vector<__half> in, w0, w1, b0, b1;
    std::vector<float> ref;
    InitializeForwardPassTestData(in, w0, w1, b0, b1);
    ComputeForwardPassReference(in, w0, w1, b0, b1, ref);

    // one allocation holding every operand, 256-byte aligned sub-buffers
    const size_t off_in = 0, off_w0 = 1024, off_w1 = 1536, off_b0 = 2048, off_b1 = 2304, off_out = 2560;
    const size_t total = off_out + kLanes * kOut * sizeof(__half);
    unsigned char *dev = nullptr;
    bool ok = Check(cudaMalloc(&dev, total), "cudaMalloc");
    std::vector<__half> out(kLanes * kOut, __float2half(0.f));
    if (ok) {
        ok = Check(cudaMemcpy(dev + off_in, in.data(), in.size() * 2, cudaMemcpyHostToDevice), "cudaMemcpy(inputs)") &&
             Check(cudaMemcpy(dev + off_w0, w0.data(), w0.size() * 2, cudaMemcpyHostToDevice), "cudaMemcpy(w0)") &&
             Check(cudaMemcpy(dev + off_w1, w1.data(), w1.size() * 2, cudaMemcpyHostToDevice), "cudaMemcpy(w1)") &&
             Check(cudaMemcpy(dev + off_b0, b0.data(), b0.size() * 2, cudaMemcpyHostToDevice), "cudaMemcpy(b0)") &&
             Check(cudaMemcpy(dev + off_b1, b1.data(), b1.size() * 2, cudaMemcpyHostToDevice), "cudaMemcpy(b1)");
    }
    if (ok) {
        ForwardPassTestKernel<<<1, kLanes>>>(
            reinterpret_cast<__half *>(dev + off_out), reinterpret_cast<const __half *>(dev + off_in),
            reinterpret_cast<const __half *>(dev + off_w0), reinterpret_cast<const __half *>(dev + off_w1),
            reinterpret_cast<const __half *>(dev + off_b0), reinterpret_cast<const __half *>(dev + off_b1));
        nt::count_launch();
        ok = Check(cudaGetLastError(), "ForwardPassTestKernel launch") &&
             Check(cudaDeviceSynchronize(), "ForwardPassTestKernel sync") &&
             Check(cudaMemcpy(out.data(), dev + off_out, out.size() * 2, cudaMemcpyDeviceToHost), "cudaMemcpy(out)");
    }
    const float tolerance = 2e-2f;
    for (int lane = 0; ok && lane < kLanes; ++lane)
        for (int i = 0; i < kOut; ++i) {
            const float a = __half2float(out[lane * kOut + i]), e = ref[lane * kOut + i];
            if (std::fabs(a - e) > tolerance) {
                std::printf("ForwardPassTest mismatch at lane=%d output=%d actual=%f expected=%f diff=%f\n", lane, i,
                            a, e, std::fabs(a - e));
                ok = false;
                break;
            }
        }
    if (dev) cudaFree(dev);
    if (ok) std::printf("ForwardPassTest passed\n");
    return ok;
}

}  // namespace neural_textures

extern "C" int32_t nt_run_forward_pass_test(void) { return neural_textures::RunForwardPassTest() ? 1 : 0; }

extern "C" nt_status nt_forward_pass_12x16x16(const void *inputs, const void *w0, const void *w1, const void *b0,
                                              const void *b1, void *outputs, nt_stream_t stream)
{
    if (!inputs || !w0 || !w1 || !b0 || !b1 || !outputs) return NT_ERR_INVALID_ARG;
    neural_textures::ForwardPassTestKernel<<<1, 32, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<__half *>(outputs), reinterpret_cast<const __half *>(inputs),
        reinterpret_cast<const __half *>(w0), reinterpret_cast<const __half *>(w1),
        reinterpret_cast<const __half *>(b0), reinterpret_cast<const __half *>(b1));
    nt::count_launch();
    return cudaGetLastError() == cudaSuccess ? NT_OK : NT_ERR_CUDA;
}

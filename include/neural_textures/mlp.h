// neural_textures/mlp.h -- header-only device library with the reference's network API.
//
// Mirrors mavenkim2/neural_textures mlp.h (same names, same argument meaning):
//   ForwardPassGeneric<in, out, act>           mlp.h:18-40
//   ForwardPass12x16xOutput                    mlp.h:42-63   (known-answer test network)
//   BackwardPassGeneric<threads, in, out, act> mlp.h:222-257
// The reference builds these on tiny-cuda-nn's warp MMA vector types; here a warp holds
// 32 samples (one per lane, as in the reference) as a WarpMatrix in the fp16 A-fragment
// layout of mma.m16n8k16 and every contraction runs on the tensor cores with fp32
// accumulation.  Weights are column-major and padded to multiples of 16 exactly as in the
// reference (W[out * AlignUp(in, 16) + in], main.cpp:195); biases have one entry per output.
//
// These functions read weights from any address space.  The fused kernels of the library
// (decode, training) use the same fragment arithmetic with shared-memory staging.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace neural_textures {

enum class LayerActivation { None, ReLU };

__host__ __device__ constexpr int AlignUp(int v, int a) { return (v + a - 1) / a * a; }

namespace detail {

__device__ __forceinline__ uint32_t pack2(float lo, float hi)
{
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ float2 unpack2(uint32_t v)
{
    __half2 h = *reinterpret_cast<__half2 *>(&v);
    return __half22float2(h);
}

__device__ __forceinline__ void mma(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Transpose an 8x8 fp16 block held one 32-bit register per lane (lane = row * 4 + colpair).
__device__ __forceinline__ uint32_t trans8x8(uint32_t v)
{
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(d) : "r"(v));
    return d;
}

}  // namespace detail

// 32 samples (rows, one per lane) x COLS fp16 columns in mma A-fragment layout:
// r[mt][kt] covers rows 16 mt .. 16 mt + 15 and columns 16 kt .. 16 kt + 15.
template <int COLS>
struct WarpMatrix {
    static_assert(COLS % 16 == 0, "WarpMatrix columns must be a multiple of 16");
    uint32_t r[2][COLS / 16][4];
};

// Per-lane row (N fp16 values of this lane's sample) -> WarpMatrix (tcnn hvec -> mma_vec).
template <int N>
__device__ inline WarpMatrix<AlignUp(N, 16)> FromLaneRows(const __half *row)
{
    constexpr int P = AlignUp(N, 16);
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    uint32_t words[P / 2];
#pragma unroll
    for (int j = 0; j < P / 2; ++j) {
        const float lo = 2 * j < N ? __half2float(row[2 * j]) : 0.f;
        const float hi = 2 * j + 1 < N ? __half2float(row[2 * j + 1]) : 0.f;
        words[j] = detail::pack2(lo, hi);
    }
    WarpMatrix<P> m;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int kt = 0; kt < P / 16; ++kt)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int src = mt * 16 + g + 8 * (q & 1);
                const int base = kt * 8 + 4 * (q >> 1);
                uint32_t v = 0;
#pragma unroll
                for (int tt = 0; tt < 4; ++tt) {
                    const uint32_t x = __shfl_sync(0xffffffffu, words[base + tt], src);
                    if (t == tt) v = x;
                }
                m.r[mt][kt][q] = v;
            }
    return m;
}

// WarpMatrix -> this lane's row (first N columns).
template <int N, int P>
__device__ inline void ToLaneRow(const WarpMatrix<P> &m, __half *row)
{
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < P / 2; ++j) {
        const int kt = j / 8, rhi = (j % 8) / 4;
        const int src = (lane & 7) * 4 + (j & 3);
        uint32_t v = 0;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int rlo = 0; rlo < 2; ++rlo) {
                const uint32_t x = __shfl_sync(0xffffffffu, m.r[mt][kt][rlo + 2 * rhi], src);
                if ((lane >> 4) == mt && ((lane >> 3) & 1) == rlo) v = x;
            }
        const float2 f = detail::unpack2(v);
        if (2 * j < N) row[2 * j] = __float2half_rn(f.x);
        if (2 * j + 1 < N) row[2 * j + 1] = __float2half_rn(f.y);
    }
}

// mlp.h:18-40: y = act(x W + b), fp16 operands, fp32 accumulation, fp16 result.
template <int inputSize, int outputSize, LayerActivation activation = LayerActivation::ReLU>
__device__ inline WarpMatrix<AlignUp(outputSize, 16)>
ForwardPassGeneric(const WarpMatrix<AlignUp(inputSize, 16)> &inputsMatrix, const __half *weightsLayer,
                   const __half *biasesLayer)
{
    constexpr int PI = AlignUp(inputSize, 16), PO = AlignUp(outputSize, 16);
    constexpr int KT = PI / 16, NT = PO / 8;
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    float acc[2][NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int n = nt * 8 + 2 * t;
        const float b0 = (biasesLayer && n < outputSize) ? __half2float(biasesLayer[n]) : 0.f;
        const float b1 = (biasesLayer && n + 1 < outputSize) ? __half2float(biasesLayer[n + 1]) : 0.f;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
            acc[mt][nt][0] = b0;
            acc[mt][nt][1] = b1;
            acc[mt][nt][2] = b0;
            acc[mt][nt][3] = b1;
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const __half *col = weightsLayer + (nt * 8 + g) * PI;
#pragma unroll
        for (int kt = 0; kt < KT; ++kt) {
            const uint32_t b0 = *reinterpret_cast<const uint32_t *>(col + kt * 16 + 2 * t);
            const uint32_t b1 = *reinterpret_cast<const uint32_t *>(col + kt * 16 + 8 + 2 * t);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) detail::mma(acc[mt][nt], inputsMatrix.r[mt][kt], b0, b1);
        }
    }
    WarpMatrix<PO> out;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int kt = 0; kt < PO / 16; ++kt)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float *c = acc[mt][2 * kt + (q >> 1)] + 2 * (q & 1);
                float lo = c[0], hi = c[1];
                if (activation == LayerActivation::ReLU) {
                    lo = fmaxf(lo, 0.f);
                    hi = fmaxf(hi, 0.f);
                }
                out.r[mt][kt][q] = detail::pack2(lo, hi);
            }
    return out;
}

// mlp.h:42-63: 12 inputs -> 16 (ReLU) -> 16 outputs, one sample per lane.
__device__ inline void ForwardPass12x16xOutput(const __half *sampledFeatures, const __half *weightsLayer0,
                                               const __half *weightsLayer1, const __half *biasesLayer0,
                                               const __half *biasesLayer1, __half *outputs16,
                                               __half *activatedHiddenLayer0 = nullptr)
{
    WarpMatrix<16> in = FromLaneRows<12>(sampledFeatures);
    WarpMatrix<16> hidden = ForwardPassGeneric<12, 16>(in, weightsLayer0, biasesLayer0);
    if (activatedHiddenLayer0) ToLaneRow<16>(hidden, activatedHiddenLayer0);
    WarpMatrix<16> out = ForwardPassGeneric<16, 16, LayerActivation::None>(hidden, weightsLayer1, biasesLayer1);
    ToLaneRow<16>(out, outputs16);
}

// The build's network: 32 inputs -> 64 (ReLU) -> 64 (ReLU) -> outputSize (linear).
template <int outputSize>
__device__ inline void ForwardPass32x64x64xOutput(const __half *networkInput32, const __half *weightsLayer0,
                                                  const __half *weightsLayer1, const __half *weightsLayer2,
                                                  const __half *biasesLayer0, const __half *biasesLayer1,
                                                  const __half *biasesLayer2, __half *outputs)
{
    WarpMatrix<32> in = FromLaneRows<32>(networkInput32);
    WarpMatrix<64> h0 = ForwardPassGeneric<32, 64>(in, weightsLayer0, biasesLayer0);
    WarpMatrix<64> h1 = ForwardPassGeneric<64, 64>(h0, weightsLayer1, biasesLayer1);
    WarpMatrix<AlignUp(outputSize, 16)> out =
        ForwardPassGeneric<64, outputSize, LayerActivation::None>(h1, weightsLayer2, biasesLayer2);
    ToLaneRow<outputSize>(out, outputs);
}

// mlp.h:222-257.  Given dL/dY of the layer (32 samples) and the layer's input (the
// post-activation output of the previous layer), accumulates dL/dW (fp32, same padded
// column-major layout as the weights) and dL/db into global memory and returns dL/dX,
// masked by the derivative of `activation` evaluated on the input (mlp.h:243-247).
// numThreads is kept for signature compatibility: the reduction here is per warp
// (shuffles + one atomic per element), the fused kernels reduce per CTA instead.
template <uint32_t numThreads, uint32_t inputSize, uint32_t outputSize,
          LayerActivation activation = LayerActivation::ReLU>
__device__ inline WarpMatrix<AlignUp(inputSize, 16)>
BackwardPassGeneric(const WarpMatrix<AlignUp(outputSize, 16)> &outputGradientMatrix,
                    const WarpMatrix<AlignUp(inputSize, 16)> &layerInput, const __half *weights,
                    float *layerWeightGradients, float *layerBiasGradients)
{
    constexpr int PI = AlignUp(inputSize, 16), PO = AlignUp(outputSize, 16);
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;

    // db = sum over the 32 rows (mlp.h:101-153)
#pragma unroll
    for (int kt = 0; kt < PO / 16; ++kt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int rlo = 0; rlo < 2; ++rlo) {
                    const float2 f = detail::unpack2(outputGradientMatrix.r[mt][kt][rlo + 2 * h]);
                    s0 += f.x;
                    s1 += f.y;
                }
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                s0 += __shfl_xor_sync(0xffffffffu, s0, o);
                s1 += __shfl_xor_sync(0xffffffffu, s1, o);
            }
            const int col = kt * 16 + 8 * h + 2 * t;
            if (g == 0 && layerBiasGradients) {
                if (col < (int)outputSize) atomicAdd(layerBiasGradients + col, s0);
                if (col + 1 < (int)outputSize) atomicAdd(layerBiasGradients + col + 1, s1);
            }
        }

    // dX = dY W^T  (B[k = out][n = in] = W[out * PI + in])
    float dx[2][PI / 8][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < PI / 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) dx[mt][nt][e] = 0.f;
#pragma unroll
    for (int kt = 0; kt < PO / 16; ++kt)
#pragma unroll
        for (int nt = 0; nt < PI / 8; ++nt) {
            const int n = nt * 8 + g;
            const int k = kt * 16 + 2 * t;
            const __half2 lo = __halves2half2(weights[k * PI + n], weights[(k + 1) * PI + n]);
            const __half2 hi = __halves2half2(weights[(k + 8) * PI + n], weights[(k + 9) * PI + n]);
            const uint32_t b0 = *reinterpret_cast<const uint32_t *>(&lo);
            const uint32_t b1 = *reinterpret_cast<const uint32_t *>(&hi);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) detail::mma(dx[mt][nt], outputGradientMatrix.r[mt][kt], b0, b1);
        }

    // dW = X^T dY over the 32 samples (K), via register transposes of 8x8 blocks
    float dw[PI / 16][PO / 8][4];
#pragma unroll
    for (int mi = 0; mi < PI / 16; ++mi)
#pragma unroll
        for (int nj = 0; nj < PO / 8; ++nj)
#pragma unroll
            for (int e = 0; e < 4; ++e) dw[mi][nj][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
        for (int mi = 0; mi < PI / 16; ++mi) {
            const uint32_t *x = layerInput.r[ks][mi];
            const uint32_t a[4] = {detail::trans8x8(x[0]), detail::trans8x8(x[2]), detail::trans8x8(x[1]),
                                   detail::trans8x8(x[3])};
#pragma unroll
            for (int nj = 0; nj < PO / 8; ++nj) {
                const uint32_t *y = outputGradientMatrix.r[ks][nj >> 1];
                const uint32_t b0 = detail::trans8x8(y[2 * (nj & 1)]);
                const uint32_t b1 = detail::trans8x8(y[2 * (nj & 1) + 1]);
                detail::mma(dw[mi][nj], a, b0, b1);
            }
        }
    }
    if (layerWeightGradients) {
#pragma unroll
        for (int mi = 0; mi < PI / 16; ++mi)
#pragma unroll
            for (int nj = 0; nj < PO / 8; ++nj)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int in = mi * 16 + g + 8 * (e >> 1);
                    const int out = nj * 8 + 2 * t + (e & 1);
                    if (in < (int)inputSize && out < (int)outputSize)
                        atomicAdd(layerWeightGradients + out * PI + in, dw[mi][nj][e]);
                }
    }

    WarpMatrix<PI> result;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int kt = 0; kt < PI / 16; ++kt)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float *c = dx[mt][2 * kt + (q >> 1)] + 2 * (q & 1);
                float lo = c[0], hi = c[1];
                if (activation == LayerActivation::ReLU) {
                    const float2 in = detail::unpack2(layerInput.r[mt][kt][q]);
                    lo = in.x > 0.f ? lo : 0.f;
                    hi = in.y > 0.f ? hi : 0.f;
                }
                result.r[mt][kt][q] = detail::pack2(lo, hi);
            }
    return result;
}

}  // namespace neural_textures

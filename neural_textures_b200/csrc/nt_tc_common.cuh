// nt_tc_common.cuh -- pieces shared by the tcgen05 training and decode kernels: the tile
// shape, the operand images of the 32 -> 64 -> 64 -> (<= 16) network in shared memory
// (core-matrix layout of nt_umma.cuh, biases folded in as an extra input column) and the
// TMEM -> fp16 activation epilogue.
#pragma once

#include "nt_kernels.cuh"
#include "nt_mma.cuh"
#include "nt_umma.cuh"

namespace nt {
namespace tc {

constexpr int kTileW = 16, kTileH = 8, kTileN = 128;  // one tile = 16 x 8 samples / texels (M = 128)
constexpr int kHC = 10;  // core-matrix chunks per H row: 64 activations, 1, 0 x 15
constexpr int kHW = kHC * 8;
constexpr uint32_t kSpinLimit = 1u << 22;

template <int C>
struct Cfg {
    static constexpr int kBias1 = 2 * C + 8;                 // column of the constant 1 in X
    static constexpr int XC = ((kBias1 + 1 + 15) / 16) * 2;  // chunks of 8 halves per X row
    static constexpr int XW = XC * 8;                        // 32 (C = 8) or 48 (C = 12)
    static constexpr int LC = C / 4;                         // X chunks holding the 2C latents
    static constexpr int NX = ((2 * C + 15) / 16) * 16;      // dX columns produced by B1
    static constexpr int DXS = 2 * C + 4;                    // fp32 dX row stride (floats)
};

__device__ __forceinline__ void st16(uint8_t *base, uint32_t off, uint32_t a, uint32_t b, uint32_t c, uint32_t d)
{
    *reinterpret_cast<uint4 *>(base + off) = make_uint4(a, b, c, d);
}

// ---- weights: shared-memory operand images with the biases folded in -------------------

// S: any shared-memory struct with the W1, W2, W3 operand images; nth threads take part.
template <int C, class S>
__device__ __forceinline__ void stage_weights_tc(S &w, const NetView &net, int tid, int nth)
{
    using K = Cfg<C>;
    constexpr int n1 = 64 * K::XC, n2 = 64 * kHC, n3 = 16 * kHC;
    for (int i = tid; i < n1 + n2 + n3; i += nth) {
        int o, j, kch, nin, pad, which;
        if (i < n1) {
            o = i / K::XC, j = i % K::XC, kch = K::XC, nin = K::kBias1, pad = 32, which = 0;
        } else if (i < n1 + n2) {
            o = (i - n1) / kHC, j = (i - n1) % kHC, kch = kHC, nin = 64, pad = 64, which = 1;
        } else {
            o = (i - n1 - n2) / kHC, j = (i - n1 - n2) % kHC, kch = kHC, nin = 64, pad = 64, which = 2;
        }
        const __half *src = net.W[which], *bias = net.b[which];
        uint8_t *dst = which == 0 ? w.W1 : (which == 1 ? w.W2 : w.W3);
        const bool row_ok = which != 2 || o < net.cout;
        uint32_t v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            __half x[2];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int in = 8 * j + 2 * e + q;
                x[q] = __float2half(0.f);
                if (row_ok) {
                    if (in < nin) x[q] = src[o * pad + in];
                    else if (in == nin) x[q] = bias[o];
                }
            }
            v[e] = (uint32_t)__half_as_ushort(x[0]) | ((uint32_t)__half_as_ushort(x[1]) << 16);
        }
        st16(dst, umma::cm_offset(o, 8 * j, kch), v[0], v[1], v[2], v[3]);
    }
}

// ---- epilogue ----------------------------------------------------------------------------

// TMEM row (32 columns from taddr) -> fp16 -> relu -> 4 chunks of an H row.  Rounding is
// monotonic and keeps 0, so relu(round(x)) has the bits of round(relu(x)) up to the sign
// of zero, which no later product or mask can see.
__device__ __forceinline__ void relu_store32(uint32_t taddr, uint8_t *H, int r, int chunk0)
{
    uint32_t v[32];
    umma::ld16(taddr, *reinterpret_cast<uint32_t(*)[16]>(v));
    umma::ld16(taddr + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
    umma::wait_ld();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t h[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)  // cvt.rn.relu: both lanes rounded to fp16, negatives to 0, in one step
            asm("cvt.rn.relu.f16x2.f32 %0, %1, %2;"
                : "=r"(h[e])
                : "f"(__uint_as_float(v[8 * q + 2 * e + 1])), "f"(__uint_as_float(v[8 * q + 2 * e])));
        st16(H, umma::cm_offset(r, 8 * (chunk0 + q), kHC), h[0], h[1], h[2], h[3]);
    }
}

// Descriptor whose start address advances by `bytes` (the address field holds addr >> 4 and
// every operand lies below 256 KB, so the field never carries into its neighbours).
__device__ __forceinline__ uint64_t dadv(uint64_t d, uint32_t bytes) { return d + (uint64_t)(bytes >> 4); }

}  // namespace tc
}  // namespace nt

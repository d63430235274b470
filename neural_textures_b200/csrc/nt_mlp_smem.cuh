// nt_mlp_smem.cuh -- shared-memory image of the 32 -> 64 -> 64 -> (<=16) network.
//
// The reference streams its weights from global memory inside every warp
// (mlp.h:29, from_linear_memory); here each CTA stages them once into padded shared rows
// and keeps them resident for all the tiles it processes.
#pragma once

#include "nt_kernels.cuh"
#include "nt_mma.cuh"

namespace nt {

struct MlpSmem {
    __half W1[64 * kStrideK32];  // [out 64][in 32]
    __half W2[64 * kStrideK64];  // [out 64][in 64]
    __half W3[16 * kStrideK64];  // [out 16][in 64]
    float b1[64];
    float b2[64];
    float b3[16];
};

__device__ __forceinline__ void stage_weights(MlpSmem &s, const NetView &net)
{
    const int tid = threadIdx.x, nth = blockDim.x;
    for (int i = tid; i < 64 * 4; i += nth) {
        const int r = i >> 2, q = i & 3;
        *reinterpret_cast<uint4 *>(&s.W1[r * kStrideK32 + q * 8]) =
            __ldg(reinterpret_cast<const uint4 *>(net.W[0] + r * 32 + q * 8));
    }
    for (int i = tid; i < 64 * 8; i += nth) {
        const int r = i >> 3, q = i & 7;
        *reinterpret_cast<uint4 *>(&s.W2[r * kStrideK64 + q * 8]) =
            __ldg(reinterpret_cast<const uint4 *>(net.W[1] + r * 64 + q * 8));
    }
    for (int i = tid; i < 16 * 8; i += nth) {
        const int r = i >> 3, q = i & 7;
        *reinterpret_cast<uint4 *>(&s.W3[r * kStrideK64 + q * 8]) =
            __ldg(reinterpret_cast<const uint4 *>(net.W[2] + r * 64 + q * 8));
    }
    for (int i = tid; i < 64; i += nth) {
        s.b1[i] = __half2float(net.b[0][i]);
        s.b2[i] = __half2float(net.b[1][i]);
    }
    for (int i = tid; i < 16; i += nth) s.b3[i] = i < net.cout ? __half2float(net.b[2][i]) : 0.f;
}

// Forward of the 32 rows owned by this warp: X (shared, stride 40) -> H1, H2 (shared,
// stride 72, fp16 post-ReLU) and the output accumulators (fp32, bias included).
template <int NT3>
__device__ __forceinline__ void warp_forward(const MlpSmem &s, const __half *X, __half *H1, __half *H2,
                                             int r0, int lane, float (&acc3)[2][NT3][4])
{
    uint32_t xa[2][2][4];
    load_a<2, 2>(xa, smem_addr(X), kStrideK32, r0, lane);
    uint32_t h[2][4][4];
    {
        float acc[2][8][4];
        acc_init_bias<2, 8>(acc, s.b1, lane);
        warp_gemm_w<2, 2, 8>(acc, xa, smem_addr(s.W1), kStrideK32, lane);
        acc_to_a<2, 4, true>(h, acc);
    }
    if (H1) store_a<2, 4>(h, H1, kStrideK64, r0, lane);
    {
        float acc[2][8][4];
        acc_init_bias<2, 8>(acc, s.b2, lane);
        warp_gemm_w<2, 4, 8>(acc, h, smem_addr(s.W2), kStrideK64, lane);
        acc_to_a<2, 4, true>(h, acc);
    }
    if (H2) store_a<2, 4>(h, H2, kStrideK64, r0, lane);
    acc_init_bias<2, NT3>(acc3, s.b3, lane);
    warp_gemm_w<2, 4, NT3>(acc3, h, smem_addr(s.W3), kStrideK64, lane);
}

// Write fp16-rounded output accumulators into a shared [rows][16] matrix (stride 24).
template <int NT3>
__device__ __forceinline__ void store_out16(const float (&acc3)[2][NT3][4], __half *Y, int r0, int lane)
{
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT3; ++nt) {
            __half *p0 = Y + (r0 + mt * 16 + g) * kStrideK16 + nt * 8 + 2 * t;
            *reinterpret_cast<uint32_t *>(p0) = pack_half2(acc3[mt][nt][0], acc3[mt][nt][1]);
            *reinterpret_cast<uint32_t *>(p0 + 8 * kStrideK16) =
                pack_half2(acc3[mt][nt][2], acc3[mt][nt][3]);
        }
}

}  // namespace nt

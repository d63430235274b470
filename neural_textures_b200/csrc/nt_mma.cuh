// nt_mma.cuh -- warp-level fp16 tensor-core primitives (mma.sync m16n8k16, fp32 accumulate)
// and the shared-memory layouts of the fused tiny MLP.
//
// Fragment layouts (PTX ISA, mma.m16n8k16 .f16): with g = lane / 4 and t = lane % 4,
//   A (16x16, row):  r0 = (g, 2t..2t+1)  r1 = (g+8, 2t..)  r2 = (g, 2t+8..)  r3 = (g+8, 2t+8..)
//   B (16x8,  col):  r0 = (k 2t..2t+1, n g)   r1 = (k 2t+8.., n g)
//   C (16x8, fp32):  c0,c1 = (g, 2t..2t+1)    c2,c3 = (g+8, 2t..2t+1)
// Two adjacent n8 accumulator tiles therefore form one k16 A fragment of the next layer,
// which keeps activations in registers between layers.
//
// Weights keep the reference's column-major layout (main.cpp:195): W[out * padIn + in], i.e.
// one row per output unit with the inputs contiguous, which is exactly the "col" B operand.
// Shared-memory rows are padded (32 -> 40, 64 -> 72, 16 -> 24 halves) so that the 8 row
// addresses of every ldmatrix phase hit 8 different 16-byte bank groups.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace nt {

constexpr int kStrideK32 = 40;  // halves per shared row of a 32-wide matrix
constexpr int kStrideK64 = 72;  // 64-wide
constexpr int kStrideK16 = 24;  // 16-wide

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t r[4], uint32_t addr)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t r[4], uint32_t addr)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2_t(uint32_t r[2], uint32_t addr)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(addr));
}

// ---------------------------------------------------------------------------------------
// Address helpers.  `base` is the shared address of row 0 / column 0, `stride` the row
// stride in halves.  All return the address this lane passes to ldmatrix.

// A fragment (rows r0..r0+15, cols c0..c0+15) of a row-major matrix.
__device__ __forceinline__ uint32_t a_frag_addr(uint32_t base, int stride, int r0, int c0, int lane)
{
    const int q = lane >> 3, r = lane & 7;
    return base + 2u * (uint32_t)((r0 + r + 8 * (q & 1)) * stride + c0 + 8 * (q >> 1));
}

// Two k16 B fragments (k0..k0+31) of one n8 tile (rows n0..n0+7) of an [n][k] matrix.
__device__ __forceinline__ uint32_t b_frag2k_addr(uint32_t base, int stride, int n0, int k0, int lane)
{
    const int q = lane >> 3, r = lane & 7;
    return base + 2u * (uint32_t)((n0 + r) * stride + k0 + 8 * q);
}

// Transposed B: B[k][n] = M[k][n] stored row-major with rows = k.  x4.trans gives the B
// fragments of n-tiles n0 and n0+8 for k-tile k0..k0+15.
__device__ __forceinline__ uint32_t bt_frag2n_addr(uint32_t base, int stride, int k0, int n0, int lane)
{
    const int q = lane >> 3, r = lane & 7;
    return base + 2u * (uint32_t)((k0 + r + 8 * (q & 1)) * stride + n0 + 8 * (q >> 1));
}

// Transposed A: A[m][k] = M[k][m] stored row-major with rows = k (samples).  x4.trans gives
// the A fragment of m-tile m0..m0+15, k-tile k0..k0+15.
__device__ __forceinline__ uint32_t at_frag_addr(uint32_t base, int stride, int k0, int m0, int lane)
{
    const int q = lane >> 3, r = lane & 7;
    return base + 2u * (uint32_t)((k0 + r + 8 * (q >> 1)) * stride + m0 + 8 * (q & 1));
}

// ---------------------------------------------------------------------------------------
// Warp-level layer: acc[MT][NT] = A[MT][KT] * W, W stored [n][k] in shared memory.
// acc must be initialised by the caller (bias or zero).

template <int MT, int KT, int NT>
__device__ __forceinline__ void warp_gemm_w(float (&acc)[MT][NT][4], const uint32_t (&a)[MT][KT][4],
                                            uint32_t w_base, int w_stride, int lane)
{
    static_assert(KT % 2 == 0, "K must be a multiple of 32");
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int kp = 0; kp < KT / 2; ++kp) {
            uint32_t b[4];
            ldsm_x4(b, b_frag2k_addr(w_base, w_stride, nt * 8, kp * 32, lane));
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                mma16816(acc[mt][nt], a[mt][2 * kp], b[0], b[1]);
                mma16816(acc[mt][nt], a[mt][2 * kp + 1], b[2], b[3]);
            }
        }
    }
}

// acc[MT][NT] += A[MT][KT] * W^T where W is stored [k][n] = [out][in] rows (the forward
// weight matrix read transposed, for the backward dX = dY W^T).  NT must be even.
template <int MT, int KT, int NT>
__device__ __forceinline__ void warp_gemm_wt(float (&acc)[MT][NT][4], const uint32_t (&a)[MT][KT][4],
                                             uint32_t w_base, int w_stride, int lane)
{
    static_assert(NT % 2 == 0, "N must be a multiple of 16");
#pragma unroll
    for (int kt = 0; kt < KT; ++kt) {
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
            uint32_t b[4];
            ldsm_x4_t(b, bt_frag2n_addr(w_base, w_stride, kt * 16, np * 16, lane));
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                mma16816(acc[mt][2 * np], a[mt][kt], b[0], b[1]);
                mma16816(acc[mt][2 * np + 1], a[mt][kt], b[2], b[3]);
            }
        }
    }
}

// Load A fragments of a row-major shared matrix (rows r0.., MT m-tiles, KT k-tiles).
template <int MT, int KT>
__device__ __forceinline__ void load_a(uint32_t (&a)[MT][KT][4], uint32_t base, int stride, int r0,
                                       int lane)
{
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int kt = 0; kt < KT; ++kt) ldsm_x4(a[mt][kt], a_frag_addr(base, stride, r0 + mt * 16, kt * 16, lane));
}

// Accumulators (NT = 2 KT n8 tiles) -> fp16 A fragments, with optional ReLU.
template <int MT, int KT, bool RELU>
__device__ __forceinline__ void acc_to_a(uint32_t (&a)[MT][KT][4], const float (&acc)[MT][2 * KT][4])
{
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int kt = 0; kt < KT; ++kt) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                v[e] = acc[mt][2 * kt][e];
                v[4 + e] = acc[mt][2 * kt + 1][e];
            }
            if (RELU) {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = fmaxf(v[e], 0.f);
            }
            a[mt][kt][0] = pack_half2(v[0], v[1]);
            a[mt][kt][1] = pack_half2(v[2], v[3]);
            a[mt][kt][2] = pack_half2(v[4], v[5]);
            a[mt][kt][3] = pack_half2(v[6], v[7]);
        }
}

// Store A fragments back to a row-major shared matrix (rows r0..).
template <int MT, int KT>
__device__ __forceinline__ void store_a(const uint32_t (&a)[MT][KT][4], __half *base, int stride, int r0,
                                        int lane)
{
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int kt = 0; kt < KT; ++kt) {
            __half *p0 = base + (r0 + mt * 16 + g) * stride + kt * 16 + 2 * t;
            __half *p1 = p0 + 8 * stride;
            *reinterpret_cast<uint32_t *>(p0) = a[mt][kt][0];
            *reinterpret_cast<uint32_t *>(p1) = a[mt][kt][1];
            *reinterpret_cast<uint32_t *>(p0 + 8) = a[mt][kt][2];
            *reinterpret_cast<uint32_t *>(p1 + 8) = a[mt][kt][3];
        }
}

// Initialise accumulators with a per-column bias (fp32 in shared memory), or zero.
template <int MT, int NT>
__device__ __forceinline__ void acc_init_bias(float (&acc)[MT][NT][4], const float *bias, int lane)
{
    const int t = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const float b0 = bias ? bias[nt * 8 + 2 * t] : 0.f;
        const float b1 = bias ? bias[nt * 8 + 2 * t + 1] : 0.f;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            acc[mt][nt][0] = b0;
            acc[mt][nt][1] = b1;
            acc[mt][nt][2] = b0;
            acc[mt][nt][3] = b1;
        }
    }
}

}  // namespace nt

// nt_umma_selftest.cu -- self-test of the tcgen05 building blocks (nt_umma.cuh) on the
// operand layouts the fused kernels use: a K-major M=128 product (the forward layers) and
// an MN-major M=64 product whose operands are the same shared-memory activation tiles read
// transposed (the weight-gradient products).  Every wait is bounded; a timeout sets bit 0
// of *status and the kernel still releases its tensor memory.
#include <cuda_fp16.h>
#include <stdint.h>

#include "nt_capi.h"
#include "nt_kernels.cuh"
#include "nt_mma.cuh"
#include "nt_umma.cuh"

namespace nt {

// A [128][32], B [64][32], H [128][64] fp16 row-major (global).
// D1 [128][64] = A B^T; D2 [64][32] = H^T A (fp32).
__global__ void __launch_bounds__(128) umma_selftest_kernel(const __half *A, const __half *B, const __half *H, float *D1,
                                                            float *D2, int *status)
{
    __shared__ __align__(128) uint8_t sA[128 * 32 * 2];
    __shared__ __align__(128) uint8_t sB[64 * 32 * 2];
    __shared__ __align__(128) uint8_t sH[128 * 64 * 2];
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4 *>(sA + umma::cm_offset(tid, 8 * j, 4)) =
            *reinterpret_cast<const uint4 *>(A + tid * 32 + 8 * j);
    if (tid < 64)
        for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4 *>(sB + umma::cm_offset(tid, 8 * j, 4)) =
                *reinterpret_cast<const uint4 *>(B + tid * 32 + 8 * j);
    for (int j = 0; j < 8; ++j)
        *reinterpret_cast<uint4 *>(sH + umma::cm_offset(tid, 8 * j, 8)) =
            *reinterpret_cast<const uint4 *>(H + tid * 64 + 8 * j);

    const uint32_t bar_a = smem_addr(&bar);
    if (warp == 0) umma::alloc(smem_addr(&tmem_base), 128);
    if (tid == 0) {
        umma::mbar_init(bar_a, 1);
        umma::mbar_fence_init();
    }
    umma::fence_async_smem();
    umma::fence_before();
    __syncthreads();
    umma::fence_after();
    const uint32_t tbase = tmem_base;

    if (tid == 0) {
        const uint32_t a0 = smem_addr(sA), b0 = smem_addr(sB), h0 = smem_addr(sH);
        // D1 = A B^T: M = 128, N = 64, K = 32 (both operands K-major)
        const uint32_t id1 = umma::idesc_f16(128, 64, 0, 0);
        for (int ks = 0; ks < 2; ++ks)
            umma::mma_f16(tbase, umma::desc(a0 + ks * 256, 128, 512), umma::desc(b0 + ks * 256, 128, 512), id1,
                          ks > 0);
        // D2 = H^T A: M = 64 (features of H), N = 32 (features of A), K = 128 samples
        const uint32_t id2 = umma::idesc_f16(64, 32, 1, 1);
        for (int ks = 0; ks < 8; ++ks)
            umma::mma_f16(tbase + 64, umma::desc(h0 + ks * 2048, 1024, 128), umma::desc(a0 + ks * 1024, 512, 128), id2,
                          ks > 0);
        umma::commit(bar_a);
    }
    if (!umma::mbar_wait(bar_a, 0)) {
        atomicOr(status, 1);
        umma::mbar_wait(bar_a, 0);  // one more bounded wait for the MMAs in flight
    }
    umma::fence_after();
    const uint32_t lane_base = tbase + ((uint32_t)(32 * warp) << 16);
    for (int c0 = 0; c0 < 64; c0 += 16) {
        uint32_t r[16];
        umma::ld16(lane_base + c0, r);
        umma::wait_ld();
        for (int j = 0; j < 16; ++j) D1[(32 * warp + lane) * 64 + c0 + j] = __uint_as_float(r[j]);
    }
    for (int c0 = 0; c0 < 32; c0 += 16) {
        uint32_t r[16];
        umma::ld16(lane_base + 64 + c0, r);
        umma::wait_ld();
        if (lane < 16)
            for (int j = 0; j < 16; ++j) D2[(16 * warp + lane) * 32 + c0 + j] = __uint_as_float(r[j]);
    }
    umma::fence_before();
    __syncthreads();
    umma::fence_after();
    if (warp == 0) umma::dealloc(tbase, 128);
}

}  // namespace nt

extern "C" nt_status nt_umma_selftest(const void *a, const void *b, const void *h, float *d1, float *d2,
                                      int32_t *status, nt_stream_t stream)
{
    if (!a || !b || !h || !d1 || !d2 || !status) return NT_ERR_INVALID_ARG;
    nt::umma_selftest_kernel<<<1, 128, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const __half *>(a), reinterpret_cast<const __half *>(b), reinterpret_cast<const __half *>(h),
        d1, d2, reinterpret_cast<int *>(status));
    nt::count_launch();
    return cudaGetLastError() == cudaSuccess ? NT_OK : NT_ERR_CUDA;
}

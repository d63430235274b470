// nt_umma.cuh -- tcgen05 (5th-generation tensor core) building blocks for sm_100a: TMEM
// allocation, shared-memory matrix descriptors, MMA issue, commit to an mbarrier, bounded
// mbarrier waits and TMEM loads.
//
// Operand layout.  Every fp16 operand tile lives in shared memory as "core matrices" of
// 8 rows x 16 bytes (8 rows x 8 halves, 128 contiguous bytes), without swizzle:
//     byte(row, k) = (row / 8) * group_stride + (k / 8) * 128 + (row % 8) * 16 + (k % 8) * 2
// with group_stride = (K / 8) * 128.  Read K-major (rows = M or N, K along a row) the
// descriptor takes LBO = 128 (next 8 k) and SBO = group_stride (next 8 rows).  The same
// bytes read MN-major (M or N = the k dimension above, K = rows) take LBO = group_stride
// and SBO = 128.  So one activation tile stored [samples][features] feeds both the forward
// product (samples = M, features = K) and the weight-gradient product (features = M,
// samples = K) without a transpose.
//
// Accumulators (fp32) live in TMEM: for M = 128, row r is lane r; for M = 64 (cta_group::1)
// row r is lane (r % 16) + 32 * (r / 16).  Warp w of a warpgroup may only touch lanes
// 32 (w % 4) .. 32 (w % 4) + 31.
#pragma once

#include <stdint.h>

namespace nt {
namespace umma {

__host__ __device__ constexpr uint32_t cm_offset(int row, int k, int kchunks)
{
    return (uint32_t)((row >> 3) * (kchunks * 128) + (k >> 3) * 128 + (row & 7) * 16 + (k & 7) * 2);
}

// Shared-memory matrix descriptor, no swizzle (layout type 0), descriptor version 1.
__device__ __forceinline__ uint64_t desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes)
{
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// Instruction descriptor for kind::f16: A, B fp16, D fp32, M x N, K-major (0) or MN-major (1).
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int a_mn, int b_mn)
{
    return (1u << 4) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        :
        : "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

// Arrive (once) on the mbarrier when every previously issued tcgen05.mma of this thread completes.
__device__ __forceinline__ void commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Make this thread's generic-proxy shared-memory writes visible to the tensor core.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void alloc(uint32_t smem_dst, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_dst), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread t of the warp gets lane (taddr.lane + t).
__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void ld8(uint32_t taddr, uint32_t (&r)[8])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- mbarrier ---------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Bounded wait for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t max_tries = (1u << 22))
{
    for (uint32_t i = 0; i < max_tries; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}

}  // namespace umma
}  // namespace nt

// nt_adam.cu -- one fused Adam launch over any set of fp16 parameter buffers with fp32
// gradient / first / second moment buffers (MLP weights, biases and both latent grids).
//
// Restates AdamUpdateParameter (mavenkim2/neural_textures train.cu:521-543) with the
// buffer semantics of OptimizeParameterBuffer (train.cu:566-588): entries whose gradient is
// exactly zero are skipped (their moments do not decay) and every consumed gradient is
// zeroed.  The reference launches the network optimizer as a single warp (train.cu:985-988)
// and the latent optimizer as a second kernel; here one launch streams all segments with
// 16-byte vector accesses.  The float operations are written out with explicit rounding in
// the order of the reference expression so the result is bit-identical to the CPU oracle;
// the bias corrections 1 - beta^t are computed once per step on the host.
#include "nt_adam_math.cuh"
#include "nt_kernels.cuh"

namespace nt {

__device__ __forceinline__ float adam_one(float w, float g, float &m, float &v, const AdamSegment &s)
{
    return adam_update(w, g, m, v, s.lr, s.beta1, s.beta2, s.eps, s.bc1, s.bc2);
}

constexpr int kAdamThreads = 256;
constexpr int kAdamPerThread = 4;
static_assert(kAdamThreads * kAdamPerThread == kAdamChunk, "chunk size shared with the host");

// One chunk (kAdamThreads x kAdamPerThread consecutive entries of one segment).
__device__ __forceinline__ void adam_chunk(const AdamLaunch &p, int b)
{
    int si = 0;
#pragma unroll 1
    while (si + 1 < p.nseg && b >= p.seg[si + 1].first_block) ++si;
    const AdamSegment &s = p.seg[si];
    const int64_t i0 = ((int64_t)(b - s.first_block) * kAdamThreads + threadIdx.x) * kAdamPerThread;
    if (i0 >= s.n) return;
    if (s.w32) {  // fp32 parameters (AdamUpdateFloatParameter, train.cu:545-564)
        if (i0 + kAdamPerThread <= s.n && ((reinterpret_cast<uintptr_t>(s.w32) | reinterpret_cast<uintptr_t>(s.g) |
                                             reinterpret_cast<uintptr_t>(s.m) | reinterpret_cast<uintptr_t>(s.v)) &
                                            15) == 0) {
            const float4 g4 = *reinterpret_cast<const float4 *>(s.g + i0);
            float4 w4 = *reinterpret_cast<const float4 *>(s.w32 + i0);
            float4 m4 = *reinterpret_cast<const float4 *>(s.m + i0);
            float4 v4 = *reinterpret_cast<const float4 *>(s.v + i0);
            if (g4.x == 0.f && g4.y == 0.f && g4.z == 0.f && g4.w == 0.f) return;
            float *wv = &w4.x, *mv = &m4.x, *vv = &v4.x;
            const float gv[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (gv[e] != 0.f) wv[e] = adam_one(wv[e], gv[e], mv[e], vv[e], s);
            *reinterpret_cast<float4 *>(s.w32 + i0) = w4;
            *reinterpret_cast<float4 *>(s.m + i0) = m4;
            *reinterpret_cast<float4 *>(s.v + i0) = v4;
            *reinterpret_cast<float4 *>(s.g + i0) = make_float4(0.f, 0.f, 0.f, 0.f);
            return;
        }
        const int64_t end = i0 + kAdamPerThread < s.n ? i0 + kAdamPerThread : s.n;
        for (int64_t i = i0; i < end; ++i) {
            const float g = s.g[i];
            if (g == 0.f) continue;
            float m = s.m[i], v = s.v[i];
            s.w32[i] = adam_one(s.w32[i], g, m, v, s);
            s.m[i] = m;
            s.v[i] = v;
            s.g[i] = 0.f;
        }
        return;
    }
    const bool vec = i0 + kAdamPerThread <= s.n && ((reinterpret_cast<uintptr_t>(s.w) & 7) == 0) &&
                     ((reinterpret_cast<uintptr_t>(s.g) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(s.m) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(s.v) & 15) == 0);
    if (vec) {
        // all four streams are requested before any value is used (one memory round trip)
        const float4 g0 = *reinterpret_cast<const float4 *>(s.g + i0);
        uint2 wraw = *reinterpret_cast<const uint2 *>(s.w + i0);
        const float4 m0 = *reinterpret_cast<const float4 *>(s.m + i0);
        const float4 v0 = *reinterpret_cast<const float4 *>(s.v + i0);
        const float gv[4] = {g0.x, g0.y, g0.z, g0.w};
        if (gv[0] == 0.f && gv[1] == 0.f && gv[2] == 0.f && gv[3] == 0.f) return;  // nothing to update or zero
        float mv[4] = {m0.x, m0.y, m0.z, m0.w};
        float vv[4] = {v0.x, v0.y, v0.z, v0.w};
        __half *wh = reinterpret_cast<__half *>(&wraw);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (gv[e] == 0.f) continue;
            wh[e] = __float2half_rn(adam_one(__half2float(wh[e]), gv[e], mv[e], vv[e], s));
        }
        *reinterpret_cast<uint2 *>(s.w + i0) = wraw;
        *reinterpret_cast<float4 *>(s.m + i0) = make_float4(mv[0], mv[1], mv[2], mv[3]);
        *reinterpret_cast<float4 *>(s.v + i0) = make_float4(vv[0], vv[1], vv[2], vv[3]);
        *reinterpret_cast<float4 *>(s.g + i0) = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
        const int64_t end = i0 + kAdamPerThread < s.n ? i0 + kAdamPerThread : s.n;
        for (int64_t i = i0; i < end; ++i) {
            const float g = s.g[i];
            if (g == 0.f) continue;
            float m = s.m[i], v = s.v[i];
            s.w[i] = __float2half_rn(adam_one(__half2float(s.w[i]), g, m, v, s));
            s.m[i] = m;
            s.v[i] = v;
            s.g[i] = 0.f;
        }
    }
}

__global__ void __launch_bounds__(kAdamThreads) adam_kernel(const AdamLaunch p) { adam_chunk(p, blockIdx.x); }

cudaError_t launch_adam(const AdamLaunch &p, cudaStream_t stream)
{
    if (p.total_blocks <= 0) return cudaSuccess;
    adam_kernel<<<p.total_blocks, kAdamThreads, 0, stream>>>(p);
    count_launch();
    return cudaGetLastError();
}

}  // namespace nt

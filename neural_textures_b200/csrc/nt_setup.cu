// nt_setup.cu -- seeded set-up kernels: synthetic target, latent initialisation, L2 flush.
//
// Not part of the reference (it loads EXR textures and initialises on the host,
// main.cpp:182-214, :436-556); the BASELINE configurations use synthetic materials.  The
// target generator follows the integer parameter derivation of the CPU oracle exactly
// (same hash, integer frequencies, integer phase reduction); only the final sine /
// exponential differ in rounding, below fp16 resolution in almost every texel.
#include <algorithm>
#include <cuda_fp16.h>
#include <stdint.h>

#include "nt_capi.h"
#include "nt_kernels.cuh"

namespace nt {

__host__ __device__ __forceinline__ uint32_t hash32(uint32_t x)
{
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

__device__ __forceinline__ uint32_t isqrt32(uint32_t n)
{
    uint32_t r = 0;
    while ((r + 1) * (r + 1) <= n) ++r;
    return r;
}

struct Sinusoid {
    int32_t fu, fv;
    float phase, amp;
};

__device__ void target_params(uint32_t seed, int32_t channel, int32_t k, Sinusoid &o)
{
    const uint32_t base = hash32(seed * 0x9E3779B9u ^ hash32((uint32_t)(channel * 64 + k + 1)));
    const uint32_t f = 1u + hash32(base ^ 0x1u) % 64u;
    const int32_t a = (int32_t)(hash32(base ^ 0x2u) % (2u * f + 1u)) - (int32_t)f;
    int32_t b = (int32_t)isqrt32(f * f - (uint32_t)(a * a));
    if (hash32(base ^ 0x3u) & 1u) b = -b;
    o.fu = a;
    o.fv = b;
    if (a == 0 && b == 0) o.fu = 1;
    o.phase = (float)(hash32(base ^ 0x4u) >> 8) * (1.0f / 16777216.0f);
    o.amp = 0.25f + 0.5f * ((float)(hash32(base ^ 0x5u) >> 8) * (1.0f / 16777216.0f));
}

__device__ __forceinline__ float frac_cycles(int32_t f, int32_t x, int32_t n)
{
    const int64_t den = 2 * (int64_t)n;
    int64_t num = ((int64_t)f * (2 * (int64_t)x + 1)) % den;
    if (num < 0) num += den;
    return (float)((double)num / (double)den);
}

__global__ void target_kernel(__half *out, int32_t w, int32_t h, int32_t channels, uint32_t seed,
                              int32_t pbr)
{
    __shared__ Sinusoid tab[16 * 16];
    for (int i = threadIdx.x; i < channels * 16; i += blockDim.x) target_params(seed, i / 16, i % 16, tab[i]);
    __syncthreads();
    const int64_t n = (int64_t)w * h;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int32_t x = (int32_t)(i % w), y = (int32_t)(i / w);
        for (int c = 0; c < channels; ++c) {
            float s = 0.f, du = 0.f, dv = 0.f;
            for (int k = 0; k < 16; ++k) {
                const Sinusoid &q = tab[c * 16 + k];
                float t = frac_cycles(q.fu, x, w) + frac_cycles(q.fv, y, h) + q.phase;
                t -= floorf(t);
                float sn, cs;
                sincospif(2.f * t, &sn, &cs);
                s = fmaf(q.amp, sn, s);
                const float dc = q.amp * 6.28318530717958647692f * cs;
                du = fmaf(dc, (float)q.fu, du);
                dv = fmaf(dc, (float)q.fv, dv);
            }
            const float hv = 1.f / (1.f + expf(-s));
            out[i * channels + c] = __float2half_rn(hv);
            if (pbr && channels == 12 && c == 9) {
                const float gg = hv * (1.f - hv) / 64.f;
                float nx = -gg * du, ny = -gg * dv, nz = 1.f;
                const float inv = rsqrtf(nx * nx + ny * ny + nz * nz);
                out[i * channels + 3] = __float2half_rn(nx * inv * 0.5f + 0.5f);
                out[i * channels + 4] = __float2half_rn(ny * inv * 0.5f + 0.5f);
                out[i * channels + 5] = __float2half_rn(nz * inv * 0.5f + 0.5f);
            }
        }
    }
}

__global__ void init_latents_kernel(__half *grid, int64_t count, uint32_t seed)
{
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t hsh = hash32(seed * 0x9E3779B9u ^ hash32((uint32_t)i ^ (uint32_t)(i >> 32) * 0x85ebca6bu));
        const float u01 = (float)(hsh >> 8) * (1.0f / 16777216.0f);
        grid[i] = __float2half_rn(2.f * u01 - 1.f);
    }
}

__global__ void flush_kernel(uint4 *p, int64_t n16, uint32_t val)
{
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
        p[i] = make_uint4(val, val, val, val);
}

// One level of a mip chain from the level below: 2x2 box average in fp32 ((a + b) + (c + d)) / 4,
// source texels clamped to the level below (odd sizes drop the last row / column), rounded to
// fp16.  One thread per (texel, channel).
__global__ void build_mip_kernel(const __half *__restrict__ src, int sw, int sh, __half *__restrict__ dst, int dw,
                                 int dh, int c)
{
    const int64_t n = (int64_t)dw * dh * c;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int k = (int)(i % c);
        const int64_t texel = i / c;
        const int x = (int)(texel % dw), y = (int)(texel / dw);
        const int x0 = min(2 * x, sw - 1), x1 = min(2 * x + 1, sw - 1);
        const int y0 = min(2 * y, sh - 1), y1 = min(2 * y + 1, sh - 1);
        const float a = __half2float(src[((int64_t)y0 * sw + x0) * c + k]);
        const float b = __half2float(src[((int64_t)y0 * sw + x1) * c + k]);
        const float d = __half2float(src[((int64_t)y1 * sw + x0) * c + k]);
        const float e = __half2float(src[((int64_t)y1 * sw + x1) * c + k]);
        dst[i] = __float2half_rn(__fmul_rn(__fadd_rn(__fadd_rn(a, b), __fadd_rn(d, e)), 0.25f));
    }
}

cudaError_t launch_build_mips(__half *chain, int32_t w, int32_t h, int32_t c, int32_t num_mips, cudaStream_t st)
{
    int64_t off = 0;
    for (int m = 1; m < num_mips; ++m) {
        const int sw = max(w >> (m - 1), 1), sh = max(h >> (m - 1), 1);
        const int dw = max(w >> m, 1), dh = max(h >> m, 1);
        __half *src = chain + off * c;
        off += (int64_t)sw * sh;
        const int64_t n = (int64_t)dw * dh * c;
        const int blocks = (int)std::min<int64_t>((n + 255) / 256, 4 * sm_count());
        build_mip_kernel<<<blocks, 256, 0, st>>>(src, sw, sh, chain + off * c, dw, dh, c);
        count_launch();
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_target(void *out, int32_t w, int32_t h, int32_t c, uint32_t seed, int32_t pbr,
                          cudaStream_t st)
{
    target_kernel<<<4 * sm_count(), 256, 0, st>>>(reinterpret_cast<__half *>(out), w, h, c, seed, pbr);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_init_latents(void *grid, int64_t count, uint32_t seed, cudaStream_t st)
{
    init_latents_kernel<<<4 * sm_count(), 256, 0, st>>>(reinterpret_cast<__half *>(grid), count, seed);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_flush(void *scratch, size_t bytes, cudaStream_t st)
{
    static uint32_t counter = 0;
    flush_kernel<<<4 * sm_count(), 512, 0, st>>>(reinterpret_cast<uint4 *>(scratch), (int64_t)(bytes / 16), ++counter);
    count_launch();
    return cudaGetLastError();
}

}  // namespace nt

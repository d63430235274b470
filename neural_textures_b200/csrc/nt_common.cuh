// nt_common.cuh -- device helpers shared by the decode, training, Adam and codec kernels.
//
// Sampling conventions restate mavenkim2/neural_textures:
//   texel centre uv * size - 0.5, floor, fraction ........ train.cu:288-291
//   wrap addressing ...................................... train.cu:65-69
//   Catmull-Rom weights (a = -0.5) ....................... filter/catmull_rom.h:56-59
//   per-sample xorshift32 RNG and seed ................... train.cu:37-58, :833
//   jittered sample per lattice cell, clamped ............ train.cu:827-844
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "nt_capi.h"

namespace nt {

constexpr int kNumSms = 148;  // B200; the host reads the real count at run time

// ---------------------------------------------------------------------------------------
// fp16 packing

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi)
{
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ float2 unpack_half2(uint32_t v)
{
    __half2 h = *reinterpret_cast<__half2 *>(&v);
    return __half22float2(h);
}

__device__ __forceinline__ float round_half(float f) { return __half2float(__float2half_rn(f)); }

// ---------------------------------------------------------------------------------------
// RNG (train.cu:37-58).  seed 0 reproduces the reference's per-sample seeds exactly.

__device__ __forceinline__ uint32_t rng_seed(uint32_t sample_index, uint32_t step, uint32_t seed)
{
    uint32_t s = sample_index ^ (step * 747796405u + 2891336453u) ^ (seed * 0x9E3779B9u);
    return s ? s : 1u;
}

__device__ __forceinline__ uint32_t rng_next(uint32_t &x)
{
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    return x;
}

__device__ __forceinline__ float rng_uniform(uint32_t &x)
{
    return (float)(rng_next(x) & 0x00FFFFFFu) * (1.0f / 16777216.0f);
}

// ---------------------------------------------------------------------------------------
// Sample placement.  Every operation is explicitly rounded (no contraction) so the
// positions, and therefore the floor() decisions of the filter, are bit-identical to the
// CPU oracle.

struct SamplerView {
    int32_t image_w, image_h;
    int32_t lattice_w, lattice_h;
    float stride_x, stride_y;
    int32_t offset_x, offset_y;
    uint32_t step, seed;
};

__device__ __forceinline__ float clampf(float x, float lo, float hi)
{
    return x < lo ? lo : (x > hi ? hi : x);
}

// a / n correctly rounded, for a size n >= 1 (the IEEE division of the reference's float
// expressions): a power of two divides exactly as the product with 2^-k, which costs one
// multiply instead of a division sequence; other sizes take the IEEE division.
__device__ __forceinline__ float div_by_size(float a, int32_t n)
{
    if ((n & (n - 1)) == 0) return __fmul_rn(a, __int_as_float((127 - (31 - __clz(n))) << 23));
    return __fdiv_rn(a, (float)n);
}

__device__ __forceinline__ void sample_uv(const SamplerView &s, int32_t ix, int32_t iy, float &u,
                                          float &v)
{
    const uint32_t index = (uint32_t)iy * (uint32_t)s.lattice_w + (uint32_t)ix;
    uint32_t st = rng_seed(index, s.step, s.seed);
    const float jx = __fsub_rn(rng_uniform(st), 0.5f);
    const float jy = __fsub_rn(rng_uniform(st), 0.5f);
    const float tx = __fadd_rn(__fadd_rn((float)ix, 0.5f), jx);
    const float ty = __fadd_rn(__fadd_rn((float)iy, 0.5f), jy);
    float px = __fadd_rn(__fmul_rn(tx, s.stride_x), (float)s.offset_x);
    float py = __fadd_rn(__fmul_rn(ty, s.stride_y), (float)s.offset_y);
    px = clampf(px, 0.5f, __fsub_rn((float)s.image_w, 0.5f));
    py = clampf(py, 0.5f, __fsub_rn((float)s.image_h, 0.5f));
    u = div_by_size(px, s.image_w);
    v = div_by_size(py, s.image_h);
}

// Decode texel centres (train.cu:926-933).
__device__ __forceinline__ void texel_uv(int32_t x, int32_t y, int32_t w, int32_t h, float &u,
                                         float &v)
{
    u = div_by_size(__fadd_rn((float)x, 0.5f), w);
    v = div_by_size(__fadd_rn((float)y, 0.5f), h);
}

// ---------------------------------------------------------------------------------------
// Catmull-Rom footprint

// Wrap c into [0, n).  The filter taps and footprint windows stay within one period of the
// grid, so one conditional correction in each direction is the common path; the modulo
// only runs for coordinates further out.
__device__ __forceinline__ int32_t wrap_coord(int32_t c, int32_t n)
{
    int32_t r = c < 0 ? c + n : c;
    r = r >= n ? r - n : r;
    if ((uint32_t)r >= (uint32_t)n) {
        r = c % n;
        r = r < 0 ? r + n : r;
    }
    return r;
}

__device__ __forceinline__ void catmull_rom_weights(float f, float w[4])
{
    w[0] = f * (f * (f * -0.5f + 1.0f) - 0.5f);
    w[1] = f * f * (f * 1.5f - 2.5f) + 1.0f;
    w[2] = f * (f * (f * -1.5f + 2.0f) + 0.5f);
    w[3] = f * f * (f * 0.5f - 0.5f);
}

// The 4x4 footprint of one sample in one grid: base tap (the [1, 1] texel, unwrapped),
// wrapped texel columns / rows and weights.
struct Footprint {
    int32_t bx, by;
    int32_t xs[4];
    int32_t ys[4];
    float wx[4];
    float wy[4];
};

// filter/catmull_rom.h:46-52: samplePos = uv * size; texPos1 = floor(samplePos - 0.5) + 0.5;
// f = samplePos - texPos1 (explicitly rounded, so the fraction is bit-identical to the
// reference's).  Returns the index of the [1, 1] tap.
__device__ __forceinline__ int32_t cr_base(float uv, int32_t size, float &f)
{
    const float sp = __fmul_rn(uv, (float)size);
    const float fl = floorf(__fsub_rn(sp, 0.5f));
    f = __fsub_rn(sp, __fadd_rn(fl, 0.5f));
    return (int32_t)fl;
}

__device__ __forceinline__ void footprint(float u, float v, int32_t w, int32_t h, Footprint &fp)
{
    float fx, fy;
    const int32_t bx = cr_base(u, w, fx), by = cr_base(v, h, fy);
    fp.bx = bx;
    fp.by = by;
    catmull_rom_weights(fx, fp.wx);
    catmull_rom_weights(fy, fp.wy);
    // bx - 1 >= -1 and bx + 2 <= w + 1 for uv in [0, 1]; one conditional wrap suffices when
    // w >= 2, and wrap_coord handles everything else.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        fp.xs[i] = wrap_coord(bx - 1 + i, w);
        fp.ys[i] = wrap_coord(by - 1 + i, h);
    }
}

// Fire-and-forget vector reduction into global memory (red.global.add.v4.f32, sm_90+): the
// four floats are added atomically per element, like atomicAdd on each, and the thread does
// not wait for the old value.  addr must be 16-byte aligned.
__device__ __forceinline__ void red_add_v4(float *addr, float a, float b, float c, float d)
{
    asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c),
                 "f"(d)
                 : "memory");
}

// Packed fp32 fused multiply-add (sm_100 fma.rn.f32x2): per lane exactly fmaf(a, b, c).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c)
{
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(r)
        : "l"(*reinterpret_cast<unsigned long long *>(&a)), "l"(*reinterpret_cast<unsigned long long *>(&b)),
          "l"(*reinterpret_cast<unsigned long long *>(&c)));
    return *reinterpret_cast<float2 *>(&r);
}

// Catmull-Rom gather of C channels (C = 4, 8, 12 or 16; channel-interleaved fp16 grid),
// fp32 accumulation: row sums first, then the weighted sum of rows (same order as the
// oracle).  Channel pairs go through the packed fp32 FMA, which rounds each lane like fmaf.
// The loads of RB footprint rows are issued before their arithmetic, so that the gather pays
// the memory latency once per RB rows instead of once per tap (RB = 4 for up to 8 channels:
// 64 registers of texels; two rows above).
template <int C>
__device__ __forceinline__ void gather_cr(const __half *__restrict__ grid, int32_t w,
                                          const Footprint &fp, float out[C])
{
    static_assert(C % 4 == 0, "channel count must be a multiple of 4");
    constexpr int Q = C / 4;          // 8-byte groups of 4 channels per texel
    constexpr int RB = C <= 8 ? 4 : 2;  // rows per load batch
    float2 acc[C / 2];
#pragma unroll
    for (int k = 0; k < C / 2; ++k) acc[k] = make_float2(0.f, 0.f);
#pragma unroll
    for (int j0 = 0; j0 < 4; j0 += RB) {
        uint2 raw[RB][4][Q];
#pragma unroll
        for (int jj = 0; jj < RB; ++jj) {
            const __half *rp = grid + (size_t)fp.ys[j0 + jj] * (size_t)w * C;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const __half *tp = rp + (size_t)fp.xs[i] * C;
                if constexpr (C % 8 == 0) {
#pragma unroll
                    for (int q = 0; q < Q / 2; ++q) {
                        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(tp) + q);
                        raw[jj][i][2 * q] = make_uint2(v.x, v.y);
                        raw[jj][i][2 * q + 1] = make_uint2(v.z, v.w);
                    }
                } else {
#pragma unroll
                    for (int q = 0; q < Q; ++q) raw[jj][i][q] = __ldg(reinterpret_cast<const uint2 *>(tp) + q);
                }
            }
        }
#pragma unroll
        for (int jj = 0; jj < RB; ++jj) {
            float2 row[C / 2];
#pragma unroll
            for (int k = 0; k < C / 2; ++k) row[k] = make_float2(0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 wx2 = make_float2(fp.wx[i], fp.wx[i]);
#pragma unroll
                for (int q = 0; q < Q; ++q) {
                    row[2 * q] = ffma2(wx2, unpack_half2(raw[jj][i][q].x), row[2 * q]);
                    row[2 * q + 1] = ffma2(wx2, unpack_half2(raw[jj][i][q].y), row[2 * q + 1]);
                }
            }
            const float2 wy2 = make_float2(fp.wy[j0 + jj], fp.wy[j0 + jj]);
#pragma unroll
            for (int k = 0; k < C / 2; ++k) acc[k] = ffma2(wy2, row[k], acc[k]);
        }
    }
#pragma unroll
    for (int k = 0; k < C / 2; ++k) {
        out[2 * k] = acc[k].x;
        out[2 * k + 1] = acc[k].y;
    }
}

// Runtime-channel Catmull-Rom gather (targets with any channel count <= 16).
__device__ __forceinline__ void gather_cr_any(const __half *__restrict__ grid, int32_t w, int32_t c,
                                              const Footprint &fp, float out[16])
{
#pragma unroll
    for (int k = 0; k < 16; ++k) out[k] = 0.f;
    for (int j = 0; j < 4; ++j) {
        float row[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) row[k] = 0.f;
        const __half *rp = grid + (size_t)fp.ys[j] * (size_t)w * c;
        for (int i = 0; i < 4; ++i) {
            const __half *tp = rp + (size_t)fp.xs[i] * c;
#pragma unroll
            for (int k = 0; k < 16; ++k)
                if (k < c) row[k] = fmaf(fp.wx[i], __half2float(tp[k]), row[k]);
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) out[k] = fmaf(fp.wy[j], row[k], out[k]);
    }
}

// Target gather with vector loads for the common channel counts (4, 8, 12, 16).
__device__ __forceinline__ void gather_target(const __half *__restrict__ t, int32_t w, int32_t c,
                                              const Footprint &fp, float out[16])
{
#pragma unroll
    for (int k = 0; k < 16; ++k) out[k] = 0.f;
    if (c == 8) {
        gather_cr<8>(t, w, fp, out);
    } else if (c == 12) {
        gather_cr<12>(t, w, fp, out);
    } else if (c == 16) {
        gather_cr<16>(t, w, fp, out);
    } else if (c == 4) {
        gather_cr<4>(t, w, fp, out);
    } else {
        gather_cr_any(t, w, c, fp, out);
    }
}

// Positional features [sin 2pi u, cos 2pi u, sin 2pi v, cos 2pi v, sin 4pi u, ...].
__device__ __forceinline__ void posenc(float u, float v, float out[8])
{
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const float m = (float)(2 << k);
        sincospif(m * u, &out[4 * k + 0], &out[4 * k + 1]);
        sincospif(m * v, &out[4 * k + 2], &out[4 * k + 3]);
    }
}

// Launch counter (host-visible through nt_launch_count).
void count_launch();

}  // namespace nt

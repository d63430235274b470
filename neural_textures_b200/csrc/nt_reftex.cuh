// nt_reftex.cuh -- reference-texture targets on the texture units (mavenkim2/neural_textures
// train.h:69-77 ReferenceTexture, train.cu:78-103 SampleReferenceTextureTrilinear, :105-157
// InitializeExpectedValues, filter/catmull_rom.h:39-89 SampleTextureCatmullRomLod).
//
// A level is filtered with Catmull-Rom from 9 hardware bilinear fetches (the published
// "bicubic filtering in fewer taps" method): on each axis the middle two of the 4 taps merge
// into one fetch placed between them at w2 / (w1 + w2), weighted w1 + w2.  The two levels of a
// fractional mip coordinate are blended (1 - t, t).
#pragma once

#include <cuda_runtime.h>

#include "nt_common.cuh"

namespace nt {

constexpr int kMaxRefTextures = NT_MAX_REFERENCE_TEXTURES;

struct RefTexView {
    cudaTextureObject_t tex;  // 0: skipped
    int32_t w, h;             // level 0
    int32_t ch;               // 1 .. 4
    int32_t mips;
};

// One bilinear fetch at normalized (x, y) of level `level`; channels past ch are 0.
__device__ __forceinline__ float4 ref_fetch(const RefTexView &r, float x, float y, float level)
{
    if (r.ch == 1) return make_float4(tex2DLod<float>(r.tex, x, y, level), 0.f, 0.f, 0.f);
    if (r.ch == 2) {
        const float2 s = tex2DLod<float2>(r.tex, x, y, level);
        return make_float4(s.x, s.y, 0.f, 0.f);
    }
    const float4 s = tex2DLod<float4>(r.tex, x, y, level);
    return make_float4(s.x, s.y, s.z, r.ch == 3 ? 0.f : s.w);
}

// One axis of the 9-fetch Catmull-Rom: weights of the 3 fetches and their normalized positions
// (catmull_rom.h:46-78: base texel centre floor(p - 0.5) + 0.5, fraction, weights, merged
// middle tap).
__device__ __forceinline__ void ref_axis(float uv, float size, float (&w)[3], float (&pos)[3])
{
    const float sp = uv * size;
    const float t1 = floorf(sp - 0.5f) + 0.5f;
    const float f = sp - t1;
    float cr[4];
    catmull_rom_weights(f, cr);
    const float w12 = cr[1] + cr[2];
    w[0] = cr[0];
    w[1] = w12;
    w[2] = cr[3];
    pos[0] = (t1 - 1.f) / size;
    pos[1] = (t1 + cr[2] / w12) / size;
    pos[2] = (t1 + 2.f) / size;
}

// Catmull-Rom sample of one level (the fetches in the reference's order: rows of y).
__device__ __forceinline__ float4 ref_catmull_rom(const RefTexView &r, float u, float v, int level)
{
    const float W = (float)max(r.w >> level, 1), H = (float)max(r.h >> level, 1);
    float wx[3], wy[3], px[3], py[3];
    ref_axis(u, W, wx, px);
    ref_axis(v, H, wy, py);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
        for (int i = 0; i < 3; ++i) {
            const float4 s = ref_fetch(r, px[i], py[j], (float)level);
            const float k = wx[i] * wy[j];
            acc.x += s.x * k;
            acc.y += s.y * k;
            acc.z += s.z * k;
            acc.w += s.w * k;
        }
    return acc;
}

// train.cu:78-103: levels floor(lod) and the next one of the texture's chain, blended.
__device__ __forceinline__ float4 ref_trilinear(const RefTexView &r, float u, float v, float lod)
{
    const int last = r.mips > 0 ? r.mips - 1 : 0;
    float mc = lod > 0.f ? lod : 0.f;  // NaN -> 0
    mc = mc < (float)last ? mc : (float)last;
    const int m0 = min((int)floorf(mc), last), m1 = min(m0 + 1, last);
    const float t = m1 > m0 ? mc - (float)m0 : 0.f;
    const float4 s0 = ref_catmull_rom(r, u, v, m0);
    if (m1 == m0) return s0;
    const float4 s1 = ref_catmull_rom(r, u, v, m1);
    const float a = 1.f - t;
    return make_float4(s0.x * a + s1.x * t, s0.y * a + s1.y * t, s0.z * a + s1.z * t, s0.w * a + s1.w * t);
}

// train.cu:105-157: the textures' channels in order fill the expected outputs.
__device__ __forceinline__ void ref_expected(const RefTexView *ref, int n, float u, float v, float lod,
                                             float (&out)[16])
{
#pragma unroll
    for (int k = 0; k < 16; ++k) out[k] = 0.f;
    int oc = 0;
    for (int t = 0; t < n && oc < 16; ++t) {
        const RefTexView &r = ref[t];
        if (!r.tex || r.ch <= 0) continue;
        const float4 s = ref_trilinear(r, u, v, lod);
        const float c4[4] = {s.x, s.y, s.z, s.w};
        for (int c = 0; c < min(r.ch, 4) && oc < 16; ++c) {
#pragma unroll
            for (int k = 0; k < 16; ++k)
                if (k == oc) out[k] = c4[c];
            ++oc;
        }
    }
}

}  // namespace nt

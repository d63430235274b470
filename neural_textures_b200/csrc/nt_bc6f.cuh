// nt_bc6f.cuh -- BC6 block features: latents stored as per-block float BC6 parameters and
// decoded differentiably (mavenkim2/neural_textures train.cu:161-182 UnquantizeEndpoints /
// DecompressBC6, :204-212 block and pixel indices, :240-261 SampleBC6FeatureTexel, and the
// backward of :436-454).
//
// A grid of C channels in block form holds, per 4x4 block (row-major, width / 4 per row),
// ceil(C / 3) channel triples of 32 floats: endpoints e0..e3 (xyz, 12 floats), 16 pixel
// indices, partition (int32 bits), mode (int32 bits, 0..9), 2 unused.  Gradients and Adam
// moments use the same layout; the partition and mode slots never receive a gradient, so
// Adam's zero-gradient skip leaves them untouched.  The float operations are written out with
// explicit rounding in the reference's order (no contraction), as in the CPU oracle.
#pragma once

#include "nt_common.cuh"

namespace nt {

constexpr int kBc6fFloats = NT_BC6F_RECORD_FLOATS;

__device__ const uint16_t c_bc6f_parts[32] = {  // train.cu:20-29
    0xCCCC, 0x8888, 0xEEEE, 0xECC8, 0xC880, 0xFEEC, 0xFEC8, 0xEC80, 0xC800, 0xFFEC, 0xFE80,
    0xE800, 0xFFE8, 0xFF00, 0xFFF0, 0xF000, 0xF710, 0x008E, 0x7100, 0x08CE, 0x008C, 0x7310,
    0x3100, 0x8CCE, 0x088C, 0x3110, 0x6666, 0x366C, 0x17E8, 0x0FF0, 0x718E, 0x399C};

__device__ __forceinline__ int bc6f_mode_bits(int mode)  // train.cu:31-34
{
    constexpr uint64_t packed = 10ull | 7ull << 4 | 11ull << 8 | 11ull << 12 | 11ull << 16 | 9ull << 20 |
                                8ull << 24 | 8ull << 28 | 8ull << 32 | 6ull << 36;
    const int m = (unsigned)mode > 9u ? 0 : mode;
    return (int)((packed >> (4 * m)) & 15u);
}

// x * 2^n.  While 2^n is a normal float (every scale a record's decode produces) this is one
// correctly rounded product of the exact value x 2^n, i.e. ldexpf(x, n); other n take ldexpf.
__device__ __forceinline__ float scale2(float x, int n)
{
    if ((unsigned)(n + 126) <= 253u) return __fmul_rn(x, __int_as_float((n + 127) << 23));
    return ldexpf(x, n);
}

// train.cu:161-167
__device__ __forceinline__ float bc6f_unquantize(float e, int b)
{
    const float scale = (31.f / 64.f) * 65536.f;
    return scale2(__fadd_rn(__fmul_rn(scale, e), 32768.f), -b);
}

// train.cu:169-182 per channel, with the intermediates of train.cu:184-202
struct Bc6fChannel {
    float w, eb0, eb1, y;
    int hy;
};

__device__ __forceinline__ Bc6fChannel bc6f_channel(float e0, float e1, int b, float x)
{
    Bc6fChannel r;
    r.eb0 = bc6f_unquantize(e0, b);
    r.eb1 = bc6f_unquantize(e1, b);
    // v / 1024 == v * 2^-10 exactly (both round the same real number)
    r.y = __fadd_rn(r.eb0, __fmul_rn(__fmul_rn(__fsub_rn(r.eb1, r.eb0), 8.f), x));
    const float hyf = fmaxf(__fsub_rn(floorf(__fmul_rn(__fsub_rn(r.y, 1.f), 0x1p-10f)), 1.f), 0.f);
    r.hy = (int)hyf;
    r.w = scale2(__fsub_rn(__fmul_rn(r.y, 0x1p-10f), (float)r.hy), r.hy - 14);
    return r;
}

// Record of triple t of the block holding texel (x, y).
__device__ __forceinline__ int64_t bc6f_record(int w, int T, int x, int y, int t)
{
    return (((int64_t)(y >> 2) * (w >> 2) + (x >> 2)) * T + t) * kBc6fFloats;
}

// Channels 3t .. 3t + 2 of texel (x, y) (train.cu:240-261): triple t of a grid with T triples.
__device__ __forceinline__ void bc6f_texel_triple(const float *__restrict__ blocks, int w, int T, int x, int y, int t,
                                                  float (&out)[3])
{
    const int pix = ((y & 3) << 2) + (x & 3);
    const float *p = blocks + bc6f_record(w, T, x, y, t);
    const int part = __float_as_int(__ldg(p + 28)) & 31, mode = __float_as_int(__ldg(p + 29));
    const int r = (c_bc6f_parts[part] >> pix) & 1;
    const int bits = bc6f_mode_bits(mode);
    const float xv = __ldg(p + 12 + pix);
#pragma unroll
    for (int c = 0; c < 3; ++c) out[c] = bc6f_channel(__ldg(p + 6 * r + c), __ldg(p + 6 * r + 3 + c), bits, xv).w;
}

// The C channels of texel (x, y).
template <int C>
__device__ __forceinline__ void bc6f_texel(const float *__restrict__ blocks, int w, int x, int y, float (&out)[C])
{
    constexpr int T = (C + 2) / 3;
#pragma unroll
    for (int t = 0; t < T; ++t) {
        float v[3];
        bc6f_texel_triple(blocks, w, T, x, y, t, v);
#pragma unroll
        for (int c = 0; c < 3; ++c)
            if (3 * t + c < C) out[3 * t + c] = v[c];
    }
}

// Catmull-Rom gather of a block-feature grid: gather_cr's footprint and order (row sums,
// then the weighted sum of rows) over decoded texels.
template <int C>
__device__ __forceinline__ void gather_bc6f(const float *__restrict__ blocks, int w, const Footprint &fp, float out[C])
{
#pragma unroll
    for (int k = 0; k < C; ++k) out[k] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float row[C];
#pragma unroll
        for (int k = 0; k < C; ++k) row[k] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float v[C];
            bc6f_texel<C>(blocks, w, fp.xs[i], fp.ys[j], v);
#pragma unroll
            for (int k = 0; k < C; ++k) row[k] = fmaf(fp.wx[i], v[k], row[k]);
        }
#pragma unroll
        for (int k = 0; k < C; ++k) out[k] = fmaf(fp.wy[j], row[k], out[k]);
    }
}

// Backward of one texel (train.cu:436-454) for the feature gradient fg (C channels, tap
// weight and 1 / num_samples applied): adds to the endpoints of its region and its pixel
// index.
template <int C>
__device__ __forceinline__ void bc6f_backward_texel(const float *__restrict__ blocks, float *grads, int w, int x,
                                                    int y, const float (&fg)[C])
{
    constexpr int T = (C + 2) / 3;
    const int pix = ((y & 3) << 2) + (x & 3);
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const int64_t rec = bc6f_record(w, T, x, y, t);
        const float *p = blocks + rec;
        float *gp = grads + rec;
        const int part = __float_as_int(__ldg(p + 28)) & 31, mode = __float_as_int(__ldg(p + 29));
        const int r = (c_bc6f_parts[part] >> pix) & 1;
        const int bits = bc6f_mode_bits(mode);
        const float xv = __ldg(p + 12 + pix);
        const float alpha = __fmul_rn(xv, 8.f);
        const float deibar_dei = scale2(31.f / 64, 16 - bits);
        float dl_dx = 0.f;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            if (3 * t + c >= C) break;
            const Bc6fChannel ch = bc6f_channel(__ldg(p + 6 * r + c), __ldg(p + 6 * r + 3 + c), bits, xv);
            const float dl_dy = scale2(fg[3 * t + c], ch.hy - 24);
            dl_dx = __fadd_rn(dl_dx, __fmul_rn(dl_dy, __fmul_rn(__fsub_rn(ch.eb1, ch.eb0), 8.f)));
            atomicAdd(gp + 6 * r + c, __fmul_rn(__fmul_rn(__fsub_rn(1.f, alpha), deibar_dei), dl_dy));
            atomicAdd(gp + 6 * r + 3 + c, __fmul_rn(__fmul_rn(alpha, deibar_dei), dl_dy));
        }
        atomicAdd(gp + 12 + pix, dl_dx);
    }
}

}  // namespace nt

/*
 * nt_oracle.c -- CPU restatement of the reference's neural-texture hot path.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline); never part of the
 * product.  Build: see oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off).
 *
 * Reference: mavenkim2/neural_textures.  Citations are file:line in that project.
 */
#define _GNU_SOURCE
#include "nt_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------------------ */
/* fp16                                                                                  */
/* ------------------------------------------------------------------------------------ */

uint16_t nto_f2h(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    const uint32_t e = ax >> 23;
    if (e >= 113) { /* normal half range or overflow */
        if (e > 142) return (uint16_t)(sign | 0x7c00u);
        uint32_t h = ((e - 112) << 10) | ((ax & 0x7fffffu) >> 13);
        const uint32_t rem = ax & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++; /* may carry into inf */
        return (uint16_t)(sign | h);
    }
    /* half subnormal: value / 2^-24 = M * 2^(e - 126) */
    const uint32_t s = 126 - e;
    if (s > 25) return (uint16_t)sign;
    const uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
    uint32_t h = mant >> s;
    const uint32_t rem = mant & ((1u << s) - 1u);
    const uint32_t half = 1u << (s - 1);
    if (rem > half || (rem == half && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

float nto_h2f(uint16_t h)
{
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    const uint32_t m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else { /* subnormal: m * 2^-24 */
            float v = (float)m * 5.9604644775390625e-8f;
            memcpy(&x, &v, 4);
            x |= sign;
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

void nto_f2h_array(const float *in, uint16_t *out, int64_t n)
{
    for (int64_t i = 0; i < n; ++i) out[i] = nto_f2h(in[i]);
}

void nto_h2f_array(const uint16_t *in, float *out, int64_t n)
{
    for (int64_t i = 0; i < n; ++i) out[i] = nto_h2f(in[i]);
}

static inline float r16(float f) { return nto_h2f(nto_f2h(f)); }

/* ------------------------------------------------------------------------------------ */
/* RNG and sample placement                                                              */
/* ------------------------------------------------------------------------------------ */

/* train.cu:833: RNG rng(sampleIndex ^ ((uint32_t)params.step * 747796405u + 2891336453u)).
 * The build adds a user seed folded in with a multiplicative hash; seed 0 keeps the
 * reference's seeding exactly. */
uint32_t nto_rng_seed(uint32_t sample_index, uint32_t step, uint32_t seed)
{
    uint32_t s = sample_index ^ (step * 747796405u + 2891336453u) ^ (seed * 0x9E3779B9u);
    return s ? s : 1u; /* train.cu:41 */
}

/* train.cu:43-51 xorshift32 */
uint32_t nto_rng_next(uint32_t *state)
{
    uint32_t x = *state;
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    *state = x;
    return x;
}

/* train.cu:53-56 */
float nto_rng_uniform(uint32_t *state)
{
    return (float)(nto_rng_next(state) & 0x00FFFFFFu) * (1.0f / 16777216.0f);
}

static inline float clampf(float x, float lo, float hi) /* train.cu:60-63 */
{
    return x < lo ? lo : (x > hi ? hi : x);
}

/* train.cu:827-844: one jittered sample per lattice cell, clamped to the image.  The
 * reference's cell is one texel of a 512^2 region (stride 1); the build allows a stride of
 * several texels so that the lattice covers the whole image.  Order of float operations:
 * t = ((float)ix + 0.5f) + jitter; pos = t * stride + offset; clamp; u = pos / width. */
void nto_sample_uv(const nto_sampler *s, int64_t index, float *u, float *v)
{
    const int32_t ix = (int32_t)(index % s->lattice_w);
    const int32_t iy = (int32_t)(index / s->lattice_w);
    uint32_t st = nto_rng_seed((uint32_t)index, (uint32_t)s->step, s->seed);
    const float jx = nto_rng_uniform(&st) - 0.5f;
    const float jy = nto_rng_uniform(&st) - 0.5f;
    float tx = ((float)ix + 0.5f) + jx;
    float ty = ((float)iy + 0.5f) + jy;
    float px = tx * s->stride_x + (float)s->offset_x;
    float py = ty * s->stride_y + (float)s->offset_y;
    px = clampf(px, 0.5f, (float)s->image_w - 0.5f);
    py = clampf(py, 0.5f, (float)s->image_h - 0.5f);
    *u = px / (float)s->image_w;
    *v = py / (float)s->image_h;
}

void nto_sample_uv_array(const nto_sampler *s, float *uv)
{
    const int64_t n = (int64_t)s->lattice_w * s->lattice_h;
    for (int64_t i = 0; i < n; ++i) nto_sample_uv(s, i, &uv[2 * i], &uv[2 * i + 1]);
}

/* ------------------------------------------------------------------------------------ */
/* Catmull-Rom sampling                                                                  */
/* ------------------------------------------------------------------------------------ */

/* filter/catmull_rom.h:56-59 (pre-expanded Catmull-Rom, a = -0.5) */
void nto_catmull_rom_weights(float f, float w[4])
{
    w[0] = f * (f * (f * -0.5f + 1.0f) - 0.5f);
    w[1] = f * f * (f * 1.5f - 2.5f) + 1.0f;
    w[2] = f * (f * (f * -1.5f + 2.0f) + 0.5f);
    w[3] = f * f * (f * 0.5f - 0.5f);
}

/* train.cu:65-69 */
int32_t nto_wrap(int32_t coord, int32_t size)
{
    int32_t r = coord % size;
    return r < 0 ? r + size : r;
}

/* filter/catmull_rom.h:46-52: samplePos = uv * size; texPos1 = floor(samplePos - 0.5) + 0.5;
 * f = samplePos - texPos1.  Returns the index of texel texPos1 (the [1, 1] tap). */
static int32_t cr_base(float uv, int32_t size, float *f)
{
    const float sp = uv * (float)size;
    const float fl = floorf(sp - 0.5f);
    *f = sp - (fl + 0.5f);
    return (int32_t)fl;
}

/* Texel-centre convention and 4x4 footprint of filter/catmull_rom.h:46-59 (texels
 * base-1 .. base+2), wrap addressing of train.cu:65-69.  The reference samples its latents
 * bilinearly and accumulates in fp16 (train.cu:263-314); the build samples them with the
 * reference's Catmull-Rom filter and accumulates in fp32: row sums first, then the
 * weighted sum of rows. */
void nto_sample_grid(const uint16_t *grid, int32_t w, int32_t h, int32_t c, float u, float v,
                     float *out, int32_t base_out[2], float wx_out[4], float wy_out[4])
{
    float fx, fy;
    const int32_t bx = cr_base(u, w, &fx), by = cr_base(v, h, &fy);
    float wx[4], wy[4];
    nto_catmull_rom_weights(fx, wx);
    nto_catmull_rom_weights(fy, wy);
    float acc[16] = {0};
    for (int j = 0; j < 4; ++j) {
        const int32_t yy = nto_wrap(by - 1 + j, h);
        float row[16] = {0};
        for (int i = 0; i < 4; ++i) {
            const int32_t xx = nto_wrap(bx - 1 + i, w);
            const uint16_t *t = grid + ((int64_t)yy * w + xx) * c;
            for (int k = 0; k < c; ++k) row[k] += wx[i] * nto_h2f(t[k]);
        }
        for (int k = 0; k < c; ++k) acc[k] += wy[j] * row[k];
    }
    for (int k = 0; k < c; ++k) out[k] = acc[k];
    if (base_out) { base_out[0] = bx; base_out[1] = by; }
    if (wx_out) memcpy(wx_out, wx, sizeof wx);
    if (wy_out) memcpy(wy_out, wy, sizeof wy);
}

/* Positional features (no reference counterpart: the reference MLP input is latents
 * only): [sin 2pi u, cos 2pi u, sin 2pi v, cos 2pi v, sin 4pi u, cos 4pi u, sin 4pi v,
 * cos 4pi v]. */
void nto_posenc(float u, float v, float out[8])
{
    for (int k = 0; k < 2; ++k) {
        const float m = (float)(2 << k); /* 2, 4: argument in units of pi */
        const double au = M_PI * (double)(m * u);
        const double av = M_PI * (double)(m * v);
        out[4 * k + 0] = (float)sin(au);
        out[4 * k + 1] = (float)cos(au);
        out[4 * k + 2] = (float)sin(av);
        out[4 * k + 3] = (float)cos(av);
    }
}

/* ------------------------------------------------------------------------------------ */
/* Network forward                                                                       */
/* ------------------------------------------------------------------------------------ */

/* One layer y[o] = b[o] + sum_i x[i] * W[o * pad_in + i] (column-major, main.cpp:195,
 * mlp.h:18-40), fp32 accumulation (double here: the oracle is the exact sum). */
/* ---- BC6 block features ------------------------------------------------------------- */

static const int32_t bc6f_part_masks[32] = { /* train.cu:20-29, gBC6HPartitionSets */
    0xCCCC, 0x8888, 0xEEEE, 0xECC8, 0xC880, 0xFEEC, 0xFEC8, 0xEC80, 0xC800, 0xFFEC, 0xFE80,
    0xE800, 0xFFE8, 0xFF00, 0xFFF0, 0xF000, 0xF710, 0x008E, 0x7100, 0x08CE, 0x008C, 0x7310,
    0x3100, 0x8CCE, 0x088C, 0x3110, 0x6666, 0x366C, 0x17E8, 0x0FF0, 0x718E, 0x399C};
static const int32_t bc6f_mode_bits[10] = {10, 7, 11, 11, 11, 9, 8, 8, 8, 6}; /* train.cu:31-34 */

/* train.cu:161-167 UnquantizeEndpoints */
static float bc6f_unquantize(float e, int32_t b)
{
    const float scale = (31.f / 64.f) * 65536.f;
    return ldexpf(scale * e + 32768.f, -b);
}

/* train.cu:169-182 DecompressBC6, per channel; also returns the intermediates the backward
 * pass needs (train.cu:184-202). */
static float bc6f_channel(float e0, float e1, int32_t b, float x, float *eb0, float *eb1, float *y_out)
{
    const int q = 3;
    const float u0 = bc6f_unquantize(e0, b), u1 = bc6f_unquantize(e1, b);
    const float y = u0 + ldexpf(u1 - u0, q) * x;
    float hyf = floorf((y - 1.f) / 1024.f) - 1.f;
    hyf = hyf > 0.f ? hyf : 0.f;
    const int32_t hy = (int32_t)hyf;
    if (eb0) *eb0 = u0;
    if (eb1) *eb1 = u1;
    if (y_out) *y_out = y;
    return ldexpf(y / 1024.f - (float)hy, hy - 14);
}

void nto_bc6f_decode(const float e0[3], const float e1[3], int32_t bits, float x, float out[3])
{
    for (int c = 0; c < 3; ++c) out[c] = bc6f_channel(e0[c], e1[c], bits, x, NULL, NULL, NULL);
}

/* train.cu:204-212 block / pixel index, :240-261 SampleBC6FeatureTexel, per channel triple */
static const float *bc6f_block(const float *blocks, int32_t w, int32_t T, int32_t x, int32_t y, int32_t t)
{
    const int64_t b = (int64_t)(y >> 2) * (w >> 2) + (x >> 2);
    return blocks + (b * T + t) * NTO_BC6F_FLOATS;
}

static int32_t bc6f_int(const float *p, int k)
{
    int32_t v;
    memcpy(&v, p + k, sizeof v);
    return v;
}

void nto_bc6f_texel(const float *blocks, int32_t w, int32_t channels, int32_t x, int32_t y, float *out)
{
    const int32_t T = (channels + 2) / 3, pix = ((y & 3) << 2) + (x & 3);
    for (int32_t t = 0; t < T; ++t) {
        const float *p = bc6f_block(blocks, w, T, x, y, t);
        const int32_t part = bc6f_int(p, 28) & 31, mode = bc6f_int(p, 29);
        const int32_t r = (bc6f_part_masks[part] >> pix) & 1;
        const int32_t bits = bc6f_mode_bits[mode < 0 || mode > 9 ? 0 : mode];
        float v[3];
        nto_bc6f_decode(p + 6 * r, p + 6 * r + 3, bits, p[12 + pix], v);
        for (int c = 0; c < 3; ++c)
            if (3 * t + c < channels) out[3 * t + c] = v[c];
    }
}

/* Catmull-Rom sample of a block-feature grid (nto_sample_grid's footprint and order). */
static void sample_blocks(const float *blocks, int32_t w, int32_t h, int32_t C, float u, float v, float *out,
                          int32_t base_out[2], float wx_out[4], float wy_out[4])
{
    float fx, fy;
    const int32_t bx = cr_base(u, w, &fx), by = cr_base(v, h, &fy);
    float wx[4], wy[4];
    nto_catmull_rom_weights(fx, wx);
    nto_catmull_rom_weights(fy, wy);
    float acc[16] = {0};
    for (int j = 0; j < 4; ++j) {
        const int32_t yy = nto_wrap(by - 1 + j, h);
        float row[16] = {0};
        for (int i = 0; i < 4; ++i) {
            const int32_t xx = nto_wrap(bx - 1 + i, w);
            float t[16];
            nto_bc6f_texel(blocks, w, C, xx, yy, t);
            for (int k = 0; k < C; ++k) row[k] += wx[i] * t[k];
        }
        for (int k = 0; k < C; ++k) acc[k] += wy[j] * row[k];
    }
    for (int k = 0; k < C; ++k) out[k] = acc[k];
    if (base_out) { base_out[0] = bx; base_out[1] = by; }
    if (wx_out) memcpy(wx_out, wx, sizeof wx);
    if (wy_out) memcpy(wy_out, wy, sizeof wy);
}

/* train.cu:436-454: gradients of one texel of a block-feature grid for the feature gradient
 * fg (C channels, tap weight and 1 / numSamples applied): endpoints of its region and its
 * pixel index. */
static void bc6f_backward_texel(const float *blocks, float *grads, int32_t w, int32_t C, int32_t x, int32_t y,
                                const float *fg)
{
    const int32_t T = (C + 2) / 3, pix = ((y & 3) << 2) + (x & 3);
    const int q = 3;
    for (int32_t t = 0; t < T; ++t) {
        const float *p = bc6f_block(blocks, w, T, x, y, t);
        float *gp = grads + (bc6f_block(blocks, w, T, x, y, t) - blocks);
        const int32_t part = bc6f_int(p, 28) & 31, mode = bc6f_int(p, 29);
        const int32_t r = (bc6f_part_masks[part] >> pix) & 1;
        const int32_t bits = bc6f_mode_bits[mode < 0 || mode > 9 ? 0 : mode];
        const float xv = p[12 + pix];
        const float alpha = ldexpf(xv, q);
        const float deibar_dei = ldexpf(31.f / 64, 16 - bits);
        float dl_dx = 0.f;
        float d0[3], d1[3];
        for (int c = 0; c < 3; ++c) {
            const float g = 3 * t + c < C ? fg[3 * t + c] : 0.f;
            float eb0, eb1, y;
            bc6f_channel(p[6 * r + c], p[6 * r + 3 + c], bits, xv, &eb0, &eb1, &y);
            float hyf = floorf((y - 1.f) / 1024.f) - 1.f;
            hyf = hyf > 0.f ? hyf : 0.f;
            const float dl_dy = ldexpf(g, (int32_t)hyf - 24);
            dl_dx += dl_dy * ldexpf(eb1 - eb0, q);
            d0[c] = (1.f - alpha) * deibar_dei * dl_dy;
            d1[c] = alpha * deibar_dei * dl_dy;
        }
        for (int c = 0; c < 3; ++c) {
#ifdef _OPENMP
#pragma omp atomic
#endif
            gp[6 * r + c] += d0[c];
#ifdef _OPENMP
#pragma omp atomic
#endif
            gp[6 * r + 3 + c] += d1[c];
        }
#ifdef _OPENMP
#pragma omp atomic
#endif
        gp[12 + pix] += dl_dx;
    }
}

static void layer(const float *x, int n_in, int pad_in, const uint16_t *W, const uint16_t *b,
                  int n_out, float *y)
{
    for (int o = 0; o < n_out; ++o) {
        double s = b ? (double)nto_h2f(b[o]) : 0.0;
        const uint16_t *col = W + (int64_t)o * pad_in;
        for (int i = 0; i < n_in; ++i) s += (double)x[i] * (double)nto_h2f(col[i]);
        y[o] = (float)s;
    }
}

/* Forward pass of one sample: sample both grids (fp32, rounded to fp16 as MLP input),
 * positional features, 32 -> 64 ReLU -> 64 ReLU -> cout.  Hidden activations are rounded
 * to fp16 (they are tensor-core operands); the output is rounded to fp16 like the
 * reference's half output vector (train.cu:878, mlp.h:65-99). */
/* Two-level blend of a mip chain (train.cu:102, :303-304): (1 - t) a + t b. */
static float mip_blend(float a, float b, float t)
{
    return (1.f - t) * a + t * b;
}

void nto_forward_sample(const nto_model *m, float u, float v, nto_fwd *f)
{
    const int C = m->channels;
    float feat[16];
    memset(f->x, 0, sizeof f->x);
    for (int g = 0; g < 2; ++g) {
        if (m->blocks[g])
            sample_blocks(m->blocks[g], m->gw[g], m->gh[g], C, u, v, feat, f->base[g], f->wx[g], f->wy[g]);
        else
            nto_sample_grid(m->grid[g], m->gw[g], m->gh[g], C, u, v, feat, f->base[g], f->wx[g],
                            f->wy[g]);
        if (m->grid_b[g] && m->mip_t[g] > 0.f) {
            float fb[16];
            nto_sample_grid(m->grid_b[g], m->gw_b[g], m->gh_b[g], C, u, v, fb, f->base_b[g], f->wx_b[g],
                            f->wy_b[g]);
            for (int k = 0; k < C; ++k) feat[k] = mip_blend(feat[k], fb[k], m->mip_t[g]);
        }
        for (int k = 0; k < C; ++k) f->x[g * C + k] = r16(feat[k]);
    }
    float pe[8];
    nto_posenc(u, v, pe);
    for (int k = 0; k < 8; ++k) f->x[2 * C + k] = r16(pe[k]);

    float t[64];
    layer(f->x, 32, 32, m->W[0], m->b[0], 64, t);
    for (int i = 0; i < 64; ++i) f->h1[i] = r16(t[i] > 0.f ? t[i] : 0.f);
    layer(f->h1, 64, 64, m->W[1], m->b[1], 64, t);
    for (int i = 0; i < 64; ++i) f->h2[i] = r16(t[i] > 0.f ? t[i] : 0.f);
    layer(f->h2, 64, 64, m->W[2], m->b[2], m->cout, t);
    for (int i = 0; i < 16; ++i) f->y[i] = i < m->cout ? r16(t[i]) : 0.f;
}

/* Catmull-Rom sample of the fp32 view of an fp16 target (filter/catmull_rom.h:39-89; the
 * reference fetches through hardware bilinear taps, the build uses the 16 exact taps). */
static void sample_target(const uint16_t *target, int32_t w, int32_t h, int32_t c, float u,
                          float v, float *out)
{
    nto_sample_grid(target, w, h, c, u, v, out, NULL, NULL, NULL);
}

/* train.cu:917-961: texel centres u = (x + 0.5) / W, forward, write outputs. */
void nto_decode_range(const nto_model *m, int32_t w, int32_t h, int64_t first, int64_t count,
                      void *out, int32_t out_f32, int32_t threads)
{
    const int cout = m->cout;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
#endif
    for (int64_t k = 0; k < count; ++k) {
        const int64_t i = first + k;
        const int32_t x = (int32_t)(i % w), y = (int32_t)(i / w);
        const float u = ((float)x + 0.5f) / (float)w;
        const float v = ((float)y + 0.5f) / (float)h;
        nto_fwd f;
        nto_forward_sample(m, u, v, &f);
        for (int c = 0; c < cout; ++c) {
            if (out_f32)
                ((float *)out)[k * cout + c] = f.y[c];
            else
                ((uint16_t *)out)[k * cout + c] = nto_f2h(f.y[c]);
        }
    }
    (void)threads;
}

void nto_decode(const nto_model *m, int32_t w, int32_t h, void *out, int32_t out_f32,
                const uint16_t *target, double *sse, int32_t threads)
{
    const int64_t n = (int64_t)w * h;
    nto_decode_range(m, w, h, 0, n, out, out_f32, threads);
    if (target && sse) { /* train.cu:955-960 */
        double s = 0.0;
        for (int64_t i = 0; i < n * m->cout; ++i) {
            const float yv = out_f32 ? ((const float *)out)[i] : nto_h2f(((const uint16_t *)out)[i]);
            const double e = (double)yv - (double)nto_h2f(target[i]);
            s += e * e;
        }
        *sse += s;
    }
}

/* ------------------------------------------------------------------------------------ */
/* Training pass                                                                         */
/* ------------------------------------------------------------------------------------ */

typedef struct grad_acc {
    double W[3][64 * 64];
    double b[3][64];
} grad_acc;

/* Backward of one sample (mlp.h:222-257 per layer, train.cu:876-912 for the loss and the
 * order).  Loss gradient: the reference rounds 2 w err / numSamples to fp16
 * (train.cu:886-887), which is subnormal at 262,144 samples; the build rounds the
 * unscaled 2 w err to fp16 and applies 1 / numSamples in fp32 to every accumulated
 * gradient, which is the same gradient without the underflow.  Hidden gradients are
 * rounded to fp16 (tensor-core operands) after the ReLU mask of the layer's input
 * (mlp.h:243-247). */
static double backward_sample(const nto_model *m, const nto_fwd *f, const float *t,
                              const float *cw, grad_acc *acc, float dx_out[32])
{
    const int cout = m->cout;
    float dy[16] = {0};
    double sse = 0.0;
    for (int c = 0; c < cout; ++c) {
        const float wgt = cw ? cw[c] : 1.0f;
        const float err = f->y[c] - t[c];
        sse += (double)wgt * (double)err * (double)err;
        dy[c] = r16(2.0f * wgt * err);
    }
    float dh2[64], dh1[64];
    for (int j = 0; j < 64; ++j) { /* dH2 = dY W3^T, W3[c * 64 + j] */
        double s = 0.0;
        for (int c = 0; c < cout; ++c) s += (double)dy[c] * nto_h2f(m->W[2][c * 64 + j]);
        dh2[j] = f->h2[j] > 0.f ? r16((float)s) : 0.f;
    }
    for (int i = 0; i < 64; ++i) { /* dH1 = dH2 W2^T, W2[j * 64 + i] */
        double s = 0.0;
        for (int j = 0; j < 64; ++j) s += (double)dh2[j] * nto_h2f(m->W[1][j * 64 + i]);
        dh1[i] = f->h1[i] > 0.f ? r16((float)s) : 0.f;
    }
    for (int k = 0; k < 32; ++k) { /* dX = dH1 W1^T, W1[i * 32 + k] */
        double s = 0.0;
        for (int i = 0; i < 64; ++i) s += (double)dh1[i] * nto_h2f(m->W[0][i * 32 + k]);
        dx_out[k] = (float)s;
    }
    /* dW[col = out][row = in] += in * dOut; db += dOut (mlp.h:101-153, :249-254) */
    for (int c = 0; c < cout; ++c) {
        acc->b[2][c] += dy[c];
        for (int j = 0; j < 64; ++j) acc->W[2][c * 64 + j] += (double)f->h2[j] * dy[c];
    }
    for (int j = 0; j < 64; ++j) {
        acc->b[1][j] += dh2[j];
        if (dh2[j] != 0.f)
            for (int i = 0; i < 64; ++i) acc->W[1][j * 64 + i] += (double)f->h1[i] * dh2[j];
    }
    for (int i = 0; i < 64; ++i) {
        acc->b[0][i] += dh1[i];
        if (dh1[i] != 0.f)
            for (int k = 0; k < 32; ++k) acc->W[0][i * 32 + k] += (double)f->x[k] * dh1[i];
    }
    return sse;
}

/* train.cu:460-509 (BackwardUnconstrainedFeaturePass) with the Catmull-Rom footprint:
 * grad[texel] += wy * wx * dL/dfeature for the 16 taps of each grid. */
static void scatter_taps(float *grad, int32_t w, int32_t h, int C, const int32_t base[2], const float wx[4],
                         const float wy[4], const float *dx, float scale)
{
    for (int j = 0; j < 4; ++j) {
        const int32_t yy = nto_wrap(base[1] - 1 + j, h);
        for (int i = 0; i < 4; ++i) {
            const int32_t xx = nto_wrap(base[0] - 1 + i, w);
            const float wgt = wy[j] * wx[i];
            float *dst = grad + ((int64_t)yy * w + xx) * C;
            for (int k = 0; k < C; ++k) {
                const float val = wgt * dx[k] * scale;
#ifdef _OPENMP
#pragma omp atomic
#endif
                dst[k] += val;
            }
        }
    }
}

static void scatter_latent(const nto_model *m, const nto_fwd *f, const float *dx, float scale,
                           float *ggrid[2], float *const ggrid_b[2])
{
    const int C = m->channels;
    for (int g = 0; g < 2; ++g) {
        if (!ggrid[g]) continue;
        if (!m->blocks[g] && m->grid_b[g] && m->mip_t[g] > 0.f) { /* two mip levels: (1 - t) and t */
            const float t = m->mip_t[g];
            float da[16], db[16];
            for (int k = 0; k < C; ++k) {
                da[k] = dx[g * C + k] * (1.f - t);
                db[k] = dx[g * C + k] * t;
            }
            scatter_taps(ggrid[g], m->gw[g], m->gh[g], C, f->base[g], f->wx[g], f->wy[g], da, scale);
            if (ggrid_b && ggrid_b[g])
                scatter_taps(ggrid_b[g], m->gw_b[g], m->gh_b[g], C, f->base_b[g], f->wx_b[g], f->wy_b[g], db, scale);
            continue;
        }
        if (m->blocks[g]) { /* train.cu:436-454 per tap of the Catmull-Rom footprint */
            for (int j = 0; j < 4; ++j) {
                const int32_t yy = nto_wrap(f->base[g][1] - 1 + j, m->gh[g]);
                for (int i = 0; i < 4; ++i) {
                    const int32_t xx = nto_wrap(f->base[g][0] - 1 + i, m->gw[g]);
                    const float wgt = f->wy[g][j] * f->wx[g][i];
                    float fg[16];
                    for (int k = 0; k < C; ++k) fg[k] = wgt * dx[g * C + k] * scale;
                    bc6f_backward_texel(m->blocks[g], ggrid[g], m->gw[g], C, xx, yy, fg);
                }
            }
            continue;
        }
        for (int j = 0; j < 4; ++j) {
            const int32_t yy = nto_wrap(f->base[g][1] - 1 + j, m->gh[g]);
            for (int i = 0; i < 4; ++i) {
                const int32_t xx = nto_wrap(f->base[g][0] - 1 + i, m->gw[g]);
                const float wgt = f->wy[g][j] * f->wx[g][i];
                float *dst = ggrid[g] + ((int64_t)yy * m->gw[g] + xx) * C;
                for (int k = 0; k < C; ++k) {
                    const float val = wgt * dx[g * C + k] * scale;
#ifdef _OPENMP
#pragma omp atomic
#endif
                    dst[k] += val;
                }
            }
        }
    }
}

double nto_train_pass_range(const nto_model *m, const nto_train_args *a, int64_t first,
                            int64_t count, float *gW[3], float *gb[3], float *ggrid[2],
                            int32_t threads)
{
    const nto_sampler *s = &a->sampler;
    const int64_t total = (int64_t)s->lattice_w * s->lattice_h;
    const float scale = 1.0f / (float)total;
    const int pad_in[3] = {32, 64, 64};
    const int n_out[3] = {64, 64, 16};
    float *no_grid[2] = {NULL, NULL};
    float **gg = a->finalize ? no_grid : ggrid;
    double sse_total = 0.0;
    int nthreads = threads > 0 ? threads : 1;
    grad_acc *accs = (grad_acc *)calloc((size_t)nthreads, sizeof(grad_acc));
#ifdef _OPENMP
#pragma omp parallel num_threads(nthreads) reduction(+ : sse_total)
#endif
    {
        int tid = 0;
#ifdef _OPENMP
        tid = omp_get_thread_num();
#endif
        grad_acc *acc = &accs[tid];
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int64_t k = 0; k < count; ++k) {
            const int64_t i = first + k;
            float u, v;
            nto_sample_uv(s, i, &u, &v);
            nto_fwd f;
            nto_forward_sample(m, u, v, &f);
            float t[16] = {0};
            float rw[16];
            const int32_t tw = a->target_w > 0 ? a->target_w : s->image_w;
            const int32_t th = a->target_h > 0 ? a->target_h : s->image_h;
            if (a->num_ref > 0)
                nto_ref_expected(a->ref, a->num_ref, u, v, a->lod, t, rw);
            else
                sample_target(a->target, tw, th, m->cout, u, v, t);
            if (a->num_ref == 0 && a->target_b && a->target_t > 0.f) {
                float tb[16] = {0};
                sample_target(a->target_b, a->target_w_b, a->target_h_b, m->cout, u, v, tb);
                for (int c = 0; c < m->cout; ++c) t[c] = mip_blend(t[c], tb[c], a->target_t);
            }
            float dx[32];
            sse_total += backward_sample(m, &f, t, a->num_ref > 0 ? rw : a->channel_weights, acc, dx);
            scatter_latent(m, &f, dx, scale, gg, a->finalize ? NULL : a->ggrid_b);
        }
    }
    for (int l = 0; l < 3; ++l) {
        const int nw = pad_in[l] * n_out[l];
        const int nb = l == 2 ? m->cout : 64;
        for (int e = 0; e < nw; ++e) {
            double s2 = 0.0;
            for (int t = 0; t < nthreads; ++t) s2 += accs[t].W[l][e];
            if (gW && gW[l]) gW[l][e] += (float)(s2 * (double)scale);
        }
        for (int e = 0; e < nb; ++e) {
            double s2 = 0.0;
            for (int t = 0; t < nthreads; ++t) s2 += accs[t].b[l][e];
            if (gb && gb[l]) gb[l][e] += (float)(s2 * (double)scale);
        }
    }
    free(accs);
    return sse_total;
}

double nto_train_pass(const nto_model *m, const nto_train_args *a, float *gW[3], float *gb[3],
                      float *ggrid[2], int32_t threads)
{
    const int64_t total = (int64_t)a->sampler.lattice_w * a->sampler.lattice_h;
    return nto_train_pass_range(m, a, 0, total, gW, gb, ggrid, threads);
}

/* ------------------------------------------------------------------------------------ */
/* Reference textures                                                                    */
/* ------------------------------------------------------------------------------------ */

static int32_t g_tex_filter_mode = 1;

void nto_set_texture_filter_mode(int32_t mode) { g_tex_filter_mode = mode; }

static float tex_weight(float a)
{
    if (g_tex_filter_mode == 1) return floorf(a * 256.f + 0.5f) / 256.f;
    if (g_tex_filter_mode == 2) return floorf(a * 256.f) / 256.f;
    return a;
}

/* One hardware bilinear fetch of level m at normalized (x, y), wrap addressing. */
static void ref_bilinear(const nto_ref_texture *t, int32_t m, float x, float y, float out[4])
{
    const int32_t cc = t->channels == 3 ? 4 : t->channels;
    const int32_t lw = nto_mip_dim(t->w, m), lh = nto_mip_dim(t->h, m);
    const float *lv = t->chain + nto_mip_offset(t->w, t->h, m) * cc;
    const float xs = (x - floorf(x)) * (float)lw - 0.5f, ys = (y - floorf(y)) * (float)lh - 0.5f;
    const float fx = floorf(xs), fy = floorf(ys);
    const float a = tex_weight(xs - fx), b = tex_weight(ys - fy);
    const int32_t x0 = nto_wrap((int32_t)fx, lw), x1 = nto_wrap((int32_t)fx + 1, lw);
    const int32_t y0 = nto_wrap((int32_t)fy, lh), y1 = nto_wrap((int32_t)fy + 1, lh);
    for (int c = 0; c < 4; ++c) {
        if (c >= t->channels || (t->channels == 3 && c == 3)) {
            out[c] = 0.f;
            continue;
        }
        const float t00 = lv[((int64_t)y0 * lw + x0) * cc + c], t10 = lv[((int64_t)y0 * lw + x1) * cc + c];
        const float t01 = lv[((int64_t)y1 * lw + x0) * cc + c], t11 = lv[((int64_t)y1 * lw + x1) * cc + c];
        out[c] = (1.f - a) * (1.f - b) * t00 + a * (1.f - b) * t10 + (1.f - a) * b * t01 + a * b * t11;
    }
}

/* filter/catmull_rom.h:39-89: Catmull-Rom from 9 bilinear fetches, the middle taps of each
 * axis merged at w2 / (w1 + w2). */
static void ref_catmull_rom(const nto_ref_texture *t, float u, float v, int32_t m, float out[4])
{
    const float size[2] = {(float)nto_mip_dim(t->w, m), (float)nto_mip_dim(t->h, m)};
    const float uv[2] = {u, v};
    float w[2][3], pos[2][3];
    for (int a = 0; a < 2; ++a) {
        const float sp = uv[a] * size[a];
        const float t1 = floorf(sp - 0.5f) + 0.5f;
        const float f = sp - t1;
        float cr[4];
        nto_catmull_rom_weights(f, cr);
        const float w12 = cr[1] + cr[2];
        w[a][0] = cr[0];
        w[a][1] = w12;
        w[a][2] = cr[3];
        pos[a][0] = (t1 - 1.f) / size[a];
        pos[a][1] = (t1 + cr[2] / w12) / size[a];
        pos[a][2] = (t1 + 2.f) / size[a];
    }
    for (int c = 0; c < 4; ++c) out[c] = 0.f;
    for (int j = 0; j < 3; ++j)
        for (int i = 0; i < 3; ++i) {
            float s[4];
            ref_bilinear(t, m, pos[0][i], pos[1][j], s);
            const float k = w[0][i] * w[1][j];
            for (int c = 0; c < 4; ++c) out[c] += s[c] * k;
        }
}

/* train.cu:78-103 */
void nto_ref_trilinear(const nto_ref_texture *t, float u, float v, float lod, float out[4])
{
    int32_t m0, m1;
    float f;
    nto_mip_select(t->num_mips, lod, &m0, &m1, &f);
    ref_catmull_rom(t, u, v, m0, out);
    if (f <= 0.f) return;
    float s1[4];
    ref_catmull_rom(t, u, v, m1, s1);
    for (int c = 0; c < 4; ++c) out[c] = out[c] * (1.f - f) + s1[c] * f;
}

void nto_ref_expected(const nto_ref_texture *t, int32_t n, float u, float v, float lod, float expected[16],
                      float weights[16])
{
    for (int k = 0; k < 16; ++k) {
        expected[k] = 0.f;
        if (weights) weights[k] = 1.f;
    }
    int oc = 0;
    for (int i = 0; i < n && oc < 16; ++i) {
        if (!t[i].chain || t[i].channels <= 0) continue;
        float s[4];
        nto_ref_trilinear(&t[i], u, v, lod, s);
        for (int c = 0; c < t[i].channels && c < 4 && oc < 16; ++c, ++oc) {
            expected[oc] = s[c];
            if (weights) weights[oc] = t[i].loss_weight;
        }
    }
}

/* ------------------------------------------------------------------------------------ */
/* Mip chains                                                                            */
/* ------------------------------------------------------------------------------------ */

int32_t nto_mip_dim(int32_t size, int32_t m) /* train.cu:214-218 */
{
    const int32_t d = size >> m;
    return d > 0 ? d : 1;
}

int64_t nto_mip_offset(int32_t w, int32_t h, int32_t m)
{
    int64_t off = 0;
    for (int32_t k = 0; k < m; ++k) off += (int64_t)nto_mip_dim(w, k) * nto_mip_dim(h, k);
    return off;
}

/* train.cu:83-87 (SampleReferenceTextureTrilinear); the feature sampler of train.cu:266-282
 * picks the same levels and weights for every lod in [0, n - 1]. */
void nto_mip_select(int32_t num_mips, float lod, int32_t *m0, int32_t *m1, float *t)
{
    const int32_t last = num_mips > 1 ? num_mips - 1 : 0;
    float c = lod > 0.f ? lod : 0.f; /* NaN -> 0 */
    if (c > (float)last) c = (float)last;
    int32_t a = (int32_t)floorf(c);
    if (a > last) a = last;
    const int32_t b = a + 1 < last ? a + 1 : last;
    *m0 = a;
    *m1 = b;
    *t = b > a ? c - (float)a : 0.f;
}

void nto_build_mips(uint16_t *chain, int32_t w, int32_t h, int32_t c, int32_t num_mips)
{
    for (int32_t m = 1; m < num_mips; ++m) {
        const int32_t sw = nto_mip_dim(w, m - 1), sh = nto_mip_dim(h, m - 1);
        const int32_t dw = nto_mip_dim(w, m), dh = nto_mip_dim(h, m);
        const uint16_t *src = chain + nto_mip_offset(w, h, m - 1) * c;
        uint16_t *dst = chain + nto_mip_offset(w, h, m) * c;
        for (int32_t y = 0; y < dh; ++y)
            for (int32_t x = 0; x < dw; ++x) {
                const int32_t x0 = 2 * x < sw ? 2 * x : sw - 1, x1 = 2 * x + 1 < sw ? 2 * x + 1 : sw - 1;
                const int32_t y0 = 2 * y < sh ? 2 * y : sh - 1, y1 = 2 * y + 1 < sh ? 2 * y + 1 : sh - 1;
                for (int32_t k = 0; k < c; ++k) {
                    const float a = nto_h2f(src[((int64_t)y0 * sw + x0) * c + k]);
                    const float b = nto_h2f(src[((int64_t)y0 * sw + x1) * c + k]);
                    const float d = nto_h2f(src[((int64_t)y1 * sw + x0) * c + k]);
                    const float e = nto_h2f(src[((int64_t)y1 * sw + x1) * c + k]);
                    dst[((int64_t)y * dw + x) * c + k] = nto_f2h(((a + b) + (d + e)) * 0.25f);
                }
            }
    }
}

/* ------------------------------------------------------------------------------------ */
/* Adam                                                                                  */
/* ------------------------------------------------------------------------------------ */

/* train.cu:528-531: t = max(step, 1); 1 - beta^t.  Computed once per step on the host
 * (the reference evaluates powf per element on the device). */
void nto_adam_bias_correction(float beta1, float beta2, int32_t step, float *bc1, float *bc2)
{
    const int t = step > 0 ? step : 1;
    *bc1 = 1.0f - powf(beta1, (float)t);
    *bc2 = 1.0f - powf(beta2, (float)t);
}

/* train.cu:533-542 with the float operations in the order written there; each product
 * and sum rounds separately (no fused multiply-add). */
static inline float adam_update(float w, float g, float *m, float *v, float lr, float b1,
                                float b2, float eps, float bc1, float bc2)
{
    const float m1 = b1 * *m + (1.f - b1) * g;
    const float m2 = b2 * *v + (1.f - b2) * g * g;
    *m = m1;
    *v = m2;
    const float mhat = m1 / bc1;
    const float vhat = m2 / bc2;
    return w - lr * mhat / (sqrtf(vhat) + eps);
}

/* train.cu:566-588 OptimizeParameterBuffer: skip zero gradients, zero them after use. */
void nto_adam_f16(uint16_t *w, float *g, float *m, float *v, int64_t n, float lr, float beta1,
                  float beta2, float eps, float bc1, float bc2)
{
    for (int64_t i = 0; i < n; ++i) {
        const float gi = g[i];
        if (gi == 0.f) continue;
        w[i] = nto_f2h(adam_update(nto_h2f(w[i]), gi, &m[i], &v[i], lr, beta1, beta2, eps, bc1,
                                   bc2));
        g[i] = 0.f;
    }
}

/* train.cu:545-564, :625-639 */
void nto_adam_f32(float *w, float *g, float *m, float *v, int64_t n, float lr, float beta1,
                  float beta2, float eps, float bc1, float bc2)
{
    for (int64_t i = 0; i < n; ++i) {
        const float gi = g[i];
        if (gi == 0.f) continue;
        w[i] = adam_update(w[i], gi, &m[i], &v[i], lr, beta1, beta2, eps, bc1, bc2);
        g[i] = 0.f;
    }
}

/* ------------------------------------------------------------------------------------ */
/* Synthetic target (2; no reference counterpart)                    */
/* ------------------------------------------------------------------------------------ */

/* "lowbias32" integer hash (C. Wellons), used for all seeded parameters. */
static uint32_t hash32(uint32_t x)
{
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

static uint32_t isqrt32(uint32_t n)
{
    uint32_t r = 0;
    while ((r + 1) * (r + 1) <= n) ++r;
    return r;
}

/* Sinusoid k of channel c: integer frequency vector (fu, fv) with |f| ~ 1..64 cycles per
 * texture (integer so the target tiles under wrap addressing), phase in cycles, amplitude. */
void nto_target_params(uint32_t seed, int32_t channel, int32_t k, int32_t *fu, int32_t *fv,
                       float *phase, float *amp)
{
    const uint32_t base = hash32(seed * 0x9E3779B9u ^ hash32((uint32_t)(channel * 64 + k + 1)));
    const uint32_t f = 1u + hash32(base ^ 0x1u) % 64u;                 /* 1..64 */
    const int32_t a = (int32_t)(hash32(base ^ 0x2u) % (2u * f + 1u)) - (int32_t)f; /* -f..f */
    int32_t b = (int32_t)isqrt32(f * f - (uint32_t)(a * a));
    if (hash32(base ^ 0x3u) & 1u) b = -b;
    *fu = a;
    *fv = b;
    if (a == 0 && b == 0) *fu = 1;
    *phase = (float)(hash32(base ^ 0x4u) >> 8) * (1.0f / 16777216.0f);
    *amp = 0.25f + 0.5f * ((float)(hash32(base ^ 0x5u) >> 8) * (1.0f / 16777216.0f));
}

/* fraction of f * (2x + 1) / (2n), computed exactly in integers */
static double frac_cycles(int32_t f, int32_t x, int32_t n)
{
    const int64_t den = 2 * (int64_t)n;
    int64_t num = ((int64_t)f * (2 * (int64_t)x + 1)) % den;
    if (num < 0) num += den;
    return (double)num / (double)den;
}

static void channel_value(uint32_t seed, int32_t c, int32_t x, int32_t y, int32_t w, int32_t h,
                          double *s_out, double *dsdu, double *dsdv)
{
    double s = 0.0, du = 0.0, dv = 0.0;
    for (int k = 0; k < 16; ++k) {
        int32_t fu, fv;
        float ph, amp;
        nto_target_params(seed, c, k, &fu, &fv, &ph, &amp);
        double t = frac_cycles(fu, x, w) + frac_cycles(fv, y, h) + (double)ph;
        t -= floor(t);
        s += amp * sin(2.0 * M_PI * t);
        const double cs = amp * 2.0 * M_PI * cos(2.0 * M_PI * t);
        du += cs * fu;
        dv += cs * fv;
    }
    *s_out = s;
    if (dsdu) *dsdu = du;
    if (dsdv) *dsdv = dv;
}

/* Per texel centre, channel value sigmoid(sum_k amp_k sin(2 pi (fu u + fv v + phase_k))).
 * pbr_normals (12 channels): channels 3..5 hold the normal derived from the height
 * channel 9, normalize(-dh/du / 64, -dh/dv / 64, 1) * 0.5 + 0.5. */
void nto_generate_target(uint16_t *out, int32_t w, int32_t h, int32_t channels, uint32_t seed,
                         int32_t pbr_normals, int32_t threads)
{
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
#endif
    for (int64_t i = 0; i < (int64_t)w * h; ++i) {
        const int32_t x = (int32_t)(i % w), y = (int32_t)(i / w);
        for (int c = 0; c < channels; ++c) {
            double s;
            channel_value(seed, c, x, y, w, h, &s, NULL, NULL);
            out[i * channels + c] = nto_f2h((float)(1.0 / (1.0 + exp(-s))));
        }
        if (pbr_normals && channels == 12) {
            double s, du, dv;
            channel_value(seed, 9, x, y, w, h, &s, &du, &dv);
            const double hv = 1.0 / (1.0 + exp(-s));
            const double g = hv * (1.0 - hv) / 64.0;
            double nx = -g * du, ny = -g * dv, nz = 1.0;
            const double len = sqrt(nx * nx + ny * ny + nz * nz);
            nx /= len; ny /= len; nz /= len;
            out[i * channels + 3] = nto_f2h((float)(nx * 0.5 + 0.5));
            out[i * channels + 4] = nto_f2h((float)(ny * 0.5 + 0.5));
            out[i * channels + 5] = nto_f2h((float)(nz * 0.5 + 0.5));
        }
    }
    (void)threads;
}

/* ------------------------------------------------------------------------------------ */
/* Known-answer test of tests/forward_pass_test.cu                                       */
/* ------------------------------------------------------------------------------------ */

/* tests/forward_pass_test.cu:45-108 (generator), 32 lanes x 12 inputs, 16x16 weights in
 * column-major W[in + out * 16], padded rows / columns zero. */
void nto_fwdtest_generate(uint16_t inputs[32 * 12], uint16_t w0[256], uint16_t w1[256],
                          uint16_t b0[16], uint16_t b1[16])
{
    for (int lane = 0; lane < 32; ++lane)
        for (int k = 0; k < 12; ++k)
            inputs[lane * 12 + k] =
                nto_f2h(0.125f + 0.01171875f * (float)(lane + 1) + 0.0068359375f * (float)(k + 1));
    for (int o = 0; o < 16; ++o)
        for (int i = 0; i < 16; ++i) {
            float val = 0.f;
            if (i < 12)
                val = 0.0625f + 0.0048828125f * (float)((3 * o + 1) % 7) +
                      0.0029296875f * (float)((5 * i + 2) % 11);
            w0[i + o * 16] = nto_f2h(val);
        }
    for (int o = 0; o < 16; ++o)
        for (int i = 0; i < 16; ++i) {
            /* the reference's condition outChannel < NT_OUTPUT_SIZE is always true */
            const float val = 0.09375f + 0.00341796875f * (float)((7 * o + 3) % 13) +
                              0.001953125f * (float)((2 * i + 5) % 9);
            w1[i + o * 16] = nto_f2h(val);
        }
    for (int o = 0; o < 16; ++o) {
        b0[o] = nto_f2h(0.046875f + 0.00390625f * (float)((4 * o + 1) % 9));
        b1[o] = nto_f2h(0.078125f + 0.005859375f * (float)((5 * o + 2) % 7));
    }
}

/* tests/forward_pass_test.cu:110-150 (fp32 host reference, ReLU on the hidden layer) */
void nto_fwdtest_reference(const uint16_t inputs[32 * 12], const uint16_t w0[256],
                           const uint16_t w1[256], const uint16_t b0[16], const uint16_t b1[16],
                           float out[32 * 16])
{
    for (int lane = 0; lane < 32; ++lane) {
        float hidden[16];
        for (int o = 0; o < 16; ++o) {
            float s = nto_h2f(b0[o]);
            for (int i = 0; i < 16; ++i) {
                const float x = i < 12 ? nto_h2f(inputs[lane * 12 + i]) : 0.f;
                s += x * nto_h2f(w0[i + o * 16]);
            }
            hidden[o] = s > 0.f ? s : 0.f;
        }
        for (int o = 0; o < 16; ++o) {
            float s = nto_h2f(b1[o]);
            for (int i = 0; i < 16; ++i) s += hidden[i] * nto_h2f(w1[i + o * 16]);
            out[lane * 16 + o] = s;
        }
    }
}

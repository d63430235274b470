/*
 * nt_oracle_codec.c -- CPU restatement of the BC6H-style latent block codec.
 *
 * TEST INFRASTRUCTURE ONLY (bit-exact checker of the CUDA codec and CPU baseline).
 *
 * The reference (mavenkim2/neural_textures) carries only a differentiable float decode of
 * BC6-like blocks (train.cu:161-202) and the 2-region partition table (train.cu:20-34); it
 * has no encoder and no integer bitstream.  This file restates the published BC6H format
 * (Direct3D 11 functional specification, BC6H; Khronos Data Format Specification, BC6H):
 * decode of all 14 modes, signed (SF16) and unsigned (UF16), and the build's own
 * deterministic integer encoder for UF16, which the CUDA encoder must match bit for bit.
 *
 * Latents are signed, and BC6H interpolates half-float bit patterns, which is meaningful
 * only within one sign; the surfaces are therefore encoded as UF16 of (value + bias)
 * (bias 4 for latents in [-4, 4]) and decoded as half(decoded - bias).
 *
 * Encoder (deterministic, integer only):
 *   1. texel half -> unsigned interpolation domain: m = min(h, 0x7BFF), x = ceil(64 m / 31)
 *      (the exact inverse of the format's final scale (x * 31) >> 6);
 *   2. endpoint fit per region: per-channel bounding box, oriented along the dominant
 *      channel by the sign of each channel's covariance with it;
 *   3. candidates: one-region modes 11..14 on all texels; the 2-region partition with the
 *      smallest sum over regions and channels of the squared box extent, with modes 1..10;
 *   4. per candidate: quantize endpoints to the mode precision (nearest unquantized value),
 *      swap endpoints where a region's anchor index would have its top bit set, check that
 *      transformed deltas fit, pick the nearest palette entry per texel; the candidate with
 *      the smallest integer squared error wins (ties: first in the order above).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "neural_textures/bc6h_format.h"
#include "nt_oracle.h"

static const NtBc6hMode MODES[NT_BC6H_NUM_MODES] = NT_BC6H_MODES_INIT;
static const uint8_t LAYOUT[NT_BC6H_NUM_MODES][82] = NT_BC6H_LAYOUT_INIT;
static const uint16_t PARTS[32] = NT_BC6H_PARTITIONS_INIT;
static const uint8_t ANCHORS[32] = NT_BC6H_ANCHORS_INIT;
static const uint8_t W3[8] = NT_BC6H_WEIGHTS3_INIT;
static const uint8_t W4[16] = NT_BC6H_WEIGHTS4_INIT;

/* ---- bit access (block bit k = bit k % 8 of byte k / 8) ------------------------------ */
static int get_bit(const uint8_t *b, int k) { return (b[k >> 3] >> (k & 7)) & 1; }
static void set_bit(uint8_t *b, int k, int v)
{
    if (v) b[k >> 3] |= (uint8_t)(1u << (k & 7));
}
static int get_bits(const uint8_t *b, int k, int n)
{
    int v = 0;
    for (int i = 0; i < n; ++i) v |= get_bit(b, k + i) << i;
    return v;
}

static int sign_extend(int v, int bits)
{
    if (bits >= 32) return v;
    const unsigned m = 1u << (bits - 1);
    const unsigned u = (unsigned)v & ((1u << bits) - 1u);
    return (int)((u ^ m) - m);
}

/* Unquantize an endpoint to the 16-bit interpolation domain (format specification). */
static int unquantize(int comp, int bits, int is_signed)
{
    if (!is_signed) {
        if (bits >= 15) return comp;
        if (comp == 0) return 0;
        if (comp == (1 << bits) - 1) return 0xFFFF;
        return ((comp << 16) + 0x8000) >> bits;
    }
    if (bits >= 16) return comp;
    int s = 0;
    if (comp < 0) {
        s = 1;
        comp = -comp;
    }
    int unq;
    if (comp == 0)
        unq = 0;
    else if (comp >= (1 << (bits - 1)) - 1)
        unq = 0x7FFF;
    else
        unq = ((comp << 15) + 0x4000) >> (bits - 1);
    return s ? -unq : unq;
}

static uint16_t finish_unquantize(int comp, int is_signed)
{
    if (!is_signed) return (uint16_t)((comp * 31) >> 6);
    comp = comp < 0 ? -(((-comp) * 31) >> 5) : (comp * 31) >> 5;
    uint16_t s = 0;
    if (comp < 0) {
        s = 0x8000;
        comp = -comp;
    }
    return (uint16_t)(s | comp);
}

int nto_bc6h_mode_index(const uint8_t block[16])
{
    const int m2 = get_bits(block, 0, 2);
    if (m2 < 2) return m2;
    const int m5 = get_bits(block, 0, 5);
    for (int i = 2; i < NT_BC6H_NUM_MODES; ++i)
        if (MODES[i].mode_value == m5) return i;
    return -1;
}

void nto_bc6h_decode_block(const uint8_t block[16], int is_signed, uint16_t out[48])
{
    const int mi = nto_bc6h_mode_index(block);
    if (mi < 0) { /* reserved mode: the format decodes such blocks to zero */
        memset(out, 0, 48 * sizeof(uint16_t));
        return;
    }
    const NtBc6hMode *M = &MODES[mi];
    int e[4][3] = {{0}};
    int d = 0;
    for (int k = 0; k < M->header_bits; ++k) {
        const int f = LAYOUT[mi][k] >> 4, bit = LAYOUT[mi][k] & 15;
        const int v = get_bit(block, k);
        if (f < 12)
            e[f / 3][f % 3] |= v << bit;
        else if (f == NT_BC6H_FIELD_D)
            d |= v << bit;
    }
    const int ne = 2 * M->regions, epb = M->endpoint_bits;
    for (int c = 0; c < 3; ++c) {
        if (is_signed) e[0][c] = sign_extend(e[0][c], epb);
        if (is_signed || M->transformed)
            for (int i = 1; i < ne; ++i) e[i][c] = sign_extend(e[i][c], M->transformed ? M->delta_bits[c] : epb);
        if (M->transformed)
            for (int i = 1; i < ne; ++i) {
                e[i][c] = (e[0][c] + e[i][c]) & ((1 << epb) - 1);
                if (is_signed) e[i][c] = sign_extend(e[i][c], epb);
            }
        for (int i = 0; i < ne; ++i) e[i][c] = unquantize(e[i][c], epb, is_signed);
    }
    const int ib = M->regions == 2 ? 3 : 4;
    int pos = M->header_bits;
    for (int px = 0; px < 16; ++px) {
        const int anchor = px == 0 || (M->regions == 2 && px == ANCHORS[d]);
        const int nb = ib - anchor;
        const int idx = get_bits(block, pos, nb);
        pos += nb;
        const int r = M->regions == 2 ? (PARTS[d] >> px) & 1 : 0;
        const int w = ib == 3 ? W3[idx] : W4[idx];
        for (int c = 0; c < 3; ++c) {
            const int a = e[2 * r][c], b = e[2 * r + 1][c];
            out[px * 3 + c] = finish_unquantize((a * (64 - w) + b * w + 32) >> 6, is_signed);
        }
    }
}

/* ---- encoder -------------------------------------------------------------------------- */

/* non-negative half (negatives and NaN clamp to 0, infinities to 0x7BFF) -> the unsigned
 * interpolation domain: the exact inverse of the format's final scale (x * 31) >> 6 */
static int to_domain(uint16_t h)
{
    int m = (h & 0x8000) ? 0 : h;
    if (m > 0x7C00) m = 0;      /* NaN */
    if (m > 0x7BFF) m = 0x7BFF; /* +inf */
    return (m * 64 + 30) / 31;
}

/* nearest unsigned endpoint of `bits` bits for domain value x (ties: the smaller one) */
static int quantize_unsigned(int x, int bits)
{
    if (bits >= 16) return x;
    const int qmax = (1 << bits) - 1;
    int q = (int)(((int64_t)x << bits) >> 16);
    if (q > qmax) q = qmax;
    if (q < qmax) {
        const int d0 = abs(unquantize(q, bits, 0) - x);
        const int d1 = abs(unquantize(q + 1, bits, 0) - x);
        if (d1 < d0) q = q + 1;
    }
    return q;
}

static void fit_endpoints(const int x[16][3], uint16_t mask, int want, int A[3], int B[3])
{
    int lo[3] = {65535, 65535, 65535}, hi[3] = {0, 0, 0};
    int64_t sum[3] = {0, 0, 0};
    int n = 0;
    for (int px = 0; px < 16; ++px) {
        if ((int)((mask >> px) & 1) != want) continue;
        ++n;
        for (int c = 0; c < 3; ++c) {
            if (x[px][c] < lo[c]) lo[c] = x[px][c];
            if (x[px][c] > hi[c]) hi[c] = x[px][c];
            sum[c] += x[px][c];
        }
    }
    if (n == 0) {
        for (int c = 0; c < 3; ++c) A[c] = B[c] = 0;
        return;
    }
    int k = 0;
    for (int c = 1; c < 3; ++c)
        if (hi[c] - lo[c] > hi[k] - lo[k]) k = c;
    for (int c = 0; c < 3; ++c) {
        int64_t cov = 0;
        if (c != k) {
            int64_t sxy = 0;
            for (int px = 0; px < 16; ++px)
                if ((int)((mask >> px) & 1) == want) sxy += (int64_t)x[px][c] * x[px][k];
            cov = (int64_t)n * sxy - sum[c] * sum[k];
        }
        if (cov < 0) {
            A[c] = hi[c];
            B[c] = lo[c];
        } else {
            A[c] = lo[c];
            B[c] = hi[c];
        }
    }
}

/* Palette index nearest to the projection of x onto the segment a -> b: t = 64 dot / |b-a|^2
 * (int64 sums converted to float with round-to-nearest, one correctly rounded division),
 * then the number of weight midpoints below t.  Only indices k0 - 1 .. k0 + 1 are then
 * evaluated exactly. */
static int project_index(const int x[3], const int a[3], const int b[3], int ib)
{
    int64_t dot = 0, len2 = 0;
    for (int c = 0; c < 3; ++c) {
        const int64_t d = (int64_t)b[c] - a[c];
        dot += ((int64_t)x[c] - a[c]) * d;
        len2 += d * d;
    }
    if (len2 == 0) return 0;
    const float t = ((float)dot * 64.0f) / (float)len2;
    const int ni = 1 << ib;
    int k0 = 0;
    for (int k = 1; k < ni; ++k) {
        const float mid = 0.5f * (float)((ib == 3 ? W3[k - 1] + W3[k] : W4[k - 1] + W4[k]));
        if (t > mid) k0 = k;
    }
    return k0;
}

static int64_t try_mode(int mi, int part, const int x[16][3], int A[2][3], int B[2][3], uint8_t out[16])
{
    const NtBc6hMode *M = &MODES[mi];
    const int regions = M->regions, epb = M->endpoint_bits, ib = regions == 2 ? 3 : 4;
    const int ni = 1 << ib;
    const uint16_t mask = regions == 2 ? PARTS[part] : 0;
    int q[2][2][3];  /* [region][endpoint][channel] */
    int u[2][2][3];
    for (int r = 0; r < regions; ++r)
        for (int c = 0; c < 3; ++c) {
            q[r][0][c] = quantize_unsigned(A[r][c], epb);
            q[r][1][c] = quantize_unsigned(B[r][c], epb);
        }
    int idx[16];
    int64_t err = 0;
    for (int pass = 0; pass < 2; ++pass) {
        for (int r = 0; r < regions; ++r)
            for (int i = 0; i < 2; ++i)
                for (int c = 0; c < 3; ++c) u[r][i][c] = unquantize(q[r][i][c], epb, 0);
        err = 0;
        for (int px = 0; px < 16; ++px) {
            const int r = (mask >> px) & 1;
            const int k0 = project_index(x[px], u[r][0], u[r][1], ib);
            int64_t best = INT64_MAX;
            int bi = 0;
            for (int k = k0 - 1; k <= k0 + 1; ++k) {
                if (k < 0 || k >= ni) continue;
                const int w = ib == 3 ? W3[k] : W4[k];
                int64_t dsum = 0;
                for (int c = 0; c < 3; ++c) {
                    const int v = (u[r][0][c] * (64 - w) + u[r][1][c] * w + 32) >> 6;
                    const int64_t dd = (int64_t)(x[px][c] - v);
                    dsum += dd * dd;
                }
                if (dsum < best) {
                    best = dsum;
                    bi = k;
                }
            }
            idx[px] = bi;
            err += best;
        }
        if (pass == 1) break;
        /* anchors must have their top index bit clear: swap that region's endpoints */
        int swapped = 0;
        for (int r = 0; r < regions; ++r) {
            const int ap = r == 0 ? 0 : ANCHORS[part];
            if (idx[ap] >= ni / 2) {
                for (int c = 0; c < 3; ++c) {
                    const int t = q[r][0][c];
                    q[r][0][c] = q[r][1][c];
                    q[r][1][c] = t;
                }
                swapped = 1;
            }
        }
        if (!swapped) break;
    }
    for (int r = 0; r < regions; ++r)
        if (idx[r == 0 ? 0 : ANCHORS[part]] >= ni / 2) return -1; /* cannot happen: swap is exact */
    /* stored endpoint values */
    int e[4][3];
    for (int r = 0; r < regions; ++r)
        for (int i = 0; i < 2; ++i)
            for (int c = 0; c < 3; ++c) e[2 * r + i][c] = q[r][i][c];
    if (M->transformed) {
        for (int i = 1; i < 2 * regions; ++i)
            for (int c = 0; c < 3; ++c) {
                const int dlt = e[i][c] - e[0][c];
                const int db = M->delta_bits[c];
                if (dlt < -(1 << (db - 1)) || dlt > (1 << (db - 1)) - 1) return -1;
                e[i][c] = dlt;
            }
    }
    memset(out, 0, 16);
    for (int k = 0; k < M->header_bits; ++k) {
        const int f = LAYOUT[mi][k] >> 4, bit = LAYOUT[mi][k] & 15;
        int v;
        if (f < 12)
            v = ((unsigned)e[f / 3][f % 3] >> bit) & 1;
        else if (f == NT_BC6H_FIELD_D)
            v = (part >> bit) & 1;
        else
            v = (M->mode_value >> bit) & 1;
        set_bit(out, k, v);
    }
    int pos = M->header_bits;
    for (int px = 0; px < 16; ++px) {
        const int anchor = px == 0 || (regions == 2 && px == ANCHORS[part]);
        const int nb = ib - anchor;
        for (int b = 0; b < nb; ++b) set_bit(out, pos + b, (idx[px] >> b) & 1);
        pos += nb;
    }
    return err;
}

void nto_bc6h_encode_block(const uint16_t texels[48], uint8_t out[16])
{
    int x[16][3];
    for (int px = 0; px < 16; ++px)
        for (int c = 0; c < 3; ++c) x[px][c] = to_domain(texels[px * 3 + c]);
    int64_t best = INT64_MAX;
    uint8_t cand[16];
    int A[2][3], B[2][3];
    /* one region: modes 11..14 */
    fit_endpoints(x, 0, 0, A[0], B[0]);
    for (int mi = 10; mi < 14; ++mi) {
        const int64_t e = try_mode(mi, 0, x, A, B, cand);
        if (e >= 0 && e < best) {
            best = e;
            memcpy(out, cand, 16);
        }
    }
    /* two regions: best partition by box extent, modes 1..10 */
    int bp = 0;
    int64_t bcost = INT64_MAX;
    for (int p = 0; p < 32; ++p) {
        int64_t cost = 0;
        for (int r = 0; r < 2; ++r) {
            int lo[3] = {65535, 65535, 65535}, hi[3] = {0, 0, 0};
            for (int px = 0; px < 16; ++px) {
                if ((int)((PARTS[p] >> px) & 1) != r) continue;
                for (int c = 0; c < 3; ++c) {
                    if (x[px][c] < lo[c]) lo[c] = x[px][c];
                    if (x[px][c] > hi[c]) hi[c] = x[px][c];
                }
            }
            for (int c = 0; c < 3; ++c) {
                const int64_t ext = (int64_t)hi[c] - lo[c];
                cost += ext * ext;
            }
        }
        if (cost < bcost) {
            bcost = cost;
            bp = p;
        }
    }
    fit_endpoints(x, PARTS[bp], 0, A[0], B[0]);
    fit_endpoints(x, PARTS[bp], 1, A[1], B[1]);
    for (int mi = 0; mi < 10; ++mi) {
        const int64_t e = try_mode(mi, bp, x, A, B, cand);
        if (e >= 0 && e < best) {
            best = e;
            memcpy(out, cand, 16);
        }
    }
    if (best == INT64_MAX) memset(out, 0, 16); /* unreachable: mode 11 always fits */
}

/* ---- surfaces ------------------------------------------------------------------------- */

static uint16_t add_bias(uint16_t h, float bias)
{
    return nto_f2h(nto_h2f(h) + bias);
}

void nto_bc6h_encode_surface(const uint16_t *data, int32_t w, int32_t h, int32_t channels,
                             int64_t cstride, int64_t rstride, int64_t tstride, float bias,
                             uint8_t *blocks, int32_t threads)
{
    const int bw = (w + 3) / 4, bh = (h + 3) / 4, nt = (channels + 2) / 3;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
#endif
    for (int64_t b = 0; b < (int64_t)nt * bh * bw; ++b) {
        const int t = (int)(b / ((int64_t)bh * bw));
        const int by = (int)((b / bw) % bh), bx = (int)(b % bw);
        uint16_t tex[48];
        for (int px = 0; px < 16; ++px) {
            int y = by * 4 + px / 4, xx = bx * 4 + px % 4;
            if (y >= h) y = h - 1; /* edge replication for partial blocks */
            if (xx >= w) xx = w - 1;
            for (int c = 0; c < 3; ++c) {
                const int ch = t * 3 + c;
                tex[px * 3 + c] = ch < channels ? add_bias(data[ch * cstride + y * rstride + xx * tstride], bias)
                                                : nto_f2h(bias);
            }
        }
        nto_bc6h_encode_block(tex, blocks + b * 16);
    }
    (void)threads;
}

void nto_bc6h_decode_surface(const uint8_t *blocks, int32_t w, int32_t h, int32_t channels,
                             int64_t cstride, int64_t rstride, int64_t tstride, float bias,
                             uint16_t *data, int32_t threads)
{
    const int bw = (w + 3) / 4, bh = (h + 3) / 4, nt = (channels + 2) / 3;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
#endif
    for (int64_t b = 0; b < (int64_t)nt * bh * bw; ++b) {
        const int t = (int)(b / ((int64_t)bh * bw));
        const int by = (int)((b / bw) % bh), bx = (int)(b % bw);
        uint16_t tex[48];
        nto_bc6h_decode_block(blocks + b * 16, 0, tex);
        for (int px = 0; px < 16; ++px) {
            const int y = by * 4 + px / 4, xx = bx * 4 + px % 4;
            if (y >= h || xx >= w) continue;
            for (int c = 0; c < 3; ++c) {
                const int ch = t * 3 + c;
                if (ch < channels) data[ch * cstride + y * rstride + xx * tstride] = nto_f2h(nto_h2f(tex[px * 3 + c]) - bias);
            }
        }
    }
    (void)threads;
}

/* ---- float BC6 block records <-> BC6H blocks ----------------------------------------------
 *
 * Bridge between the reference's float BC6 block records (train.cu:161-212: per channel
 * triple of a 4x4 block 32 floats, endpoints [region][endpoint][xyz] at 0..11, pixel
 * indices at 12..27, partition and mode as int32 bits at 28 and 29) and the integer BC6H
 * bitstream above.  The reference decodes ebar = (31744 e + 32768) 2^-b and
 * y = ebar0 + 8 (ebar1 - ebar0) x, y standing for a half-float bit pattern; the format reaches
 * the half bits (v * 31) >> 6 from unquantized endpoints u and weights w / 64.  Taking
 * ebar = 31 u / 64 and x = w / 512 maps one onto the other (the reference has no such bridge;
 * its block-feature path starts from and ends in float records).
 *
 * from BC6H: e = (31 u 2^b / 64 - 32768) / 31744 (double, one rounding, then float),
 *   x = w / 512; two-region modes keep their partition and mode (the reference's ten mode
 *   precisions are those of BC6H modes 1-10, train.cu:31-34); one-region modes (11-14) give
 *   both regions the same endpoints, partition 0 and record mode 0 (10 bits); reserved modes
 *   give records that decode to zero (e = -32768 / 31744, x = 0).
 * to BC6H: endpoint targets U = round(64 ebar / 31) in [0, 65535]; texel targets
 *   T = round(64 U0 + (U1 - U0) 512 x) in [0, 64 * 65535] (units of 1/64); candidates: the
 *   record's mode, the other two-region modes in order, then the one-region modes 11-14 when
 *   both regions' targets are equal; per candidate the endpoints are quantized to the mode
 *   precision (nearest unquantized value), each texel takes the palette index with the
 *   smallest sum_c (T_c - 64 v_c)^2 (ties: lower index), a region whose anchor index has its
 *   top bit set swaps its endpoints and flips its indices (w(n-1-i) = 64 - w(i): the decoded
 *   values do not change), transformed deltas must fit; the smallest error wins (ties: the
 *   earlier candidate).  A record made from a block therefore returns a block that decodes to
 *   the same texels.
 */
#define BC6F_FLOATS 32

static float bc6f_ebar(float e, int b) /* train.cu:161-167 */
{
    const float scale = (31.f / 64.f) * 65536.f;
    return ldexpf(scale * e + 32768.f, -b);
}

static float bc6f_endpoint_param(int u, int b)
{
    return (float)(((double)(31 * u) * ldexp(1.0, b - 6) - 32768.0) / 31744.0);
}

static const int BC6F_MODE_BITS[10] = {10, 7, 11, 11, 11, 9, 8, 8, 8, 6}; /* train.cu:31-34 */

static int bc6f_mode_of(const float rec[BC6F_FLOATS])
{
    int32_t m;
    memcpy(&m, &rec[29], 4);
    return (uint32_t)m > 9u ? 0 : m;
}

void nto_bc6f_from_bc6h_block(const uint8_t block[16], float rec[BC6F_FLOATS])
{
    memset(rec, 0, BC6F_FLOATS * sizeof(float));
    int32_t part = 0, mode = 0;
    const int mi = nto_bc6h_mode_index(block);
    if (mi < 0) {
        for (int k = 0; k < 12; ++k) rec[k] = bc6f_endpoint_param(0, 10);
    } else {
        const NtBc6hMode *M = &MODES[mi];
        int e[4][3] = {{0}};
        int d = 0;
        for (int k = 0; k < M->header_bits; ++k) {
            const int f = LAYOUT[mi][k] >> 4, bit = LAYOUT[mi][k] & 15;
            const int v = get_bit(block, k);
            if (f < 12)
                e[f / 3][f % 3] |= v << bit;
            else if (f == NT_BC6H_FIELD_D)
                d |= v << bit;
        }
        const int ne = 2 * M->regions, epb = M->endpoint_bits;
        for (int c = 0; c < 3; ++c) {
            if (M->transformed)
                for (int i = 1; i < ne; ++i) e[i][c] = (e[0][c] + sign_extend(e[i][c], M->delta_bits[c])) & ((1 << epb) - 1);
            for (int i = 0; i < ne; ++i) e[i][c] = unquantize(e[i][c], epb, 0);
        }
        const int two = M->regions == 2;
        const int b = two ? epb : 10;
        if (two) {
            part = d;
            mode = mi;
        }
        for (int r = 0; r < 2; ++r)
            for (int i = 0; i < 2; ++i)
                for (int c = 0; c < 3; ++c) rec[6 * r + 3 * i + c] = bc6f_endpoint_param(e[two ? 2 * r + i : i][c], b);
        const int ib = two ? 3 : 4;
        int pos = M->header_bits;
        for (int px = 0; px < 16; ++px) {
            const int nb = ib - (px == 0 || (two && px == ANCHORS[d]));
            const int idx = get_bits(block, pos, nb);
            pos += nb;
            rec[12 + px] = (float)(ib == 3 ? W3[idx] : W4[idx]) / 512.f;
        }
    }
    memcpy(&rec[28], &part, 4);
    memcpy(&rec[29], &mode, 4);
}

/* Candidate mi for the record targets; returns the error or -1 when the deltas do not fit. */
static int64_t bc6f_try_mode(int mi, int part, const int U[2][2][3], const int64_t T[16][3], uint8_t out[16])
{
    const NtBc6hMode *M = &MODES[mi];
    const int regions = M->regions, epb = M->endpoint_bits, ib = regions == 2 ? 3 : 4;
    const int ni = 1 << ib;
    const uint16_t mask = regions == 2 ? PARTS[part] : 0;
    int q[2][2][3], u[2][2][3];
    for (int r = 0; r < 2; ++r)
        for (int i = 0; i < 2; ++i)
            for (int c = 0; c < 3; ++c) {
                q[r][i][c] = quantize_unsigned(U[r][i][c], epb);
                u[r][i][c] = unquantize(q[r][i][c], epb, 0);
            }
    int idx[16];
    int64_t err = 0;
    for (int px = 0; px < 16; ++px) {
        const int r = (mask >> px) & 1;
        int64_t best = INT64_MAX;
        int bi = 0;
        for (int k = 0; k < ni; ++k) {
            const int w = ib == 3 ? W3[k] : W4[k];
            int64_t dsum = 0;
            for (int c = 0; c < 3; ++c) {
                const int v = (u[r][0][c] * (64 - w) + u[r][1][c] * w + 32) >> 6;
                const int64_t dd = T[px][c] - 64 * (int64_t)v;
                dsum += dd * dd;
            }
            if (dsum < best) {
                best = dsum;
                bi = k;
            }
        }
        idx[px] = bi;
        err += best;
    }
    for (int r = 0; r < regions; ++r) {
        const int ap = r == 0 ? 0 : ANCHORS[part];
        if (idx[ap] < ni / 2) continue;
        for (int c = 0; c < 3; ++c) {
            const int t = q[r][0][c];
            q[r][0][c] = q[r][1][c];
            q[r][1][c] = t;
        }
        for (int px = 0; px < 16; ++px)
            if ((int)((mask >> px) & 1) == r) idx[px] = ni - 1 - idx[px];
    }
    int e[4][3];
    for (int r = 0; r < 2; ++r)
        for (int i = 0; i < 2; ++i)
            for (int c = 0; c < 3; ++c) e[2 * r + i][c] = r < regions ? q[r][i][c] : 0;
    if (M->transformed) {
        /* the decoder adds deltas modulo 2^epb, so the difference is taken modulo 2^epb */
        for (int i = 1; i < 2 * regions; ++i)
            for (int c = 0; c < 3; ++c) {
                const int dlt = sign_extend(e[i][c] - e[0][c], epb);
                const int db = M->delta_bits[c];
                if (dlt < -(1 << (db - 1)) || dlt > (1 << (db - 1)) - 1) return -1;
                e[i][c] = dlt;
            }
    }
    memset(out, 0, 16);
    for (int k = 0; k < M->header_bits; ++k) {
        const int f = LAYOUT[mi][k] >> 4, bit = LAYOUT[mi][k] & 15;
        int v;
        if (f < 12)
            v = ((unsigned)e[f / 3][f % 3] >> bit) & 1;
        else if (f == NT_BC6H_FIELD_D)
            v = (part >> bit) & 1;
        else
            v = (M->mode_value >> bit) & 1;
        set_bit(out, k, v);
    }
    int pos = M->header_bits;
    for (int px = 0; px < 16; ++px) {
        const int nb = ib - (px == 0 || (regions == 2 && px == ANCHORS[part]));
        for (int b = 0; b < nb; ++b) set_bit(out, pos + b, (idx[px] >> b) & 1);
        pos += nb;
    }
    return err;
}

static double bc6f_clamp(double v, double hi)
{
    return fmin(fmax(v, 0.0), hi); /* NaN -> 0 */
}

void nto_bc6f_to_bc6h_block(const float rec[BC6F_FLOATS], uint8_t out[16])
{
    int32_t part;
    memcpy(&part, &rec[28], 4);
    part &= 31;
    const int own = bc6f_mode_of(rec), b = BC6F_MODE_BITS[own];
    int U[2][2][3];
    for (int r = 0; r < 2; ++r)
        for (int i = 0; i < 2; ++i)
            for (int c = 0; c < 3; ++c) {
                const double t = (double)bc6f_ebar(rec[6 * r + 3 * i + c], b) * 64.0 / 31.0;
                U[r][i][c] = (int)floor(bc6f_clamp(t, 65535.0) + 0.5);
            }
    int64_t T[16][3];
    for (int px = 0; px < 16; ++px) {
        const int r = (PARTS[part] >> px) & 1;
        const double a = 512.0 * (double)rec[12 + px];
        for (int c = 0; c < 3; ++c) {
            const double t = 64.0 * U[r][0][c] + (double)(U[r][1][c] - U[r][0][c]) * a;
            T[px][c] = (int64_t)floor(bc6f_clamp(t, 64.0 * 65535.0) + 0.5);
        }
    }
    int64_t best = INT64_MAX;
    uint8_t cand[16];
    for (int k = 0; k < 14; ++k) {
        int mi;
        if (k == 0)
            mi = own;
        else if (k <= 9)
            mi = k - 1 < own ? k - 1 : k;
        else
            mi = k;
        if (mi >= 10 && memcmp(U[0], U[1], sizeof U[0]) != 0) break;
        const int64_t e = bc6f_try_mode(mi, mi < 10 ? part : 0, U, T, cand);
        if (e >= 0 && e < best) {
            best = e;
            memcpy(out, cand, 16);
        }
    }
    if (best == INT64_MAX) memset(out, 0, 16); /* unreachable: mode 10 (6 bits) always fits */
}

/* records [block row][block column][triple][32] <-> blocks [triple][block row][block column] */
void nto_bc6f_from_bc6h_surface(const uint8_t *blocks, int32_t w, int32_t h, int32_t channels, float *records)
{
    const int bw = w / 4, bh = h / 4, nt = (channels + 2) / 3;
    for (int t = 0; t < nt; ++t)
        for (int by = 0; by < bh; ++by)
            for (int bx = 0; bx < bw; ++bx)
                nto_bc6f_from_bc6h_block(blocks + (((int64_t)t * bh + by) * bw + bx) * 16,
                                         records + (((int64_t)by * bw + bx) * nt + t) * BC6F_FLOATS);
}

void nto_bc6f_to_bc6h_surface(const float *records, int32_t w, int32_t h, int32_t channels, uint8_t *blocks)
{
    const int bw = w / 4, bh = h / 4, nt = (channels + 2) / 3;
    for (int t = 0; t < nt; ++t)
        for (int by = 0; by < bh; ++by)
            for (int bx = 0; bx < bw; ++bx)
                nto_bc6f_to_bc6h_block(records + (((int64_t)by * bw + bx) * nt + t) * BC6F_FLOATS,
                                       blocks + (((int64_t)t * bh + by) * bw + bx) * 16);
}

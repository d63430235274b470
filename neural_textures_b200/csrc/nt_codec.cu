// nt_codec.cu -- BC6H latent block codec: encode (UF16 of value + bias) and decode.
//
// The reference (mavenkim2/neural_textures) has a differentiable float decode of BC6-like
// blocks (train.cu:161-202) over the format's 2-region partition table (train.cu:20-34) and
// no integer bitstream.  This file implements the published BC6H bitstream (all 14 modes on
// decode; modes 1-10 with the best-scoring partition and modes 11-14 on encode) with a
// deterministic integer encoder; the CPU oracle (oracle/nt_oracle_codec.c) restates the same
// algorithm and the two must agree bit for bit.  Latent planes are grouped in channel
// triples (the reference's latent unit is a float3 feature, train.h:39, :59); signed
// latents are stored as UF16 of (value + bias) because BC6H interpolates half-float bit
// patterns, which is meaningful only within one sign.
//
// Decode: one thread per 4x4 block; a warp covers 32 consecutive blocks of a block row, so
// every texel row of a plane is written as 256 contiguous bytes, and the 16-byte blocks move
// as one vector access each.  Encode: 16 lanes per block, one texel each (the search's
// per-texel work in parallel, its sums and extents by shuffles).
#include <cuda_fp16.h>
#include <stdint.h>

#include "neural_textures/bc6h_format.h"
#include "nt_bc6f.cuh"
#include "nt_bc6h_unpack.cuh"
#include "nt_capi.h"
#include "nt_kernels.cuh"

namespace nt {

__device__ const NtBc6hMode c_modes[NT_BC6H_NUM_MODES] = NT_BC6H_MODES_INIT;
__device__ const uint8_t c_layout[NT_BC6H_NUM_MODES][82] = NT_BC6H_LAYOUT_INIT;
__device__ const uint16_t c_parts[32] = NT_BC6H_PARTITIONS_INIT;
__device__ const uint8_t c_anchors[32] = NT_BC6H_ANCHORS_INIT;

struct Block128 {
    uint32_t w[4];
    __device__ __forceinline__ int bit(int k) const { return (w[k >> 5] >> (k & 31)) & 1; }
    __device__ __forceinline__ int bits(int k, int n) const
    {
        // n <= 4 and the field never straddles more than two words
        const int wi = k >> 5, sh = k & 31;
        uint64_t v = w[wi];
        if (wi < 3) v |= (uint64_t)w[wi + 1] << 32;
        return (int)((v >> sh) & ((1u << n) - 1u));
    }
    __device__ __forceinline__ void set(int k, int v)
    {
        if (v) w[k >> 5] |= 1u << (k & 31);
    }
};

__device__ __forceinline__ int sign_extend(int v, int bits)
{
    const unsigned m = 1u << (bits - 1);
    const unsigned u = (unsigned)v & ((1u << bits) - 1u);
    return (int)((u ^ m) - m);
}

__device__ __forceinline__ int unquantize(int comp, int bits, bool is_signed)
{
    if (!is_signed) {
        if (bits >= 15) return comp;
        if (comp == 0) return 0;
        if (comp == (1 << bits) - 1) return 0xFFFF;
        return ((comp << 16) + 0x8000) >> bits;
    }
    if (bits >= 16) return comp;
    const bool s = comp < 0;
    if (s) comp = -comp;
    int unq;
    if (comp == 0)
        unq = 0;
    else if (comp >= (1 << (bits - 1)) - 1)
        unq = 0x7FFF;
    else
        unq = ((comp << 15) + 0x4000) >> (bits - 1);
    return s ? -unq : unq;
}

__device__ __forceinline__ uint16_t finish_unquantize(int comp, bool is_signed)
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

// Mode index of each 5-bit mode value (-1: reserved), built from the mode table.
struct ModeOf5 {
    int8_t v[32];
};
constexpr ModeOf5 make_mode_of5()
{
    constexpr NtBc6hMode m[NT_BC6H_NUM_MODES] = NT_BC6H_MODES_INIT;
    ModeOf5 t{};
    for (int i = 0; i < 32; ++i) t.v[i] = -1;
    for (int i = 2; i < NT_BC6H_NUM_MODES; ++i) t.v[m[i].mode_value & 31] = (int8_t)i;
    return t;
}
__device__ const ModeOf5 c_mode_of5 = make_mode_of5();

__device__ __forceinline__ int mode_index(const Block128 &b)
{
    const int m2 = b.w[0] & 3;
    return m2 < 2 ? m2 : c_mode_of5.v[b.w[0] & 31];
}

// Interpolation weight of index i: round(64 i / 7) for 3-bit and round(64 i / 15) for 4-bit
// indices, the BC6H weight tables (equal to NT_BC6H_WEIGHTS3_INIT / NT_BC6H_WEIGHTS4_INIT
// for every index; tests/test_codec_cpu.py checks the tables against the same formula).
__device__ __forceinline__ int bc6h_weight(int idx, bool three_bit)
{
    return three_bit ? (128 * idx + 7) / 14 : (128 * idx + 15) / 30;
}

// The block's endpoints, unquantised (e[2 r + i][c]: region r, endpoint i), its mode and its
// partition; false for a reserved mode.
__device__ __forceinline__ bool decode_endpoints(const Block128 &b, bool is_signed, int (&e)[4][3], NtBc6hMode &M,
                                                 int &d)
{
    const int mi = mode_index(b);
    if (mi < 0) return false;
    M = c_modes[mi];
    const uint64_t lo = (uint64_t)b.w[0] | ((uint64_t)b.w[1] << 32), hi = (uint64_t)b.w[2] | ((uint64_t)b.w[3] << 32);
    d = 0;
    bc6h_unpack_header(mi, lo, hi, e, d);
    const int ne = 2 * M.regions, epb = M.endpoint_bits;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        if (is_signed) e[0][c] = sign_extend(e[0][c], epb);
#pragma unroll
        for (int i = 1; i < 4; ++i) {
            if (i >= ne) break;
            if (is_signed || M.transformed) e[i][c] = sign_extend(e[i][c], M.transformed ? M.delta_bits[c] : epb);
            if (M.transformed) {
                e[i][c] = (e[0][c] + e[i][c]) & ((1 << epb) - 1);
                if (is_signed) e[i][c] = sign_extend(e[i][c], epb);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (i < ne) e[i][c] = unquantize(e[i][c], epb, is_signed);
    }
    return true;
}

__device__ __forceinline__ void decode_block(const Block128 &b, bool is_signed, uint16_t out[48])
{
    int e[4][3];
    NtBc6hMode M;
    int d = 0;
    if (!decode_endpoints(b, is_signed, e, M, d)) {
#pragma unroll
        for (int i = 0; i < 48; ++i) out[i] = 0;
        return;
    }
    const uint64_t hi = (uint64_t)b.w[2] | ((uint64_t)b.w[3] << 32);
    const bool two = M.regions == 2;
    const int ib = two ? 3 : 4;
    const int anchor1 = two ? c_anchors[d] : -1;
    const uint32_t pmask = two ? c_parts[d] : 0u;
    // the index bits follow the header (82 or 65 bits, so all within the high word)
    uint64_t s = hi >> (M.header_bits - 64);
    // a (64 - w) + b w = 64 a + (b - a) w, and an arithmetic shift floors, so
    // (a (64 - w) + b w + 32) >> 6 == a + (((b - a) w + 32) >> 6) exactly
    int dl[2][3];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        dl[0][c] = e[1][c] - e[0][c];
        dl[1][c] = e[3][c] - e[2][c];
    }
#pragma unroll
    for (int px = 0; px < 16; ++px) {
        const int nb = ib - ((px == 0 || px == anchor1) ? 1 : 0);
        const int idx = (int)(s & ((1u << nb) - 1u));
        s >>= nb;
        const int w = bc6h_weight(idx, two);
        const int r = (pmask >> px) & 1;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const int a = r ? e[2][c] : e[0][c], dd = r ? dl[1][c] : dl[0][c];
            out[px * 3 + c] = finish_unquantize(a + ((dd * w + 32) >> 6), is_signed);
        }
    }
}

// UF16 block -> its 16 texels' three channels minus `bias`, as fp16, through a palette: the
// interpolated colour of each index value is formed once (16 entries: index i of a one-region
// block, or 8 r + i for region r of a two-region block), stored at pal[k * stride] (shared
// memory private to the thread: (c0, c1) in .x, (c2, 0) in .y) and looked up per texel.  The
// same operations as decode_block followed by the bias step of bc6h_decode_kernel, evaluated
// per palette entry instead of per texel, so the texels are bit-identical.
template <int kStride>
__device__ __forceinline__ void decode_block_palette(const Block128 &b, float bias, uint2 *pal, uint2 (&tx)[16])
{
    const auto entry = [&](int v0, int v1, int v2) {
        const float2 f01 = __half22float2(__halves2half2(__ushort_as_half((uint16_t)v0), __ushort_as_half((uint16_t)v1)));
        const __half2 o01 = __floats2half2_rn(f01.x - bias, f01.y - bias);
        const __half o2 = __float2half_rn(__half2float(__ushort_as_half((uint16_t)v2)) - bias);
        return make_uint2(*reinterpret_cast<const uint32_t *>(&o01), (uint32_t)__half_as_ushort(o2));
    };
    int e[4][3];
    NtBc6hMode M;
    int d = 0;
    if (!decode_endpoints(b, false, e, M, d)) {  // reserved mode: every texel decodes to 0
        const uint2 z = entry(0, 0, 0);
#pragma unroll
        for (int px = 0; px < 16; ++px) tx[px] = z;
        return;
    }
    const bool two = M.regions == 2;
    int dl[2][3];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        dl[0][c] = e[1][c] - e[0][c];
        dl[1][c] = e[3][c] - e[2][c];
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const int w = two ? bc6h_weight(k & 7, true) : bc6h_weight(k, false);
        const bool r1 = two && k >= 8;
        int v[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const int a = r1 ? e[2][c] : e[0][c], dd = r1 ? dl[1][c] : dl[0][c];
            v[c] = finish_unquantize(a + ((dd * w + 32) >> 6), false);
        }
        pal[k * kStride] = entry(v[0], v[1], v[2]);
    }
    const uint64_t hi = (uint64_t)b.w[2] | ((uint64_t)b.w[3] << 32);
    const int ib = two ? 3 : 4;
    const int anchor1 = two ? c_anchors[d] : -1;
    const uint32_t pmask = two ? c_parts[d] : 0u;
    uint64_t s = hi >> (M.header_bits - 64);
#pragma unroll
    for (int px = 0; px < 16; ++px) {
        const int nb = ib - ((px == 0 || px == anchor1) ? 1 : 0);
        const int idx = (int)(s & ((1u << nb) - 1u));
        s >>= nb;
        const int k = two ? (int)(((pmask >> px) & 1u) << 3) | idx : idx;
        tx[px] = pal[k * kStride];
    }
}

// ---- encoder ---------------------------------------------------------------------------

__device__ __forceinline__ int to_domain(uint16_t h)
{
    int m = (h & 0x8000) ? 0 : h;
    if (m > 0x7C00) m = 0;
    if (m > 0x7BFF) m = 0x7BFF;
    return (m * 64 + 30) / 31;
}

__device__ __forceinline__ int quantize_unsigned(int x, int bits)
{
    if (bits >= 16) return x;
    const int qmax = (1 << bits) - 1;
    int q = (int)(((int64_t)x << bits) >> 16);
    if (q > qmax) q = qmax;
    if (q < qmax) {
        const int d0 = abs(unquantize(q, bits, false) - x);
        const int d1 = abs(unquantize(q + 1, bits, false) - x);
        if (d1 < d0) q = q + 1;
    }
    return q;
}

// Palette index nearest to the projection of x onto a -> b (same arithmetic as the CPU
// oracle: int64 sums, round-to-nearest conversions, one IEEE division).
__device__ __forceinline__ int project_index(const int x[3], const int a[3], const int b[3], int ib)
{
    int64_t dot = 0, len2 = 0;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const int64_t d = (int64_t)b[c] - a[c];
        dot += ((int64_t)x[c] - a[c]) * d;
        len2 += d * d;
    }
    if (len2 == 0) return 0;
    const float t = __fdiv_rn(__fmul_rn(__ll2float_rn(dot), 64.0f), __ll2float_rn(len2));
    // k0 = #{k >= 1 : t > mid_k} with mid_k = (w_{k-1} + w_k) / 2 (increasing in k): start from
    // the nearest weight and step across the exact midpoints, which gives the same count as
    // testing every midpoint
    const int ni = 1 << ib;
    const bool three = ib == 3;
    const float tc = fminf(fmaxf(t, 0.f), 64.f);
    int k0 = (int)(tc * (float)(ni - 1) * (1.f / 64.f) + 0.5f);
    k0 = min(max(k0, 0), ni - 1);
    auto mid = [&](int k) { return 0.5f * (float)(bc6h_weight(k - 1, three) + bc6h_weight(k, three)); };
#pragma unroll 1
    while (k0 < ni - 1 && t > mid(k0 + 1)) ++k0;
#pragma unroll 1
    while (k0 > 0 && !(t > mid(k0))) --k0;
    return k0;
}

// One evaluated candidate: stored endpoints (after the delta transform), indices (4 bits
// each), mode and partition.
struct Cand {
    int e[4][3];
    uint64_t idx;
    int mi, part;
};

// Bitstream of a candidate: header fields through the mode's bit layout, then the indices
// (anchor indices one bit shorter).
__device__ void pack_block(const Cand &cd, Block128 &out)
{
    const int mi = cd.mi, part = cd.part;
    const NtBc6hMode M = c_modes[mi];
    const int regions = M.regions, ib = regions == 2 ? 3 : 4;
    const int anchor1 = regions == 2 ? c_anchors[part] : 0;
    int e[4][3], idx[16];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 3; ++c) e[i][c] = cd.e[i][c];
#pragma unroll
    for (int px = 0; px < 16; ++px) idx[px] = (int)((cd.idx >> (4 * px)) & 15u);
    out.w[0] = out.w[1] = out.w[2] = out.w[3] = 0u;
#pragma unroll 1
    for (int k = 0; k < M.header_bits; ++k) {
        const int ent = c_layout[mi][k];
        const int f = ent >> 4, bit = ent & 15;
        int v = 0;
        if (f < 12) {
#pragma unroll
            for (int qf = 0; qf < 12; ++qf)
                if (qf == f) v = ((unsigned)e[qf / 3][qf % 3] >> bit) & 1;
        } else if (f == NT_BC6H_FIELD_D) {
            v = (part >> bit) & 1;
        } else {
            v = (M.mode_value >> bit) & 1;
        }
        out.set(k, v);
    }
    int pos = M.header_bits;
#pragma unroll
    for (int px = 0; px < 16; ++px) {
        const int nb = ib - ((px == 0 || (regions == 2 && px == anchor1)) ? 1 : 0);
        for (int bb = 0; bb < nb; ++bb) out.set(pos + bb, (idx[px] >> bb) & 1);
        pos += nb;
    }
}

// ---- cooperative encoder: 16 lanes per block, one texel per lane -------------------------
//
// The same search as encode_block (modes 11-14 on the whole block, the partition with the
// smallest summed squared channel extents, modes 1-10 on it; strict improvement keeps the
// first best) with the per-texel work spread over a half warp: each lane projects and scores
// its own texel, integer sums and extents are reduced with shuffles (exact in any order), and
// the per-candidate endpoint work is split across lanes and broadcast.  Bit-identical to
// encode_block.  Shuffles name only the 16 lanes of the block, so the two blocks of a warp may
// take different branches.

struct Grp {
    unsigned mask;  // the block's 16 lanes
    int px;         // this lane's texel (row-major in the 4x4 block)
    int base;       // lane of texel 0
};

__device__ __forceinline__ int grp_min(const Grp &g, int v)
{
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(g.mask, v, o));
    return v;
}
__device__ __forceinline__ int grp_max(const Grp &g, int v)
{
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(g.mask, v, o));
    return v;
}
__device__ __forceinline__ int grp_sum(const Grp &g, int v)
{
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(g.mask, v, o);
    return v;
}
__device__ __forceinline__ long long grp_sum64(const Grp &g, long long v)
{
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(g.mask, v, o);
    return v;
}
__device__ __forceinline__ int grp_at(const Grp &g, int v, int px) { return __shfl_sync(g.mask, v, g.base + px); }

// fit_endpoints over the texels whose partition bit equals `want`.
__device__ __forceinline__ void fit_endpoints_grp(const Grp &g, const int (&x)[3], uint32_t mask, int want, int A[3], int B[3])
{
    const bool mem = (int)((mask >> g.px) & 1) == want;
    const int ones = __popc(mask & 0xFFFFu);
    const int n = want ? ones : 16 - ones;
    int lo[3], hi[3], sum[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        lo[c] = grp_min(g, mem ? x[c] : 65535);
        hi[c] = grp_max(g, mem ? x[c] : 0);
        sum[c] = grp_sum(g, mem ? x[c] : 0);
    }
    if (n == 0) {
#pragma unroll
        for (int c = 0; c < 3; ++c) A[c] = B[c] = 0;
        return;
    }
    int k = 0;
    if (hi[1] - lo[1] > hi[k] - lo[k]) k = 1;
    if (hi[2] - lo[2] > hi[k] - lo[k]) k = 2;
    const int xk = k == 0 ? x[0] : (k == 1 ? x[1] : x[2]);
    const int sk = k == 0 ? sum[0] : (k == 1 ? sum[1] : sum[2]);
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        // every lane takes part in both sums (c == k contributes nothing: cov stays 0)
        const long long sxy = grp_sum64(g, mem && c != k ? (long long)x[c] * xk : 0ll);
        const long long cov = c != k ? (long long)n * sxy - (long long)sum[c] * sk : 0ll;
        if (cov < 0) {
            A[c] = hi[c];
            B[c] = lo[c];
        } else {
            A[c] = lo[c];
            B[c] = hi[c];
        }
    }
}

// try_mode for one candidate; returns the block's squared error (the same on every lane) or
// -1 when the mode cannot hold the endpoints.  e: the stored endpoints; idx: this lane's index.
__device__ __forceinline__ int64_t try_mode_grp(const Grp &g, int mi, int part, const int (&x)[3], const int A[2][3],
                                const int B[2][3], int (&e)[4][3], int &idx)
{
    const NtBc6hMode M = c_modes[mi];
    const int regions = M.regions, epb = M.endpoint_bits, ib = regions == 2 ? 3 : 4;
    const int ni = 1 << ib;
    const uint32_t mask = regions == 2 ? c_parts[part] : 0u;
    const int anchor1 = regions == 2 ? c_anchors[part] : 0;
    // endpoint value v = 6 r + 3 i + c: lane v quantizes it
    int myq = 0;
    if (g.px < 12) {
        const int r = g.px / 6, i = (g.px / 3) & 1, c = g.px % 3;
        const int src = i ? (r ? B[1][c] : B[0][c]) : (r ? A[1][c] : A[0][c]);
        myq = r < regions ? quantize_unsigned(src, epb) : 0;
    }
    int q[2][2][3];
#pragma unroll
    for (int v = 0; v < 12; ++v) q[v / 6][(v / 3) & 1][v % 3] = grp_at(g, myq, v);
    const int r = (mask >> g.px) & 1;
    int64_t err = 0;
    int bi = 0;
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
        int a3[3], b3[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            a3[c] = unquantize(r ? q[1][0][c] : q[0][0][c], epb, false);
            b3[c] = unquantize(r ? q[1][1][c] : q[0][1][c], epb, false);
        }
        const int k0 = project_index(x, a3, b3, ib);
        int64_t best = INT64_MAX;
        bi = 0;
#pragma unroll
        for (int dk = -1; dk <= 1; ++dk) {
            const int kk = k0 + dk;
            if (kk < 0 || kk >= ni) continue;
            const int w = bc6h_weight(kk, ib == 3);
            int64_t dsum = 0;
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const int v = (a3[c] * (64 - w) + b3[c] * w + 32) >> 6;
                const int64_t dd = (int64_t)(x[c] - v);
                dsum += dd * dd;
            }
            if (dsum < best) {
                best = dsum;
                bi = kk;
            }
        }
        err = grp_sum64(g, best);
        if (pass == 1) break;
        bool swapped = false;
        const int a0 = grp_at(g, bi, 0), a1 = grp_at(g, bi, anchor1);
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            if (rr >= regions) break;
            if ((rr == 0 ? a0 : a1) >= ni / 2) {
#pragma unroll
                for (int c = 0; c < 3; ++c) {
                    const int t = q[rr][0][c];
                    q[rr][0][c] = q[rr][1][c];
                    q[rr][1][c] = t;
                }
                swapped = true;
            }
        }
        if (!swapped) break;
    }
#pragma unroll
    for (int rr = 0; rr < 2; ++rr)
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int c = 0; c < 3; ++c) e[2 * rr + i][c] = q[rr][i][c];
    if (M.transformed) {
#pragma unroll
        for (int i = 1; i < 4; ++i) {
            if (i >= 2 * regions) break;
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const int dlt = e[i][c] - e[0][c];
                const int db = M.delta_bits[c];
                if (dlt < -(1 << (db - 1)) || dlt > (1 << (db - 1)) - 1) return -1;
                e[i][c] = dlt;
            }
        }
    }
    idx = bi;
    return err;
}

// pack_block with the header bits spread over the lanes and each lane's index bits placed by
// the lane; the words are OR-reduced, so every lane returns the whole block.
__device__ __forceinline__ void pack_block_grp(const Grp &g, int mi, int part, const int (&e)[4][3], int idx, Block128 &out)
{
    const NtBc6hMode M = c_modes[mi];
    const int regions = M.regions, ib = regions == 2 ? 3 : 4;
    const int anchor1 = regions == 2 ? c_anchors[part] : 0;
    out.w[0] = out.w[1] = out.w[2] = out.w[3] = 0u;
#pragma unroll 1
    for (int k = g.px; k < M.header_bits; k += 16) {
        const int ent = c_layout[mi][k];
        const int f = ent >> 4, bit = ent & 15;
        int v = 0;
        if (f < 12) {
#pragma unroll
            for (int qf = 0; qf < 12; ++qf)
                if (qf == f) v = ((unsigned)e[qf / 3][qf % 3] >> bit) & 1;
        } else if (f == NT_BC6H_FIELD_D) {
            v = (part >> bit) & 1;
        } else {
            v = (M.mode_value >> bit) & 1;
        }
        out.set(k, v);
    }
    // index bits: texel px starts after the header and the indices of texels 0 .. px - 1, the
    // anchors' indices one bit shorter
    const int px = g.px;
    const bool anchor = px == 0 || (regions == 2 && px == anchor1);
    const int nb = ib - (anchor ? 1 : 0);
    const int pos = M.header_bits + px * ib - (px > 0 ? 1 : 0) - (regions == 2 && anchor1 < px ? 1 : 0);
    for (int bb = 0; bb < nb; ++bb) out.set(pos + bb, (idx >> bb) & 1);
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) out.w[w] |= __shfl_xor_sync(g.mask, out.w[w], o);
}

// The first-best partition (strictly smallest summed squared extents of its two regions) over
// the block's texels: lane j scores partitions j and j + 16.
__device__ __forceinline__ int best_partition_grp(const Grp &g, const int (&x)[3])
{
    int64_t pc[2] = {0, 0};
    const uint32_t pm0 = c_parts[g.px], pm1 = c_parts[g.px + 16];
    int lo[2][2][3], hi[2][2][3];  // [candidate][region][channel]
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr)
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                lo[j][rr][c] = 65535;
                hi[j][rr][c] = 0;
            }
#pragma unroll
    for (int t = 0; t < 16; ++t) {
        int xt[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) xt[c] = grp_at(g, x[c], t);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const bool r1 = ((j ? pm1 : pm0) >> t) & 1;
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                if (r1) {
                    lo[j][1][c] = min(lo[j][1][c], xt[c]);
                    hi[j][1][c] = max(hi[j][1][c], xt[c]);
                } else {
                    lo[j][0][c] = min(lo[j][0][c], xt[c]);
                    hi[j][0][c] = max(hi[j][0][c], xt[c]);
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr)
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const int64_t ext = (int64_t)hi[j][rr][c] - lo[j][rr][c];
                pc[j] += ext * ext;
            }
    long long bcost = pc[0];
    int bp = g.px;
    if (pc[1] < bcost) {
        bcost = pc[1];
        bp = g.px + 16;
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
        const long long oc = __shfl_xor_sync(g.mask, bcost, o);
        const int op = __shfl_xor_sync(g.mask, bp, o);
        if (oc < bcost || (oc == bcost && op < bp)) {
            bcost = oc;
            bp = op;
        }
    }
    return bp;
}

// encode_block for the texel x (domain values) of this lane: modes 11-14 (indices 10-13) on
// the whole block, then the best partition and modes 1-10 on it, in one loop (one copy of the
// candidate code).
__device__ void encode_block_grp(const Grp &g, const int (&x)[3], Block128 &out)
{
    int64_t best = INT64_MAX;
    int we[4][3] = {}, wmi = 0, wpart = 0, widx = 0;
    int e[4][3], idx = 0;
    int A[2][3], B[2][3];
    fit_endpoints_grp(g, x, 0u, 0, A[0], B[0]);
#pragma unroll
    for (int c = 0; c < 3; ++c) A[1][c] = B[1][c] = 0;
    int bp = 0;
#pragma unroll 1
    for (int step = 0; step < 14; ++step) {
        if (step == 4) {
            bp = best_partition_grp(g, x);
            fit_endpoints_grp(g, x, c_parts[bp], 0, A[0], B[0]);
            fit_endpoints_grp(g, x, c_parts[bp], 1, A[1], B[1]);
        }
        const int mi = step < 4 ? 10 + step : step - 4, part = step < 4 ? 0 : bp;
        const int64_t er = try_mode_grp(g, mi, part, x, A, B, e, idx);
        if (er >= 0 && er < best) {
            best = er;
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < 3; ++c) we[i][c] = e[i][c];
            wmi = mi;
            wpart = part;
            widx = idx;
        }
    }
    if (best == INT64_MAX) out.w[0] = out.w[1] = out.w[2] = out.w[3] = 0u;
    else pack_block_grp(g, wmi, wpart, we, widx, out);
}

struct CodecLaunch {
    __half *data;
    int32_t w, h, channels;
    int64_t cstride, rstride, tstride;
    float bias;
    uint4 *blocks;
    int32_t bw, bh, ntrip;
    int32_t rows4;  // planar, 8-byte aligned rows of whole blocks: 4 texels move as one uint2
};

constexpr int kEncThreads = 128;  // 8 blocks of 16 lanes per CTA

// grid: (ceil(block columns / 8), block rows, channel triples); 16 lanes per block, one texel
// per lane (texels past the surface edge repeat the last row / column)
__global__ void __launch_bounds__(kEncThreads) bc6h_encode_kernel(const CodecLaunch p)
{
    const int lane = threadIdx.x & 31;
    Grp g;
    g.px = lane & 15;
    g.base = lane & 16;
    g.mask = 0xFFFFu << g.base;
    const int bx = blockIdx.x * (kEncThreads / 16) + (threadIdx.x >> 4), by = blockIdx.y, t = blockIdx.z;
    if (bx >= p.bw) return;  // all 16 lanes of the block
    const int y = min(by * 4 + g.px / 4, p.h - 1), xx = min(bx * 4 + g.px % 4, p.w - 1);
    const uint16_t biash = __half_as_ushort(__float2half_rn(p.bias));
    int x[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const int ch = t * 3 + c;
        uint16_t h = biash;
        if (ch < p.channels)
            h = __half_as_ushort(__float2half_rn(__half2float(p.data[ch * p.cstride + y * p.rstride + xx * p.tstride]) + p.bias));
        x[c] = to_domain(h);
    }
    Block128 out;
    encode_block_grp(g, x, out);
    if (g.px == 0) p.blocks[((int64_t)t * p.bh + by) * p.bw + bx] = make_uint4(out.w[0], out.w[1], out.w[2], out.w[3]);
}

// grid: (ceil(block columns / 128), block rows, channel triples); one thread per block
__global__ void __launch_bounds__(128) bc6h_decode_kernel(const CodecLaunch p)
{
    const int bx = blockIdx.x * blockDim.x + threadIdx.x, by = blockIdx.y, t = blockIdx.z;
    if (bx < p.bw) do {
        const int64_t b = ((int64_t)t * p.bh + by) * p.bw + bx;
        const uint4 raw = p.blocks[b];
        Block128 blk;
        blk.w[0] = raw.x;
        blk.w[1] = raw.y;
        blk.w[2] = raw.z;
        blk.w[3] = raw.w;
        if (p.rows4) {  // whole blocks of a planar surface: palette decode, 4 texels per store
            __shared__ uint2 pal[16 * 128];
            uint2 tx[16];
            decode_block_palette<128>(blk, p.bias, pal + threadIdx.x, tx);
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const int ch = t * 3 + c;
                if (ch >= p.channels) break;
                const uint32_t sel = c == 1 ? 0x7632u : 0x5410u;  // high or low halves
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const uint2 *q = tx + 4 * r;
                    const uint32_t w0 = c == 2 ? __byte_perm(q[0].y, q[1].y, sel) : __byte_perm(q[0].x, q[1].x, sel);
                    const uint32_t w1 = c == 2 ? __byte_perm(q[2].y, q[3].y, sel) : __byte_perm(q[2].x, q[3].x, sel);
                    *reinterpret_cast<uint2 *>(p.data + ch * p.cstride + (int64_t)(by * 4 + r) * p.rstride + bx * 4) =
                        make_uint2(w0, w1);
                }
            }
            continue;
        }
        uint16_t tex[48];
        decode_block(blk, false, tex);
#pragma unroll
        for (int px = 0; px < 16; ++px) {
            const int y = by * 4 + px / 4, xx = bx * 4 + px % 4;
            if (y >= p.h || xx >= p.w) continue;
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const int ch = t * 3 + c;
                if (ch < p.channels)
                    p.data[ch * p.cstride + y * p.rstride + xx * p.tstride] =
                        __float2half_rn(__half2float(__ushort_as_half(tex[px * 3 + c])) - p.bias);
            }
        }
    } while (0);
}

// Raw block decode (no bias, no surface): 48 fp16 bit patterns per block, signed or
// unsigned interpretation (for checking the bitstream against other decoders).
__global__ void bc6h_decode_raw_kernel(const uint4 *blocks, int64_t n, int is_signed, uint16_t *out)
{
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < n; b += (int64_t)gridDim.x * blockDim.x) {
        const uint4 raw = blocks[b];
        Block128 blk;
        blk.w[0] = raw.x;
        blk.w[1] = raw.y;
        blk.w[2] = raw.z;
        blk.w[3] = raw.w;
        uint16_t tex[48];
        decode_block(blk, is_signed != 0, tex);
        for (int i = 0; i < 48; ++i) out[b * 48 + i] = tex[i];
    }
}

static CodecLaunch make_launch(const NtBc6hSurface *s, const void *blocks, float bias)
{
    CodecLaunch L;
    L.data = reinterpret_cast<__half *>(s->data);
    L.w = s->width;
    L.h = s->height;
    L.channels = s->channels;
    L.cstride = s->channel_stride;
    L.rstride = s->row_stride;
    L.tstride = s->texel_stride;
    L.bias = bias;
    L.blocks = reinterpret_cast<uint4 *>(const_cast<void *>(blocks));
    L.bw = (s->width + 3) / 4;
    L.bh = (s->height + 3) / 4;
    L.ntrip = (s->channels + 2) / 3;
    L.rows4 = s->texel_stride == 1 && s->width % 4 == 0 && s->height % 4 == 0 && s->row_stride % 4 == 0 &&
              s->channel_stride % 4 == 0 && (reinterpret_cast<uintptr_t>(s->data) & 7u) == 0;
    return L;
}

cudaError_t launch_bc6h(const NtBc6hSurface *s, const void *blocks, float bias, bool encode, cudaStream_t st)
{
    const CodecLaunch L = make_launch(s, blocks, bias);
    if (L.bh > 65535 || L.ntrip > 65535) return cudaErrorInvalidValue;
    const dim3 grid((L.bw + 127) / 128, L.bh, L.ntrip);
    if (encode)
        bc6h_encode_kernel<<<dim3((L.bw + kEncThreads / 16 - 1) / (kEncThreads / 16), L.bh, L.ntrip), kEncThreads, 0,
                             st>>>(L);
    else
        bc6h_decode_kernel<<<grid, 128, 0, st>>>(L);
    count_launch();
    return cudaGetLastError();
}

// ---- float BC6 block records <-> BC6H blocks ---------------------------------------------
//
// Records are the reference's float BC6 block parameters (train.cu:161-212, the
// BLOCK_FEATURES latents): per channel triple of a 4x4 block 32 floats, endpoints
// [region][endpoint][xyz] at 0..11, pixel indices at 12..27, partition and mode as int32
// bits at 28 and 29.  The reference's float decode ebar = (31744 e + 32768) 2^-b,
// y = ebar0 + 8 (ebar1 - ebar0) x stands for a half-float bit pattern, which the format
// reaches as (v * 31) >> 6 from unquantized endpoints u and weights w / 64; ebar = 31 u / 64
// and x = w / 512 map one onto the other (the reference itself has no such bridge).
//
// from BC6H: e = (31 u 2^b / 64 - 32768) / 31744 (one double rounding, then float),
//   x = w / 512; two-region blocks keep partition and mode (the reference's ten precisions
//   are BC6H modes 1-10, train.cu:31-34); one-region blocks give both regions the same
//   endpoints, partition 0, record mode 0; reserved modes give records that decode to zero.
// to BC6H: endpoint targets U = round(64 ebar / 31) in [0, 65535], texel targets
//   T = round(64 U0 + (U1 - U0) 512 x) in [0, 64 * 65535]; candidates: the record's mode,
//   the other two-region modes, then the one-region modes when both regions' targets agree;
//   endpoints quantized to the nearest unquantized value, per texel the palette index with
//   the smallest sum_c (T_c - 64 v_c)^2 (ties: lower index), anchor fix-up by swapping a
//   region's endpoints and flipping its indices (w(n-1-i) = 64 - w(i) keeps every decoded
//   value), transformed deltas taken modulo 2^bits must fit; smallest error wins (ties: the
//   earlier candidate).  Integer error and exact double targets: bit-identical to the CPU
//   restatement in the oracle.

__device__ __forceinline__ float bc6f_endpoint_param(int u, int b)
{
    const double v = __dmul_rn((double)(31 * u), ldexp(1.0, b - 6));
    return __double2float_rn(__ddiv_rn(__dadd_rn(v, -32768.0), 31744.0));
}

// grid: (ceil(block columns / 128), block rows, channel triples); one thread per record
__global__ void __launch_bounds__(128) bc6f_from_bc6h_kernel(const uint4 *__restrict__ blocks, float *__restrict__ records,
                                                             int bw, int bh, int nt)
{
    const int bx = blockIdx.x * blockDim.x + threadIdx.x, by = blockIdx.y, t = blockIdx.z;
    if (bx >= bw) return;
    const uint4 raw = blocks[((int64_t)t * bh + by) * bw + bx];
    Block128 blk;
    blk.w[0] = raw.x;
    blk.w[1] = raw.y;
    blk.w[2] = raw.z;
    blk.w[3] = raw.w;
    float rec[kBc6fFloats];
#pragma unroll
    for (int k = 0; k < kBc6fFloats; ++k) rec[k] = 0.f;
    int part = 0, mode = 0;
    const int mi = mode_index(blk);
    if (mi < 0) {
#pragma unroll
        for (int k = 0; k < 12; ++k) rec[k] = bc6f_endpoint_param(0, 10);
    } else {
        const NtBc6hMode M = c_modes[mi];
        const uint64_t lo = (uint64_t)blk.w[0] | ((uint64_t)blk.w[1] << 32),
                       hi = (uint64_t)blk.w[2] | ((uint64_t)blk.w[3] << 32);
        int e[4][3];
        int d = 0;
        bc6h_unpack_header(mi, lo, hi, e, d);
        const int ne = 2 * M.regions, epb = M.endpoint_bits;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
#pragma unroll
            for (int i = 1; i < 4; ++i)
                if (i < ne && M.transformed) e[i][c] = (e[0][c] + sign_extend(e[i][c], M.delta_bits[c])) & ((1 << epb) - 1);
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (i < ne) e[i][c] = unquantize(e[i][c], epb, false);
        }
        const bool two = M.regions == 2;
        const int b = two ? epb : 10;
        if (two) {
            part = d;
            mode = mi;
        }
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int c = 0; c < 3; ++c) rec[6 * r + 3 * i + c] = bc6f_endpoint_param(two ? e[2 * r + i][c] : e[i][c], b);
        const int ib = two ? 3 : 4;
        const int anchor1 = two ? c_anchors[d] : -1;
        uint64_t sbits = hi >> (M.header_bits - 64);
#pragma unroll
        for (int px = 0; px < 16; ++px) {
            const int nb = ib - ((px == 0 || px == anchor1) ? 1 : 0);
            const int idx = (int)(sbits & ((1u << nb) - 1u));
            sbits >>= nb;
            rec[12 + px] = __fdiv_rn((float)bc6h_weight(idx, two), 512.f);
        }
    }
    rec[28] = __int_as_float(part);
    rec[29] = __int_as_float(mode);
    float4 *out = reinterpret_cast<float4 *>(records + (((int64_t)by * bw + bx) * nt + t) * kBc6fFloats);
#pragma unroll
    for (int k = 0; k < kBc6fFloats / 4; ++k) out[k] = make_float4(rec[4 * k], rec[4 * k + 1], rec[4 * k + 2], rec[4 * k + 3]);
}

// One candidate mode for the record targets; returns the error or -1 when the deltas do not fit.
__device__ int64_t bc6f_try_mode(int mi, int part, const int (&U)[2][2][3], const int32_t (&T)[16][3], Cand &out)
{
    const NtBc6hMode M = c_modes[mi];
    const int regions = M.regions, epb = M.endpoint_bits, ib = regions == 2 ? 3 : 4;
    const int ni = 1 << ib;
    const uint32_t mask = regions == 2 ? c_parts[part] : 0u;
    const int anchor1 = regions == 2 ? c_anchors[part] : 0;
    int q[2][2][3], u[2][2][3];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                q[r][i][c] = quantize_unsigned(U[r][i][c], epb);
                u[r][i][c] = unquantize(q[r][i][c], epb, false);
            }
    int idx[16];
    int64_t err = 0;
#pragma unroll
    for (int px = 0; px < 16; ++px) {
        const int r = (mask >> px) & 1;
        int64_t best = INT64_MAX;
        int bi = 0;
#pragma unroll 1
        for (int k = 0; k < ni; ++k) {
            const int w = bc6h_weight(k, ib == 3);
            int64_t dsum = 0;
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const int a = r ? u[1][0][c] : u[0][0][c], bb = r ? u[1][1][c] : u[0][1][c];
                const int v = (a * (64 - w) + bb * w + 32) >> 6;
                const int64_t dd = (int64_t)(T[px][c] - 64 * v);
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
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        if (r >= regions) break;
        const int ap = r == 0 ? 0 : anchor1;
        int aidx = 0;
#pragma unroll
        for (int px = 0; px < 16; ++px)
            if (px == ap) aidx = idx[px];
        if (aidx < ni / 2) continue;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const int t = q[r][0][c];
            q[r][0][c] = q[r][1][c];
            q[r][1][c] = t;
        }
#pragma unroll
        for (int px = 0; px < 16; ++px)
            if ((int)((mask >> px) & 1) == r) idx[px] = ni - 1 - idx[px];
    }
    int e[4][3];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int c = 0; c < 3; ++c) e[2 * r + i][c] = r < regions ? q[r][i][c] : 0;
    if (M.transformed) {
        // the decoder adds deltas modulo 2^epb, so the difference is taken modulo 2^epb
#pragma unroll
        for (int i = 1; i < 4; ++i) {
            if (i >= 2 * regions) break;
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const int dlt = sign_extend(e[i][c] - e[0][c], epb);
                const int db = M.delta_bits[c];
                if (dlt < -(1 << (db - 1)) || dlt > (1 << (db - 1)) - 1) return -1;
                e[i][c] = dlt;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 3; ++c) out.e[i][c] = e[i][c];
    uint64_t pk = 0;
#pragma unroll
    for (int px = 0; px < 16; ++px) pk |= (uint64_t)idx[px] << (4 * px);
    out.idx = pk;
    out.mi = mi;
    out.part = part;
    return err;
}

__device__ __forceinline__ double clamp_target(double v, double hi) { return fmin(fmax(v, 0.0), hi); }  // NaN -> 0

// grid: (ceil(block columns / 128), block rows, channel triples); one thread per record
__global__ void __launch_bounds__(128) bc6f_to_bc6h_kernel(const float *__restrict__ records, uint4 *__restrict__ blocks,
                                                           int bw, int bh, int nt)
{
    const int bx = blockIdx.x * blockDim.x + threadIdx.x, by = blockIdx.y, t = blockIdx.z;
    if (bx >= bw) return;
    const float4 *in = reinterpret_cast<const float4 *>(records + (((int64_t)by * bw + bx) * nt + t) * kBc6fFloats);
    float rec[kBc6fFloats];
#pragma unroll
    for (int k = 0; k < kBc6fFloats / 4; ++k) {
        const float4 v = __ldg(in + k);
        rec[4 * k] = v.x;
        rec[4 * k + 1] = v.y;
        rec[4 * k + 2] = v.z;
        rec[4 * k + 3] = v.w;
    }
    const int part = __float_as_int(rec[28]) & 31;
    const int own = (unsigned)__float_as_int(rec[29]) > 9u ? 0 : __float_as_int(rec[29]);
    const int b = bc6f_mode_bits(own);
    int U[2][2][3];
#pragma unroll
    for (int k = 0; k < 12; ++k) {
        const double v = __ddiv_rn(__dmul_rn((double)bc6f_unquantize(rec[k], b), 64.0), 31.0);
        U[k / 6][(k / 3) & 1][k % 3] = (int)floor(__dadd_rn(clamp_target(v, 65535.0), 0.5));
    }
    int32_t T[16][3];  // <= 64 * 65535
    const uint32_t pmask = c_parts[part];
#pragma unroll
    for (int px = 0; px < 16; ++px) {
        const int r = (pmask >> px) & 1;
        const double a = __dmul_rn(512.0, (double)rec[12 + px]);
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const int u0 = r ? U[1][0][c] : U[0][0][c], u1 = r ? U[1][1][c] : U[0][1][c];
            const double v = __dadd_rn(__dmul_rn(64.0, (double)u0), __dmul_rn((double)(u1 - u0), a));
            T[px][c] = (int32_t)floor(__dadd_rn(clamp_target(v, 64.0 * 65535.0), 0.5));
        }
    }
    bool same = true;
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int c = 0; c < 3; ++c) same = same && U[0][i][c] == U[1][i][c];
    int64_t best = INT64_MAX;
    Cand cand, winner;
#pragma unroll 1
    for (int k = 0; k < 14; ++k) {
        const int mi = k == 0 ? own : (k <= 9 ? (k - 1 < own ? k - 1 : k) : k);
        if (mi >= 10 && !same) break;
        const int64_t e = bc6f_try_mode(mi, mi < 10 ? part : 0, U, T, cand);
        if (e >= 0 && e < best) {
            best = e;
            winner = cand;
        }
    }
    Block128 out;
    if (best == INT64_MAX) out.w[0] = out.w[1] = out.w[2] = out.w[3] = 0u;  // unreachable: mode 10 always fits
    else pack_block(winner, out);
    blocks[((int64_t)t * bh + by) * bw + bx] = make_uint4(out.w[0], out.w[1], out.w[2], out.w[3]);
}

cudaError_t launch_bc6f_convert(const void *blocks, float *records, int32_t w, int32_t h, int32_t channels,
                                bool to_records, cudaStream_t st)
{
    const int bw = w / 4, bh = h / 4, nt = (channels + 2) / 3;
    if (bh > 65535 || nt > 65535) return cudaErrorInvalidValue;
    const dim3 grid((bw + 127) / 128, bh, nt);
    uint4 *bl = reinterpret_cast<uint4 *>(const_cast<void *>(blocks));
    if (to_records)
        bc6f_from_bc6h_kernel<<<grid, 128, 0, st>>>(bl, records, bw, bh, nt);
    else
        bc6f_to_bc6h_kernel<<<grid, 128, 0, st>>>(records, bl, bw, bh, nt);
    count_launch();
    return cudaGetLastError();
}

__global__ void fetch_texels_kernel(cudaTextureObject_t tex, int w, int h, float4 *out)
{
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
    if (x < w && y < h) out[(size_t)y * w + x] = tex2D<float4>(tex, x + 0.5f, y + 0.5f);
}

cudaError_t hardware_decode(const void *blocks, int bw, int bh, int is_signed, float *rgba)
{
    const int w = bw * 4, h = bh * 4;
    cudaChannelFormatDesc desc = cudaCreateChannelDesc(
        16, 16, 16, 0,
        is_signed ? cudaChannelFormatKindSignedBlockCompressed6H : cudaChannelFormatKindUnsignedBlockCompressed6H);
    cudaArray_t arr = nullptr;
    cudaTextureObject_t tex = 0;
    float4 *dout = nullptr;
    cudaError_t e = cudaMallocArray(&arr, &desc, w, h);
    if (e == cudaSuccess)
        e = cudaMemcpy2DToArray(arr, 0, 0, blocks, (size_t)bw * 16, (size_t)bw * 16, bh, cudaMemcpyDefault);
    if (e == cudaSuccess) {
        cudaResourceDesc rd = {};
        rd.resType = cudaResourceTypeArray;
        rd.res.array.array = arr;
        cudaTextureDesc td = {};
        td.addressMode[0] = td.addressMode[1] = cudaAddressModeClamp;
        td.filterMode = cudaFilterModePoint;
        td.readMode = cudaReadModeElementType;
        td.normalizedCoords = 0;
        e = cudaCreateTextureObject(&tex, &rd, &td, nullptr);
    }
    if (e == cudaSuccess) e = cudaMalloc(&dout, (size_t)w * h * sizeof(float4));
    if (e == cudaSuccess) {
        fetch_texels_kernel<<<dim3((w + 127) / 128, h), 128>>>(tex, w, h, dout);
        count_launch();
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(rgba, dout, (size_t)w * h * sizeof(float4), cudaMemcpyDeviceToHost);
    if (dout) cudaFree(dout);
    if (tex) cudaDestroyTextureObject(tex);
    if (arr) cudaFreeArray(arr);
    return e;
}

cudaError_t launch_bc6h_raw(const void *blocks, int64_t n, int is_signed, void *out, cudaStream_t st)
{
    const int64_t want = (n + 127) / 128;
    const int grid = (int)(want < 64 * (int64_t)sm_count() ? want : 64 * (int64_t)sm_count());
    bc6h_decode_raw_kernel<<<grid > 0 ? grid : 1, 128, 0, st>>>(reinterpret_cast<const uint4 *>(blocks), n,
                                                                 is_signed, reinterpret_cast<uint16_t *>(out));
    count_launch();
    return cudaGetLastError();
}

}  // namespace nt

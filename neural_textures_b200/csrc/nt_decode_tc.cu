// nt_decode_tc.cu -- decode (inference) of every texel centre on the tcgen05 tensor cores.
//
// Same contract as nt_decode.cu (Inference / RunInference, mavenkim2/neural_textures
// train.cu:917-961, :974-977): texel centres u = (x + 0.5) / W, Catmull-Rom sampling of both
// latent grids, positional features, the 32 -> 64 -> 64 -> cout network, fp16 (or fp32)
// outputs and an optional squared error against a target.
//
// A CTA of 4 warps owns one 16 x 8 texel tile (M = 128, texel r = TMEM lane r, one thread per
// texel) at a time; four CTAs share an SM (a fifth measured 37% slower: its shared memory
// leaves the gathers too little L1).  With NT_DEC_SPLIT=2 a CTA has 8 warps and the two
// threads of a texel split the gather (grid 0 / grid 1 and the positional features) and the
// epilogue columns.  Per tile:
//     gather -> F1 -> E1 -> F2 -> E2 -> F3 -> outputs
// with the products of nt_train_tc.cu's forward half (biases folded in as a constant-1
// input column; H2 overwrites H1, whose last reader is F2).  Every wait is bounded.
#include <cstdlib>
#include <cstring>

#include "nt_tc_common.cuh"

namespace nt {

__device__ unsigned int g_decode_status;  // bit 0: a bounded wait of the decode kernel gave up

namespace tc {

#ifndef NT_DEC_SPLIT
#define NT_DEC_SPLIT 1
#endif
#ifndef NT_DEC_CTAS
#define NT_DEC_CTAS 4
#endif
constexpr int kSplit = NT_DEC_SPLIT;           // threads per texel (1 or 2)
constexpr int kDecThreads = 128 * kSplit;
constexpr int kDecCtas = NT_DEC_CTAS;          // CTAs per SM
constexpr uint32_t kDecTmemCols = 64;

template <int C>
struct DecSmem {
    alignas(128) uint8_t W1[64 * Cfg<C>::XW * 2];
    alignas(128) uint8_t W2[64 * kHW * 2];
    alignas(128) uint8_t W3[16 * kHW * 2];
    alignas(128) uint8_t X[kTileN * Cfg<C>::XW * 2];
    alignas(128) uint8_t H[kTileN * kHW * 2];  // H1e, then H2e
    alignas(8) uint64_t done;
    uint32_t tmem_base;
    float red[kDecThreads / 32];
};

// 4 latents (8 bytes) at input column k (a multiple of 4) of X row r.
__device__ __forceinline__ void st8(uint8_t *X, int r, int k, int xc, uint32_t a, uint32_t b)
{
    *reinterpret_cast<uint2 *>(X + umma::cm_offset(r, k, xc)) = make_uint2(a, b);
}

// ---- separable gather of a texel tile ----------------------------------------------------
//
// Texel centres are regular, so every texel of an image column has the same horizontal
// Catmull-Rom base and weights, and every texel of an image row the same vertical ones.  Per
// tile and grid, pass 1 forms the horizontal 4-tap sums of each needed grid row at each of
// the 16 image columns (into the idle activation buffer), pass 2 the 4-tap vertical sum per
// texel.  Same operations in the same order as gather_cr (row sums first, then the
// weighted sum of rows), so the features are bit-identical.

template <int C>
__host__ __device__ constexpr int sep_rows() { return (kTileN * kHW * 2) / (2 * kTileW * C * 4); }  // rows per grid that fit

// Base row of image row y in a grid of height gh (footprint()'s arithmetic).
__device__ __forceinline__ int base_row(int y, int image_h, int gh, float &f)
{
    const float v = div_by_size(__fadd_rn((float)y, 0.5f), image_h);
    return cr_base(v, gh, f);
}

// Pass 1 (all threads): rows [by_first - 1, by_first - 1 + nr) of grid g at columns x0..x0+15.
template <int C>
__device__ __forceinline__ void sep_pass1(float *hs, const DecodeLaunch &p, int g, int row0, int nr, int x0, int tid,
                                          int nth)
{
    for (int k = tid; k < nr * kTileW; k += nth) {
        const int ri = k / kTileW, xi = k - ri * kTileW, x = x0 + xi;
        float2 row[C / 2];
#pragma unroll
        for (int q = 0; q < C / 2; ++q) row[q] = make_float2(0.f, 0.f);
        if (x < p.image_w) {
            float fx;
            const float u = div_by_size(__fadd_rn((float)x, 0.5f), p.image_w);
            const int bx = cr_base(u, p.gw[g], fx);
            float wx[4];
            catmull_rom_weights(fx, wx);
            const __half *rp = p.grid[g] + (size_t)wrap_coord(row0 + ri, p.gh[g]) * p.gw[g] * C;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const __half *tp = rp + (size_t)wrap_coord(bx - 1 + i, p.gw[g]) * C;
                const float2 w2 = make_float2(wx[i], wx[i]);
#pragma unroll
                for (int q = 0; q < C / 4; ++q) {
                    const uint2 raw = __ldg(reinterpret_cast<const uint2 *>(tp) + q);
                    row[2 * q] = ffma2(w2, unpack_half2(raw.x), row[2 * q]);
                    row[2 * q + 1] = ffma2(w2, unpack_half2(raw.y), row[2 * q + 1]);
                }
            }
        }
        float4 *o = reinterpret_cast<float4 *>(hs + (size_t)(ri * kTileW + xi) * C);
#pragma unroll
        for (int q = 0; q < C / 4; ++q) o[q] = make_float4(row[2 * q].x, row[2 * q].y, row[2 * q + 1].x, row[2 * q + 1].y);
    }
}

// ---- window staging: the next tile's pass-1 texels copied into X while this tile computes --
//
// After F1 has read X, the texels that the next tile's pass 1 reads (per grid, rows
// row0 .. row0 + nr - 1 and columns col0 .. col0 + ncol - 1 of the unwrapped grid, wrapped at
// copy time) are copied into X with cp.async; the next tile waits for them, forms its row sums
// from shared memory, and only then overwrites X with its features.  The row sums take the
// same operations in the same order as sep_pass1, so they are bit-identical.

struct DecWin {
    int row0, nr, col0, ncol;
};

// Unwrapped base texel of image column x in a grid of width gw (sep_pass1's arithmetic).
__device__ __forceinline__ int base_col(int x, int image_w, int gw)
{
    float f;
    return cr_base(div_by_size(__fadd_rn((float)x, 0.5f), image_w), gw, f);
}

// The windows of `tile`: 2 when both fit the separable path and X together (staged), 1 when
// they fit the separable path only, 0 when a grid needs more rows than the row-sum buffer.
template <int C>
__device__ __forceinline__ int dec_windows(const DecodeLaunch &p, int tile, DecWin (&w)[2])
{
    const int x0 = (tile % p.tiles_x) * kTileW, y0 = (tile / p.tiles_x) * kTileH;
    const int xlast = min(x0 + kTileW, p.image_w) - 1, ylast = min(y0 + kTileH, p.image_h) - 1;
    int texels = 0;
    bool ok = true;
#pragma unroll
    for (int g = 0; g < 2; ++g) {
        float fdum;
        const int b0 = base_row(y0, p.image_h, p.gh[g], fdum), b1 = base_row(ylast, p.image_h, p.gh[g], fdum);
        const int c0 = base_col(x0, p.image_w, p.gw[g]), c1 = base_col(xlast, p.image_w, p.gw[g]);
        w[g].row0 = b0 - 1;
        w[g].nr = b1 - b0 + 4;
        w[g].col0 = c0 - 1;
        w[g].ncol = c1 - c0 + 4;
        ok = ok && w[g].nr <= sep_rows<C>();
        texels += w[g].nr * w[g].ncol;
    }
    return !ok ? 0 : (texels * C * 2 <= kTileN * Cfg<C>::XW * 2 ? 2 : 1);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void *src)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Byte offset of grid g's window in X.
template <int C>
__device__ __forceinline__ int win_offset(const DecWin (&w)[2], int g)
{
    return g ? w[0].nr * w[0].ncol * C * 2 : 0;
}

template <int C>
__device__ __forceinline__ void stage_windows(uint8_t *X, const DecodeLaunch &p, const DecWin (&w)[2], int tid, int nth)
{
#pragma unroll
    for (int g = 0; g < 2; ++g) {
        const uint32_t base = smem_addr(X) + win_offset<C>(w, g);
        const int n = w[g].nr * w[g].ncol;
        for (int k = tid; k < n; k += nth) {
            const int ri = k / w[g].ncol, ci = k - ri * w[g].ncol;
            const __half *src = p.grid[g] + ((size_t)wrap_coord(w[g].row0 + ri, p.gh[g]) * p.gw[g] +
                                             wrap_coord(w[g].col0 + ci, p.gw[g])) * C;
            if constexpr (C == 8) {
                cp_async16(base + k * 16, src);
            } else {
#pragma unroll
                for (int j = 0; j < C / 4; ++j) cp_async8(base + k * C * 2 + 8 * j, src + 4 * j);
            }
        }
    }
}

// Pass 1 of grid g from its staged window (sep_pass1 with shared-memory taps).
template <int C>
__device__ __forceinline__ void sep_pass1_win(float *hs, const uint8_t *win, const DecWin &w, const DecodeLaunch &p,
                                              int g, int x0, int tid, int nth)
{
    for (int k = tid; k < w.nr * kTileW; k += nth) {
        const int ri = k / kTileW, xi = k - ri * kTileW, x = x0 + xi;
        float2 row[C / 2];
#pragma unroll
        for (int q = 0; q < C / 2; ++q) row[q] = make_float2(0.f, 0.f);
        if (x < p.image_w) {
            float fx;
            const float u = div_by_size(__fadd_rn((float)x, 0.5f), p.image_w);
            const int bx = cr_base(u, p.gw[g], fx);
            float wx[4];
            catmull_rom_weights(fx, wx);
            const uint8_t *rp = win + (size_t)ri * w.ncol * C * 2;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint8_t *tp = rp + (size_t)(bx - 1 + i - w.col0) * C * 2;
                const float2 w2 = make_float2(wx[i], wx[i]);
#pragma unroll
                for (int q = 0; q < C / 4; ++q) {
                    const uint2 raw = *reinterpret_cast<const uint2 *>(tp + 8 * q);
                    row[2 * q] = ffma2(w2, unpack_half2(raw.x), row[2 * q]);
                    row[2 * q + 1] = ffma2(w2, unpack_half2(raw.y), row[2 * q + 1]);
                }
            }
        }
        float4 *o = reinterpret_cast<float4 *>(hs + (size_t)(ri * kTileW + xi) * C);
#pragma unroll
        for (int q = 0; q < C / 4; ++q) o[q] = make_float4(row[2 * q].x, row[2 * q].y, row[2 * q + 1].x, row[2 * q + 1].y);
    }
}

// Pass 2 (one texel): weighted sum of its 4 staged rows.
template <int C>
__device__ __forceinline__ void sep_pass2(const float *hs, int ri0, int xi, const float (&wy)[4], float (&f)[C])
{
    float2 acc[C / 2];
#pragma unroll
    for (int q = 0; q < C / 2; ++q) acc[q] = make_float2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float4 *rp = reinterpret_cast<const float4 *>(hs + (size_t)((ri0 + j) * kTileW + xi) * C);
        const float2 w2 = make_float2(wy[j], wy[j]);
#pragma unroll
        for (int q = 0; q < C / 4; ++q) {
            const float4 v = rp[q];
            acc[2 * q] = ffma2(w2, make_float2(v.x, v.y), acc[2 * q]);
            acc[2 * q + 1] = ffma2(w2, make_float2(v.z, v.w), acc[2 * q + 1]);
        }
    }
#pragma unroll
    for (int q = 0; q < C / 2; ++q) {
        f[2 * q] = acc[q].x;
        f[2 * q + 1] = acc[q].y;
    }
}

// Stage boundary (operands fenced to the async proxy, CTA barrier that also agrees on
// failure), thread 0 issues the stage's products, every thread runs `meanwhile` and then
// waits for them.
template <int C, typename F>
__device__ __forceinline__ bool dec_stage(int stage, const DecSmem<C> &s, uint32_t tmem, uint32_t done, uint32_t &ph,
                                          bool &failed, int tid, F &&meanwhile)
{
    using K = Cfg<C>;
    using umma::desc;
    using umma::idesc_f16;
    using umma::mma_f16;
    constexpr uint32_t XG = K::XC * 128, HG = kHC * 128;
    umma::fence_async_smem();
    umma::fence_before();
    if (__syncthreads_or(failed)) {
        failed = true;
        return false;
    }
    umma::fence_after();
    if (tid == 0) {
        const uint64_t dh = desc(smem_addr(s.H), 128, HG);
        if (stage == 0) {
            const uint64_t dx = desc(smem_addr(s.X), 128, XG), dw = desc(smem_addr(s.W1), 128, XG);
#pragma unroll
            for (int ks = 0; ks < K::XC / 2; ++ks)
                mma_f16(tmem, dadv(dx, ks * 256), dadv(dw, ks * 256), idesc_f16(128, 64, 0, 0), ks > 0);
        } else if (stage == 1) {
            const uint64_t dw = desc(smem_addr(s.W2), 128, HG);
#pragma unroll
            for (int ks = 0; ks < kHC / 2; ++ks)
                mma_f16(tmem, dadv(dh, ks * 256), dadv(dw, ks * 256), idesc_f16(128, 64, 0, 0), ks > 0);
        } else {
            const uint64_t dw = desc(smem_addr(s.W3), 128, HG);
#pragma unroll
            for (int ks = 0; ks < kHC / 2; ++ks)
                mma_f16(tmem, dadv(dh, ks * 256), dadv(dw, ks * 256), idesc_f16(128, 16, 0, 0), ks > 0);
        }
        umma::commit(done);
    }
    meanwhile();
    if (!umma::mbar_wait(done, ph, kSpinLimit)) {
        failed = true;
        atomicOr(&g_decode_status, 1u);
        umma::mbar_wait(done, ph, kSpinLimit);  // one more bounded wait for the products in flight
    }
    ph ^= 1u;
    umma::fence_after();
    return true;
}

// MIP: a fractional mip coordinate; grid g also reads a second level with weight mip_t[g].
template <int C, bool MIP>
__global__ void __launch_bounds__(kDecThreads, kDecCtas) decode_tc_kernel(const DecodeLaunch p)
{
    using K = Cfg<C>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    DecSmem<C> &s = *reinterpret_cast<DecSmem<C> *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r = tid & (kTileN - 1), half = tid >> 7;  // half is 0 when kSplit == 1

    stage_weights_tc<C>(s, p.net, tid, kDecThreads);
    if (warp == 0) umma::alloc(smem_addr(&s.tmem_base), kDecTmemCols);
    if (tid == 0) {
        umma::mbar_init(smem_addr(&s.done), 1);
        umma::mbar_fence_init();
    }
    umma::fence_async_smem();
    umma::fence_before();
    __syncthreads();
    umma::fence_after();
    const uint32_t tmem = s.tmem_base;
    const uint32_t Rl = tmem + ((uint32_t)(32 * (warp & 3)) << 16);  // this warp's lanes
    const uint32_t done = smem_addr(&s.done);
    const int ntiles = p.tiles_x * p.tiles_y;
    const int cout = p.net.cout;
    uint32_t ph = 0;
    bool failed = false;
    float sse = 0.f;

    DecWin w[2];  // this tile's windows (computed when the tile before staged them)
    int wmode = 0;
    if ((int)blockIdx.x < ntiles) {
        wmode = dec_windows<C>(p, blockIdx.x, w);
        if (wmode == 2) stage_windows<C>(s.X, p, w, tid, kDecThreads);
    }
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int x = (tile % p.tiles_x) * kTileW + (r & (kTileW - 1));
        const int y = (tile / p.tiles_x) * kTileH + (r >> 4);
        const bool valid = x < p.image_w && y < p.image_h;

        // ---- gather: separable passes through shared memory (direct taps if rows overflow) ---
        {
            const int x0 = (tile % p.tiles_x) * kTileW;
            const bool sep = wmode > 0;
            const int row0[2] = {w[0].row0, w[1].row0};
            float *hs0 = reinterpret_cast<float *>(s.H), *hs1 = hs0 + sep_rows<C>() * kTileW * C;
            if (wmode == 2) {  // the windows were staged into X during the tile before
                cp_async_wait_all();
                __syncthreads();
                sep_pass1_win<C>(hs0, s.X, w[0], p, 0, x0, tid, kDecThreads);
                sep_pass1_win<C>(hs1, s.X + win_offset<C>(w, 1), w[1], p, 1, x0, tid, kDecThreads);
                __syncthreads();  // X is overwritten below
            } else if (sep) {
                sep_pass1<C>(hs0, p, 0, w[0].row0, w[0].nr, x0, tid, kDecThreads);
                sep_pass1<C>(hs1, p, 1, w[1].row0, w[1].nr, x0, tid, kDecThreads);
                __syncthreads();
            }
            float u = 0.f, v = 0.f;
            if (valid) texel_uv(x, y, p.image_w, p.image_h, u, v);
#pragma unroll
            for (int gg = 0; gg < 3 - kSplit; ++gg) {
                const int g = kSplit == 2 ? half : gg;
                float f[C];
#pragma unroll
                for (int k = 0; k < C; ++k) f[k] = 0.f;
                if (valid) {
                    if (sep) {
                        float fy, wy[4];
                        const int by = cr_base(v, p.gh[g], fy);
                        catmull_rom_weights(fy, wy);
                        sep_pass2<C>(g ? hs1 : hs0, by - 1 - row0[g], r & (kTileW - 1), wy, f);
                    } else {
                        Footprint fp;
                        footprint(u, v, p.gw[g], p.gh[g], fp);
                        gather_cr<C>(p.grid[g], p.gw[g], fp, f);
                    }
                    if constexpr (MIP) {
                        const float t = p.mip_t[g];
                        if (t > 0.f) {  // second mip level: (1 - t) level m0 + t level m1
                            Footprint fb;
                            footprint(u, v, p.gw_b[g], p.gh_b[g], fb);
                            float fl[C];
                            gather_cr<C>(p.grid_b[g], p.gw_b[g], fb, fl);
                            const float omt = __fsub_rn(1.f, t);
#pragma unroll
                            for (int k = 0; k < C; ++k) f[k] = __fadd_rn(__fmul_rn(omt, f[k]), __fmul_rn(t, fl[k]));
                        }
                    }
                }
#pragma unroll
                for (int q = 0; q < C / 4; ++q)
                    st8(s.X, r, g * C + 4 * q, K::XC, pack_half2(f[4 * q], f[4 * q + 1]),
                        pack_half2(f[4 * q + 2], f[4 * q + 3]));
            }
            if (half == kSplit - 1) {
                uint32_t pk[4] = {0u, 0u, 0u, 0u};
                if (valid) {
                    float pe[8];
                    posenc(u, v, pe);
#pragma unroll
                    for (int k = 0; k < 4; ++k) pk[k] = pack_half2(pe[2 * k], pe[2 * k + 1]);
                }
                st16(s.X, umma::cm_offset(r, 8 * K::LC, K::XC), pk[0], pk[1], pk[2], pk[3]);
                st16(s.X, umma::cm_offset(r, 8 * (K::LC + 1), K::XC), pack_half2(1.f, 0.f), 0u, 0u, 0u);
                if constexpr (K::XC > K::LC + 2)
                    st16(s.X, umma::cm_offset(r, 8 * (K::LC + 2), K::XC), 0u, 0u, 0u, 0u);
            }
        }
        const auto nothing = [] {};
        if (!dec_stage<C>(0, s, tmem, done, ph, failed, tid, nothing)) break;

        // ---- E1: H1e = [relu(Z1) | 1 | 0] ------------------------------------------------
#pragma unroll
        for (int b = 0; b < 3 - kSplit; ++b) relu_store32(Rl + 32 * (half + b), s.H, r, 4 * (half + b));
        if (half == kSplit - 1) st16(s.H, umma::cm_offset(r, 64, kHC), pack_half2(1.f, 0.f), 0u, 0u, 0u);
        if (half == 0) st16(s.H, umma::cm_offset(r, 72, kHC), 0u, 0u, 0u, 0u);
        // while F2 runs (F1 has read X): stage the next tile's windows
        const auto stage_next = [&] {
            if (tile + (int)gridDim.x < ntiles) {
                wmode = dec_windows<C>(p, tile + gridDim.x, w);
                if (wmode == 2) stage_windows<C>(s.X, p, w, tid, kDecThreads);
            }
        };
        if (!dec_stage<C>(1, s, tmem, done, ph, failed, tid, stage_next)) break;

        // ---- E2: H2e over H1e (the constant columns stay) ----------------------------------
#pragma unroll
        for (int b = 0; b < 3 - kSplit; ++b) relu_store32(Rl + 32 * (half + b), s.H, r, 4 * (half + b));
        if (!dec_stage<C>(2, s, tmem, done, ph, failed, tid, nothing)) break;

        // ---- outputs: half 0 channels 0..7, half 1 channels 8..15 -------------------------
        {
            uint32_t v[16];
            umma::ld16(Rl, v);
            umma::wait_ld();
#pragma unroll
            for (int hb = 0; hb < 3 - kSplit; ++hb) {
                const int h8 = half + hb;  // channel group of 8
                if (!valid || (h8 > 0 && cout <= 8)) continue;
                const int c0 = 8 * h8, c1 = min(cout, c0 + 8);
                const size_t texel = (size_t)y * p.image_w + x;
                float yv[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) yv[e] = round_half(__uint_as_float(h8 ? v[8 + e] : v[e]));
                const int ostride = p.out_stride;
                if (!p.out_f32 && ostride == 8 && h8 == 0) {
                    *reinterpret_cast<uint4 *>(reinterpret_cast<__half *>(p.out) + texel * 8) =
                        make_uint4(pack_half2(yv[0], yv[1]), pack_half2(yv[2], yv[3]), pack_half2(yv[4], yv[5]),
                                   pack_half2(yv[6], yv[7]));
                } else if (!p.out_f32) {
                    __half *o = reinterpret_cast<__half *>(p.out) + texel * ostride;
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        if (c0 + e < c1) o[c0 + e] = __float2half_rn(yv[e]);
                } else {
                    float *o = reinterpret_cast<float *>(p.out) + texel * ostride;
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        if (c0 + e < c1) o[c0 + e] = yv[e];
                }
                if (ostride > cout && h8 == (cout - 1) / 8) {  // zero channels cout .. stride - 1
                    for (int c = cout; c < ostride; ++c) {
                        if (p.out_f32) reinterpret_cast<float *>(p.out)[texel * ostride + c] = 0.f;
                        else reinterpret_cast<__half *>(p.out)[texel * ostride + c] = __float2half_rn(0.f);
                    }
                }
                if (p.target) {
                    const __half *t = p.target + texel * cout;
                    float tv[8];
                    if (cout == 8 && (reinterpret_cast<uintptr_t>(p.target) & 15u) == 0) {  // one 16-byte load
                        const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(t));
                        const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const float2 f2 = __half22float2(*reinterpret_cast<const __half2 *>(&w4[q]));
                            tv[2 * q] = f2.x;
                            tv[2 * q + 1] = f2.y;
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e) tv[e] = c0 + e < c1 ? __half2float(t[c0 + e]) : 0.f;
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        if (c0 + e < c1) {
                            const float d = yv[e] - tv[e];
                            sse = fmaf(d, d, sse);
                        }
                } else if (p.num_ref > 0 && p.mse_accum) {  // reference textures (train.cu:946-960)
                    float uu, vv, ex[16];
                    texel_uv(x, y, p.image_w, p.image_h, uu, vv);
                    ref_expected(p.ref, p.num_ref, uu, vv, p.ref_lod, ex);
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        if (c0 + e < c1) {
                            float te = 0.f;
#pragma unroll
                            for (int k = 0; k < 16; ++k)
                                if (k == c0 + e) te = ex[k];
                            const float d = yv[e] - te;
                            sse = fmaf(d, d, sse);
                        }
                }
            }
        }
        umma::fence_before();  // the next tile's F1 overwrites the accumulator after its barrier
    }

    cp_async_wait_all();  // copies staged for a tile that a failed stage left untouched
    if (p.mse_accum) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sse += __shfl_xor_sync(0xffffffffu, sse, o);
        if (lane == 0) s.red[warp] = sse;
    }
    __syncthreads();
    if (p.mse_accum && tid == 0) {
        float tot = 0.f;
        for (int w = 0; w < kDecThreads / 32; ++w) tot += s.red[w];
        atomicAdd(p.mse_accum, tot);
    }
    if (warp == 0) {
        umma::fence_after();
        umma::dealloc(tmem, kDecTmemCols);
    }
}

template <int C, bool MIP>
static cudaError_t launch_dec_t(DecodeLaunch p, cudaStream_t stream)
{
    const size_t smem = sizeof(DecSmem<C>);
    cudaError_t e = set_smem_limit(reinterpret_cast<const void *>(decode_tc_kernel<C, MIP>), smem);
    if (e != cudaSuccess) return e;
    p.tiles_x = (p.image_w + kTileW - 1) / kTileW;
    p.tiles_y = (p.image_h + kTileH - 1) / kTileH;
    const int ntiles = p.tiles_x * p.tiles_y;
    const int cap = kDecCtas * sm_count();
    const int grid = ntiles < cap ? ntiles : cap;
    decode_tc_kernel<C, MIP><<<grid, kDecThreads, smem, stream>>>(p);
    count_launch();
    return cudaGetLastError();
}

}  // namespace tc

cudaError_t launch_decode_tc(const DecodeLaunch &p, int channels, cudaStream_t stream)
{
    const bool mip = p.mip_t[0] > 0.f || p.mip_t[1] > 0.f;
    if (channels == 8) return mip ? tc::launch_dec_t<8, true>(p, stream) : tc::launch_dec_t<8, false>(p, stream);
    if (channels == 12) return mip ? tc::launch_dec_t<12, true>(p, stream) : tc::launch_dec_t<12, false>(p, stream);
    return cudaErrorInvalidValue;
}

// Host: the decode kernel's status word (cleared on request).
cudaError_t read_decode_status(uint32_t *status, bool clear)
{
    cudaError_t e = cudaMemcpyFromSymbol(status, g_decode_status, sizeof(uint32_t));
    if (e != cudaSuccess || !clear) return e;
    const uint32_t zero = 0;
    return cudaMemcpyToSymbol(g_decode_status, &zero, sizeof(uint32_t));
}

}  // namespace nt

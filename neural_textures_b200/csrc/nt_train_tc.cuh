// nt_train_tc.cuh -- pieces of the tcgen05 training kernel (nt_train_tc.cu) that do not depend
// on how a kernel lays out its shared memory: tile windows of the
// Catmull-Rom footprints, row sharding, the latent-gradient scatters (tensor-core window
// sums, column sweep, per-tap atomics), the activation-gradient epilogue and the tensor-core
// products of one training stage.
//
// References (mavenkim2/neural_textures): latent scatter train.cu:460-509 (per tap, here
// summed per window texel first), backward per layer mlp.h:222-257, BC6 backward
// train.cu:436-454.
#pragma once

#include <climits>
#include <cmath>

#include "nt_bc6f.cuh"
#include "nt_kernels.cuh"
#include "nt_mma.cuh"
#include "nt_tc_common.cuh"
#include "nt_umma.cuh"

namespace nt {

// bit 0: a bounded wait of a training kernel gave up; bit 1: a sharded call reached a row its
// shard does not store (read back by nt_read_device_status).
static __device__ unsigned int g_device_status;

namespace tc {

constexpr int kThreadsTC = 256;
constexpr int kMaxWinW = 40;  // widest footprint window the sweep handles (texels)
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColW1 = 0, kColW2 = 64, kColTile = 192;
// TMEM columns of one CTA (256): dW1 (M = 64, N = XW) at 0, dW2 (M = 64, N = 72) at 64, dW3^T
// (M = 128, N = 16) after dW1 for C = 12 (at 48: dW1 is 48 wide) or at 160 for C = 8, the stage
// accumulator at 192 (64 columns).  C = 12 keeps the second channel group of the latent
// scatter at 136 (grid 0, N = 32) and 168 (grid 1, N = 16).
template <int C>
struct Cols {
    static constexpr uint32_t W3 = C == 12 ? 48u : 160u;
    static constexpr uint32_t ScatB0 = 136, ScatB1 = 168;
};

// Tensor-core latent scatter: per grid, the window is at most sc_w(g) texels wide and
// sc_h(g) texels high (else the tile takes the column sweep).
__host__ __device__ constexpr int sc_w(int g) { return g ? 16 : 32; }
__host__ __device__ constexpr int sc_h(int g) { return g ? 8 : 12; }

struct Window {
    int32_t x0, w, span, ok;
    int32_t y0, h, tc;  // window rows; tc: fits the tensor-core scatter
    int32_t cand_x[kMaxWinW];  // lo | hi << 16 of the candidate lattice columns
};


// ---- row sharding ----------------------------------------------------------------------
//
// Source s (0, 1: latent grids, 2: target) may hold only p.rows[s] rows, starting at full
// row p.org[s] and wrapping.  A row outside them is never read or written: it is skipped
// and bit 1 of the device status word is set (the caller's shard plan is wrong).

__device__ __forceinline__ int stored_row(const TrainLaunch &p, int src, int row, int h)
{
    const int r = wrap_coord(row - p.org[src], h);
    if (r >= p.rows[src]) {
        atomicOr(&g_device_status, 2u);
        return -1;
    }
    return r;
}

// Footprint rows -> stored rows; a missing row gets weight 0 (and is flagged).
__device__ __forceinline__ void shard_rows(const TrainLaunch &p, int src, int h, Footprint &fp)
{
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int r = stored_row(p, src, fp.by - 1 + j, h);
        fp.ys[j] = r < 0 ? 0 : r;
        if (r < 0) fp.wy[j] = 0.f;
    }
}

// ---- footprint windows of a tile (for the latent-gradient sweep) ------------------------

// Per-warp min / max of the footprint bases per lattice column (lanes L and L + 16 share a
// column) and per lattice row (half-warp).
__device__ __forceinline__ void extents_partial(int32_t (&part)[4][4][kTileW], int bx, int by, bool valid, int ws,
                                                int lane)
{
    int cmin = valid ? bx : INT_MAX, cmax = valid ? bx : INT_MIN;
    cmin = min(cmin, __shfl_xor_sync(0xffffffffu, cmin, 16));
    cmax = max(cmax, __shfl_xor_sync(0xffffffffu, cmax, 16));
    int rmin = valid ? by : INT_MAX, rmax = valid ? by : INT_MIN;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
        rmin = min(rmin, __shfl_xor_sync(0xffffffffu, rmin, o));
        rmax = max(rmax, __shfl_xor_sync(0xffffffffu, rmax, o));
    }
    if (lane < 16) {
        part[0][ws][lane] = cmin;
        part[1][ws][lane] = cmax;
    }
    if ((lane & 15) == 0) {
        part[2][ws][lane >> 4] = rmin;
        part[3][ws][lane >> 4] = rmax;
    }
}

// One warp: column / row extents of grid gi over the 4 warp partials, window origin and
// size, and whether the window suits the column sweep / the tensor-core scatter.
template <class S>
__device__ __forceinline__ void finalize_window_tc(S &s, int gi, int lane)
{
    int lo_v = INT_MAX, hi_v = INT_MIN;
    if (lane < 16) {
        for (int w = 0; w < 4; ++w) {
            lo_v = min(lo_v, s.part[gi][0][w][lane]);
            hi_v = max(hi_v, s.part[gi][1][w][lane]);
        }
        s.colext[gi][0][lane] = lo_v;
        s.colext[gi][1][lane] = hi_v;
    } else if (lane < 16 + kTileH) {
        const int e = lane - 16, w = e >> 1, half = e & 1;
        lo_v = s.part[gi][2][w][half];
        hi_v = s.part[gi][3][w][half];
        s.rowmin[gi][e] = lo_v;
    }
    const bool narrow = lo_v == INT_MAX || (long long)hi_v - lo_v <= 1;
    const bool all_narrow = __all_sync(0xffffffffu, narrow);
    int mn = lo_v, mx = hi_v;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
        mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const int cmin = __shfl_sync(0xffffffffu, mn, 0), cmax = __shfl_sync(0xffffffffu, mx, 0);
    const int rmin = __shfl_sync(0xffffffffu, mn, 16), rmax = __shfl_sync(0xffffffffu, mx, 16);
    __syncwarp();
    Window &W = s.win[gi];
    const bool nonempty = cmin <= cmax && rmin <= rmax;
    const long long ww = nonempty ? (long long)cmax - cmin + 4 : 0;
    const bool ok = nonempty && ww <= kMaxWinW && all_narrow;
    const long long wh = nonempty ? (long long)rmax - rmin + 4 : 0;
    if (lane == 0) {
        W.x0 = cmin - 1;
        W.w = (int)ww;
        W.ok = ok;
        W.y0 = rmin - 1;
        W.h = nonempty ? (int)wh : 0;
        W.tc = nonempty && ww <= sc_w(gi) && wh <= sc_h(gi);
    }
}

// One warp: candidate lattice-column range of every window column of grid gi and the
// longest range (only the column sweep needs them).
template <class S>
__device__ __forceinline__ void window_cands(S &s, int gi, int lane)
{
    Window &W = s.win[gi];
    int span = 0;
    if (W.ok) {
        for (int idx = lane; idx < W.w; idx += 32) {
            const int tx = W.x0 + idx;
            int lo = kTileW, hi = -1;
            for (int c = 0; c < kTileW; ++c) {
                if (s.colext[gi][0][c] <= tx + 1 && s.colext[gi][1][c] >= tx - 2) {
                    lo = min(lo, c);
                    hi = max(hi, c);
                }
            }
            W.cand_x[idx] = lo | (hi << 16);
            span = max(span, hi - lo + 1);
        }
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) span = max(span, __shfl_xor_sync(0xffffffffu, span, o));
    if (lane == 0) W.span = span;
}

// ---- latent-gradient column sweep ------------------------------------------------------------
//
// The gradient of latent texel (tx, ty) is the sum over the tile's samples of wy(ty) wx(tx) dX.
// One thread takes one window column tx and a chunk of lattice rows; only the lattice columns
// whose footprints reach tx (cand_x) contribute, and a sample's footprint covers rows
// by - 1 .. by + 2, so five running row sums R[0..4] per channel, shifted down one row at a
// time, collect every contribution before the finished row is added to global memory.

// Gradient buffer, size and stored row of grid g at the call's first mip level (LB false) or at
// the second level of a fractional mip coordinate (LB true; such calls are unsharded).
template <bool LB>
__device__ __forceinline__ float *lvl_grad(const TrainLaunch &p, int g) { return LB ? p.ggrid_b[g] : p.ggrid[g]; }
template <bool LB>
__device__ __forceinline__ int lvl_w(const TrainLaunch &p, int g) { return LB ? p.gw_b[g] : p.gw[g]; }
template <bool LB>
__device__ __forceinline__ int lvl_h(const TrainLaunch &p, int g) { return LB ? p.gh_b[g] : p.gh[g]; }
template <bool LB>
__device__ __forceinline__ int lvl_row(const TrainLaunch &p, int g, int row, int h)
{
    if constexpr (LB) return wrap_coord(row, h);
    return stored_row(p, g, row, h);
}

// Latent gradient sum of one texel (x 1 / num_samples) into the grid gradients, or, for block
// features, through the BC6 backward into the texel's block records (train.cu:436-454; the
// backward is linear in the feature gradient, so summing a texel's taps first is exact).
template <int C, bool BLK, bool LB = false>
__device__ __forceinline__ void flush_row(const TrainLaunch &p, int gi, int tx, int ty, const float (&row)[C])
{
    bool any = false;
#pragma unroll
    for (int c = 0; c < C; ++c) any |= row[c] != 0.f;
    if (!any) return;
    const int gw = lvl_w<LB>(p, gi), gh = lvl_h<LB>(p, gi);
    const float sc = p.inv_num_samples;
    const int sy = lvl_row<LB>(p, gi, ty, gh);
    if (sy < 0) return;
    if constexpr (BLK) {
        float fg[C];
#pragma unroll
        for (int c = 0; c < C; ++c) fg[c] = row[c] * sc;
        bc6f_backward_texel<C>(reinterpret_cast<const float *>(p.grid[gi]), p.ggrid[gi], gw, wrap_coord(tx, gw), sy, fg);
        return;
    }
    float4 *dst = reinterpret_cast<float4 *>(lvl_grad<LB>(p, gi) + ((size_t)sy * gw + wrap_coord(tx, gw)) * C);
#pragma unroll
    for (int q = 0; q < C / 4; ++q)
        red_add_v4(reinterpret_cast<float *>(dst + q), row[4 * q] * sc, row[4 * q + 1] * sc, row[4 * q + 2] * sc,
                   row[4 * q + 3] * sc);
}

// S: the tile's footprints (base, wts, win, rowmin); dx: fp32 dX rows (Cfg<C>::DXS floats per
// sample, grid g's channels at g * C); NTH threads take part.
template <int C, int L, bool BLK, bool LB = false, int NTH = kThreadsTC, class S>
__device__ __forceinline__ void sweep_tc(const S &s, const float *dx, const TrainLaunch &p, int r)
{
    constexpr int kRows = 2, kChunks = kTileH / kRows, DXS = Cfg<C>::DXS;
    const int nt0 = s.win[0].w * kChunks;
    const int ntot = nt0 + s.win[1].w * kChunks;
    for (int k = r; k < ntot; k += NTH) {
        const int gi = k < nt0 ? 0 : 1;
        const Window &W = s.win[gi];
        const int kk = gi ? k - nt0 : k;
        const int chunk = kk / W.w, lx = kk % W.w;
        const int tx = W.x0 + lx;
        const int cx = W.cand_x[lx];
        const int lo = cx & 0xffff, hi = cx >> 16;
        if (hi < lo) continue;
        float R[5][C];
#pragma unroll
        for (int m = 0; m < 5; ++m)
#pragma unroll
            for (int c = 0; c < C; ++c) R[m][c] = 0.f;
        int fy_cur = INT_MIN;
#pragma unroll
        for (int rr = 0; rr < kRows; ++rr) {
            const int cj = chunk * kRows + rr;
            const int rmin = s.rowmin[gi][cj];
            if (rmin == INT_MAX) continue;
            const int fy = rmin - 1;
            if (fy_cur == INT_MIN) fy_cur = fy;
            while (fy > fy_cur) {
                flush_row<C, BLK, LB>(p, gi, tx, fy_cur, R[0]);
#pragma unroll
                for (int m = 0; m < 4; ++m)
#pragma unroll
                    for (int c = 0; c < C; ++c) R[m][c] = R[m + 1][c];
#pragma unroll
                for (int c = 0; c < C; ++c) R[4][c] = 0.f;
                ++fy_cur;
            }
#pragma unroll
            for (int b = 0; b < L; ++b) {
                const int ci = min(lo + b, kTileW - 1);
                const bool inr = lo + b <= hi;
                const int sidx = cj * kTileW + ci;
                const short2 bs = s.base[gi][sidx];
                const int kx = tx - bs.x + 1;
                const float wxv = (inr && (unsigned)kx <= 3u) ? s.wts[gi][sidx][kx & 3] : 0.f;
                const float4 wy = *reinterpret_cast<const float4 *>(&s.wts[gi][sidx][4]);
                const bool e1 = bs.y - 1 - fy != 0;
                float wxd[C];
                const float4 *d4 = reinterpret_cast<const float4 *>(dx + sidx * DXS + gi * C);
#pragma unroll
                for (int q = 0; q < C / 4; ++q) {
                    const float4 d = d4[q];
                    wxd[4 * q + 0] = wxv * d.x;
                    wxd[4 * q + 1] = wxv * d.y;
                    wxd[4 * q + 2] = wxv * d.z;
                    wxd[4 * q + 3] = wxv * d.w;
                }
                const float wyv[5] = {e1 ? 0.f : wy.x, e1 ? wy.x : wy.y, e1 ? wy.y : wy.z, e1 ? wy.z : wy.w,
                                      e1 ? wy.w : 0.f};
#pragma unroll
                for (int m = 0; m < 5; ++m)
#pragma unroll
                    for (int c = 0; c < C; ++c) R[m][c] = fmaf(wyv[m], wxd[c], R[m][c]);
            }
        }
        if (fy_cur == INT_MIN) continue;
#pragma unroll
        for (int m = 0; m < 5; ++m) flush_row<C, BLK, LB>(p, gi, tx, fy_cur + m, R[m]);
    }
}

// Per-sample, per-tap vector atomics (windows the sweep does not handle); block features
// take the BC6 backward per tap.
template <int C, bool BLK, bool LB = false, class S>
__device__ __forceinline__ void scatter_taps_tc(const S &s, const float *dx, const TrainLaunch &p, int gi, int r)
{
    const float *dxr = dx + r * Cfg<C>::DXS + gi * C;
    const int gw = lvl_w<LB>(p, gi), gh = lvl_h<LB>(p, gi);
    const short2 b = s.base[gi][r];
    const float scale = p.inv_num_samples;
    for (int j = 0; j < 4; ++j) {
        const int yy = lvl_row<LB>(p, gi, b.y - 1 + j, gh);
        if (yy < 0) continue;
        for (int i = 0; i < 4; ++i) {
            const int xx = wrap_coord(b.x - 1 + i, gw);
            if constexpr (BLK) {
                const float wgt = __fmul_rn(s.wts[gi][r][4 + j], s.wts[gi][r][i]);
                float fg[C];
#pragma unroll
                for (int k = 0; k < C; ++k) fg[k] = __fmul_rn(__fmul_rn(wgt, dxr[k]), scale);
                bc6f_backward_texel<C>(reinterpret_cast<const float *>(p.grid[gi]), p.ggrid[gi], gw, xx, yy, fg);
                continue;
            }
            const float wgt = s.wts[gi][r][i] * s.wts[gi][r][4 + j] * scale;
            float4 *dst = reinterpret_cast<float4 *>(lvl_grad<LB>(p, gi) + ((size_t)yy * gw + xx) * C);
#pragma unroll
            for (int q = 0; q < C / 4; ++q)
                red_add_v4(reinterpret_cast<float *>(dst + q), wgt * dxr[4 * q], wgt * dxr[4 * q + 1],
                           wgt * dxr[4 * q + 2], wgt * dxr[4 * q + 3]);
        }
    }
}

// ---- epilogue helpers -------------------------------------------------------------------

// TMEM row (32 columns) rounded to fp16 and masked by the ReLU of the activation row stored
// at the same place in H (lanes where the activation is not > 0 become +0), written over it.
// `wbar` / `wph`: products that still read H (the weight gradients) are waited for right
// before the stores, so the TMEM and shared loads overlap them.
__device__ __forceinline__ void mask_store32(uint32_t taddr, uint8_t *H, int r, int chunk0, uint32_t wbar,
                                             uint32_t wph, bool &failed)
{
    uint32_t v[32];
    umma::ld16(taddr, *reinterpret_cast<uint32_t(*)[16]>(v));
    umma::ld16(taddr + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
    uint4 a[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) a[q] = *reinterpret_cast<const uint4 *>(H + umma::cm_offset(r, 8 * (chunk0 + q), kHC));
    umma::wait_ld();
    const __half2 zero = __float2half2_rn(0.f);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t aw[4] = {a[q].x, a[q].y, a[q].z, a[q].w};
        uint32_t h[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const __half2 g = __floats2half2_rn(__uint_as_float(v[8 * q + 2 * e]), __uint_as_float(v[8 * q + 2 * e + 1]));
            const unsigned m = __hgt2_mask(*reinterpret_cast<const __half2 *>(&aw[e]), zero);
            h[e] = *reinterpret_cast<const uint32_t *>(&g) & m;
        }
        if (q == 0 && !umma::mbar_wait(wbar, wph, kSpinLimit)) {
            failed = true;
            atomicOr(&g_device_status, 1u);
        }
        st16(H, umma::cm_offset(r, 8 * (chunk0 + q), kHC), h[0], h[1], h[2], h[3]);
    }
}

// ---- tensor-core latent scatter -------------------------------------------------------------
//
// dG[y][x][c] = sum_s wy_s(y) wx_s(x) dX_s[c] over the tile's window is the product
// G^T[(y, c)][x] = sum_s Q[s][(y, c)] A[s][x] with Q[s][(y, c)] = wy_s(y) dX_s[c] (zero outside
// the sample's 4 rows) and A[s][x] = wx_s(x) (zero outside its 4 columns), both fp16 rows
// of one sample, read MN-major.  Channels 0-7 of a window row make one 16-byte core-matrix
// row (M = (y, c)).  With C = 12 a second product with the same A follows once the first has
// read Q: the Q tiles are rewritten with channels 8-11, two consecutive window rows per
// 16-byte row (M = (y / 2, (y % 2) 4 + c - 8)), so the operands keep the 8-channel footprint.

// Number of 16-byte Q rows per sample for grid G: channel group a (0-7), b (8-11, C = 12).
__host__ __device__ constexpr int sc_qa(int g) { return sc_h(g); }
__host__ __device__ constexpr int sc_qb(int g) { return sc_h(g) / 2; }

// Operand rows of sample r for grid g (compile-time grid so the row lengths are constants).
// S: the tile's footprints (base, wts, win); T: the scatter operand tiles (Q0, Q1, A0, A1).
// PART 0 writes channels 0-7 into Q and the column weights into A; PART 1 (C = 12, once the
// first product has read Q) writes channels 8-11 into the same Q tiles in the packed layout.
template <int C, int G, int PART = 0, class S, class T>
__device__ __forceinline__ void scatter_rows(const S &s, T &t, int r, bool valid, const float (&dx)[C])
{
    static_assert(C == 8 || C == 12, "8 or 12 latent channels");
    static_assert(PART == 0 || C == 12, "a second part only for 12 channels");
    constexpr int NQ = PART ? sc_qb(G) : sc_qa(G), NA = sc_w(G) / 8;
    uint8_t *Q = G ? t.Q1 : t.Q0;
    uint8_t *A = G ? t.A1 : t.A0;
#pragma unroll
    for (int y = 0; y < NQ; ++y) st16(Q, umma::cm_offset(r, 8 * y, NQ), 0u, 0u, 0u, 0u);
    if constexpr (PART == 0) {
#pragma unroll
        for (int k = 0; k < NA; ++k) st16(A, umma::cm_offset(r, 8 * k, NA), 0u, 0u, 0u, 0u);
    }
    if (!valid) return;  // dX is zero there, and the footprint may lie outside the window
    const Window &W = s.win[G];
    const short2 b = s.base[G][r];
    const int oy = b.y - 1 - W.y0, ox = b.x - 1 - W.x0;
    const float4 wy = *reinterpret_cast<const float4 *>(&s.wts[G][r][4]);
    const float wyv[4] = {wy.x, wy.y, wy.z, wy.w};
    if constexpr (PART == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            st16(Q, umma::cm_offset(r, 8 * (oy + j), NQ), pack_half2(wyv[j] * dx[0], wyv[j] * dx[1]),
                 pack_half2(wyv[j] * dx[2], wyv[j] * dx[3]), pack_half2(wyv[j] * dx[4], wyv[j] * dx[5]),
                 pack_half2(wyv[j] * dx[6], wyv[j] * dx[7]));
        const float4 wx = *reinterpret_cast<const float4 *>(&s.wts[G][r][0]);
        const float wxv[4] = {wx.x, wx.y, wx.z, wx.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
            *reinterpret_cast<__half *>(A + umma::cm_offset(r, ox + i, NA)) = __float2half_rn(wxv[i]);
    } else {
        constexpr int c8 = C > 8 ? 8 : 0;  // (C = 12 here)
#pragma unroll
        for (int j = 0; j < 4; ++j) {  // 8 bytes: channels 8-11 of window row oy + j
            const int y = oy + j;
            *reinterpret_cast<uint2 *>(Q + umma::cm_offset(r, 8 * (y >> 1) + 4 * (y & 1), NQ)) =
                make_uint2(pack_half2(wyv[j] * dx[c8], wyv[j] * dx[c8 + 1]),
                           pack_half2(wyv[j] * dx[c8 + 2], wyv[j] * dx[c8 + 3]));
        }
    }
}

// Staged window sums -> global latent gradients (x 1 / num_samples), one float4 reduction
// per 4 channels of every window texel.
// S: the tile's footprints (win); F: the staged window sums (g0, g1); NTH threads take part.
// Grid 0's slots and grid 1's slots run as separate loops, so that each grid's buffers, sizes
// and stored rows are compile-time selections.
template <int C, int G, bool LB, int NTH, class S, class F>
__device__ __forceinline__ void scatter_reduce_grid(const S &s, const F &f, const TrainLaunch &p, int tid)
{
    constexpr int W = sc_w(G), NQ = C / 4, n = sc_h(G) * W * NQ;  // (row, column, quad) slots
    const float sc = p.inv_num_samples;
    const Window &win = s.win[G];
    const int gw = lvl_w<LB>(p, G), gh = lvl_h<LB>(p, G);
    float *grad = lvl_grad<LB>(p, G);
    const float *src0 = G ? f.g1 : f.g0;
#pragma unroll
    for (int it = 0; it < (n + NTH - 1) / NTH; ++it) {
        const int k = tid + it * NTH;
        if (n % NTH != 0 && k >= n) break;
        const int q = k % NQ, x = (k / NQ) & (W - 1), y = k / (NQ * W);
        if (x >= win.w || y >= win.h) continue;
        const float4 v = *reinterpret_cast<const float4 *>(src0 + (y * (W + 1) + x) * C + 4 * q);
        if (v.x == 0.f && v.y == 0.f && v.z == 0.f && v.w == 0.f) continue;
        const int sy = lvl_row<LB>(p, G, win.y0 + y, gh);
        if (sy < 0) continue;
        red_add_v4(grad + ((size_t)sy * gw + wrap_coord(win.x0 + x, gw)) * C + 4 * q, v.x * sc, v.y * sc, v.z * sc,
                   v.w * sc);
    }
}

template <int C, bool LB = false, int NTH = kThreadsTC, class S, class F>
__device__ __forceinline__ void scatter_reduce(const S &s, const F &f, const TrainLaunch &p, int tid)
{
    scatter_reduce_grid<C, 0, LB, NTH>(s, f, p, tid);
    scatter_reduce_grid<C, 1, LB, NTH>(s, f, p, tid);
}

// ---- tensor-core products -------------------------------------------------------------------


template <int C>
struct Descs {
    uint64_t x, h1, h2, dy, w1, w2, w3;  // K-major views (LBO 128)
    uint64_t x_mn, h1_mn, h2_mn, dy_mn, w1_mn, w2_mn, w3_mn;  // MN-major views
    uint64_t q0, q1, a0, a1;  // latent scatter operands (MN-major)
    uint64_t q0b, q1b;        // Q0 / Q1 holding channels 8-11 (C = 12)
};

// Issue the products of one stage (thread 0 only) and commit them to `done` (the weight
// gradients of B3 / B2 / B1 come from issue_dw).
template <int C>
__device__ __forceinline__ void issue_stage(int stage, const Descs<C> &d, uint32_t tmem, uint32_t done)
{
    using K = Cfg<C>;
    using umma::idesc_f16;
    using umma::mma_f16;
    constexpr uint32_t XG = K::XC * 128, HG = kHC * 128;
    const uint32_t R = tmem + kColTile;
    switch (stage) {
    case 0:  // F1
#pragma unroll
        for (int ks = 0; ks < K::XC / 2; ++ks)
            mma_f16(R, dadv(d.x, ks * 256), dadv(d.w1, ks * 256), idesc_f16(128, 64, 0, 0), ks > 0);
        break;
    case 1:  // F2
#pragma unroll
        for (int ks = 0; ks < kHC / 2; ++ks)
            mma_f16(R, dadv(d.h1, ks * 256), dadv(d.w2, ks * 256), idesc_f16(128, 64, 0, 0), ks > 0);
        break;
    case 2:  // F3
#pragma unroll
        for (int ks = 0; ks < kHC / 2; ++ks)
            mma_f16(R, dadv(d.h2, ks * 256), dadv(d.w3, ks * 256), idesc_f16(128, 16, 0, 0), ks > 0);
        break;
    case 3:  // B3: dH2 = dY W3; dW3^T += H2e^T dY
        mma_f16(R, d.dy, d.w3_mn, idesc_f16(128, 64, 0, 1), 0);
        break;
    case 4:  // B2: dH1 = dZ2 W2; dW2 += dZ2^T H1e
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
            mma_f16(R, dadv(d.h2, ks * 256), dadv(d.w2_mn, ks * 2 * HG), idesc_f16(128, 64, 0, 1), ks > 0);
        break;
    case 6:  // latent scatter: G0^T = Q0^T A0 (M128 N32), G1^T = Q1^T A1 (M64 N16), K = 128 samples
#pragma unroll
        for (int ks = 0; ks < kTileN / 16; ++ks)
            mma_f16(R, dadv(d.q0, ks * 2 * sc_qa(0) * 128), dadv(d.a0, ks * 2 * sc_w(0) / 8 * 128),
                    idesc_f16(128, sc_w(0), 1, 1), ks > 0);
#pragma unroll
        for (int ks = 0; ks < kTileN / 16; ++ks)
            mma_f16(R + sc_w(0), dadv(d.q1, ks * 2 * sc_qa(1) * 128), dadv(d.a1, ks * 2 * sc_w(1) / 8 * 128),
                    idesc_f16(64, sc_w(1), 1, 1), ks > 0);
        break;
    case 7:  // latent scatter, channels 8-11 (C = 12): M = 48 (grid 0) / 32 (grid 1), read as M = 64
        if constexpr (C == 12) {
#pragma unroll
            for (int ks = 0; ks < kTileN / 16; ++ks)
                mma_f16(tmem + Cols<C>::ScatB0, dadv(d.q0b, ks * 2 * sc_qb(0) * 128),
                        dadv(d.a0, ks * 2 * sc_w(0) / 8 * 128), idesc_f16(64, sc_w(0), 1, 1), ks > 0);
#pragma unroll
            for (int ks = 0; ks < kTileN / 16; ++ks)
                mma_f16(tmem + Cols<C>::ScatB1, dadv(d.q1b, ks * 2 * sc_qb(1) * 128),
                        dadv(d.a1, ks * 2 * sc_w(1) / 8 * 128), idesc_f16(64, sc_w(1), 1, 1), ks > 0);
        }
        break;
    default:  // B1: dX = dZ1 W1; dW1 += dZ1^T X
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
            mma_f16(R, dadv(d.h1, ks * 256), dadv(d.w1_mn, ks * 2 * XG), idesc_f16(128, K::NX, 0, 1), ks > 0);
        break;
    }
    umma::commit(done);
}

// Issue the weight-gradient products of B3 / B2 / B1 (stage 3 / 4 / 5) and commit them to
// `dwdone`.  They write only the dW accumulator columns; the commit covers the products of the
// calling thread alone, so they must not be issued by the thread that issues the stage.
template <int C>
__device__ __forceinline__ void issue_dw(int stage, const Descs<C> &d, uint32_t tmem, bool first, uint32_t dwdone)
{
    using K = Cfg<C>;
    using umma::idesc_f16;
    using umma::mma_f16;
    constexpr uint32_t XG = K::XC * 128, HG = kHC * 128;
    const uint32_t acc0 = first ? 0u : 1u;  // the first tile of the CTA starts the gradient sums
    if (stage == 3) {
#pragma unroll
        for (int ks = 0; ks < kTileN / 16; ++ks)
            mma_f16(tmem + Cols<C>::W3, dadv(d.h2_mn, ks * 2 * HG), dadv(d.dy_mn, ks * 512), idesc_f16(128, 16, 1, 1),
                    ks > 0 ? 1u : acc0);
    } else if (stage == 4) {
#pragma unroll
        for (int ks = 0; ks < kTileN / 16; ++ks)
            mma_f16(tmem + kColW2, dadv(d.h2_mn, ks * 2 * HG), dadv(d.h1_mn, ks * 2 * HG), idesc_f16(64, 72, 1, 1),
                    ks > 0 ? 1u : acc0);
    } else {
#pragma unroll
        for (int ks = 0; ks < kTileN / 16; ++ks)
            mma_f16(tmem + kColW1, dadv(d.h1_mn, ks * 2 * HG), dadv(d.x_mn, ks * 2 * XG), idesc_f16(64, K::XW, 1, 1),
                    ks > 0 ? 1u : acc0);
    }
    umma::commit(dwdone);
}

}  // namespace tc
}  // namespace nt

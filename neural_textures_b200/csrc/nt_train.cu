// nt_train.cu -- fused training pass: sample -> MLP forward -> weighted L2 -> MLP backward
// -> weight/bias gradient reduction -> latent-gradient accumulation, in one persistent kernel.
//
// Replaces TrainLoopPass / TrainLoop (mavenkim2/neural_textures train.cu:818-915, :979-983),
// the per-warp gradient reductions of mlp.h:101-220 and the per-sample latent scatter of
// train.cu:460-509.
//
// Work decomposition.  A CTA of 8 warps owns a 16 x 16 tile of lattice cells (one jittered
// sample per cell, 256 samples) at a time and loops over tiles (persistent grid, one CTA
// per SM).
//  * gather: every thread gathers one sample (both latent grids + the target, Catmull-Rom,
//    16-byte loads) and records its footprints (base texel + 4 + 4 weights per grid);
//  * MLP: every warp runs the three layers forward and backward for its 32 rows with fp16
//    tensor-core MMAs and fp32 accumulation;
//  * weight gradients: each warp owns a fixed slice of dW1 / dW2 / dW3 and accumulates it
//    in registers across every tile it processes, so the global weight-gradient buffers
//    see one atomic per element per CTA (the reference adds per warp and step);
//  * latent gradients ("dual gather"): instead of 16 taps x C atomics per sample, each
//    texel of the tile's footprint window sums the contributions of the samples whose
//    footprint covers it, read from shared memory (candidate cells form a contiguous range
//    per window row / column because sample positions are monotonic in the lattice index),
//    and adds the window to the global gradient with one float4 reduction per 4 channels.
//    Texels on a window border also receive contributions from neighbouring tiles; the
//    reductions make those sums exact.
#include <climits>
#include <cstdlib>
#include <cstring>

#include "nt_mlp_smem.cuh"

namespace nt {

constexpr int kMaxWin = 64;  // window side cap; larger footprints fall back to per-tap atomics

struct GridWindow {
    int32_t x0, y0;            // first window texel (unwrapped)
    int32_t w, h;              // window size (0 when the fallback is used)
    int32_t span;              // longest candidate range (cells) over window columns
    int32_t sweep_ok;          // every lattice row / column spans at most two base texels
    int32_t cand_x[kMaxWin];   // per window column: lo | hi << 16 of candidate lattice columns
    int32_t cand_y[kMaxWin];
};

struct TrainSmem {
    MlpSmem mlp;
    __half X[kTileSamples * kStrideK32];    // MLP input
    __half H1[kTileSamples * kStrideK64];   // layer-1 output (post-ReLU)
    __half H2[kTileSamples * kStrideK64];   // layer-2 output, later dL/dH1
    __half DY[kTileSamples * kStrideK16];   // fp16 output, later dL/dY (x num_samples)
    __half DH2[kTileSamples * kStrideK64];  // dL/dH2, later dL/dX (fp32, 36 floats per row)
    short2 base[2][kTileSamples];           // footprint base texel per grid and sample
    float wts[2][kTileSamples][8];          // wx[4], wy[4] per grid and sample
    int32_t part[2][4][kThreads / 32][kTileSide];  // per-warp min / max of footprint bases
    int32_t fin[2][4][kTileSide];           // per lattice column / row: min, max base
    GridWindow win[2];
    float red[kThreads / 32];
};

constexpr int kDxStride = kStrideK64 / 2;  // floats per dX row (same bytes as a DH2 row)

// Mask fp32 accumulators (rows r0.., NT n8 tiles) with the ReLU of `act` (post-activation
// fp16 matrix at the same positions), round to fp16 A fragments and store them to `dst`.
template <int NT>
__device__ __forceinline__ void mask_relu_store(const float (&acc)[2][NT][4], const __half *act,
                                                __half *dst, uint32_t (&a)[2][NT / 2][4], int r0,
                                                int lane)
{
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int off0 = (r0 + mt * 16 + g) * kStrideK64 + nt * 8 + 2 * t;
            const int off1 = off0 + 8 * kStrideK64;
            const float2 h0 = unpack_half2(*reinterpret_cast<const uint32_t *>(act + off0));
            const float2 h1 = unpack_half2(*reinterpret_cast<const uint32_t *>(act + off1));
            const uint32_t p0 = pack_half2(h0.x > 0.f ? acc[mt][nt][0] : 0.f, h0.y > 0.f ? acc[mt][nt][1] : 0.f);
            const uint32_t p1 = pack_half2(h1.x > 0.f ? acc[mt][nt][2] : 0.f, h1.y > 0.f ? acc[mt][nt][3] : 0.f);
            *reinterpret_cast<uint32_t *>(dst + off0) = p0;
            *reinterpret_cast<uint32_t *>(dst + off1) = p1;
            a[mt][nt >> 1][(nt & 1) * 2 + 0] = p0;
            a[mt][nt >> 1][(nt & 1) * 2 + 1] = p1;
        }
}

// Per-warp min / max of the footprint bases of each lattice column (lanes L, L+16 share a
// column) and of each lattice row (half-warp), written to s.part.  Invalid samples
// contribute the neutral values.
__device__ __forceinline__ void footprint_extents(TrainSmem &s, int gi, int bx, int by, bool valid, int warp,
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
        s.part[gi][0][warp][lane] = cmin;
        s.part[gi][1][warp][lane] = cmax;
    }
    if ((lane & 15) == 0) {  // lattice row of this half-warp = 2 warp + lane / 16
        s.part[gi][2][warp][lane >> 4] = rmin;
        s.part[gi][3][warp][lane >> 4] = rmax;
    }
}

// One warp finalises the window of grid gi: column / row extents over the 8 warp partials,
// window origin and size, and the candidate lattice range of every window column / row.
__device__ __forceinline__ void finalize_window(TrainSmem &s, int gi, int lane)
{
    const int nw = kThreads / 32;
    const int e = lane & 15;
    int lo_v, hi_v;
    if (lane < 16) {  // lattice column e
        lo_v = INT_MAX;
        hi_v = INT_MIN;
        for (int w = 0; w < nw; ++w) {
            lo_v = min(lo_v, s.part[gi][0][w][e]);
            hi_v = max(hi_v, s.part[gi][1][w][e]);
        }
    } else {  // lattice row e: rows 2w and 2w + 1 live in warp w
        const int w = e >> 1, half = e & 1;
        lo_v = s.part[gi][2][w][half];
        hi_v = s.part[gi][3][w][half];
    }
    s.fin[gi][lane < 16 ? 0 : 2][e] = lo_v;
    s.fin[gi][lane < 16 ? 1 : 3][e] = hi_v;
    // the column sweep needs every valid lattice column / row to span <= 2 base texels
    const bool narrow = lo_v == INT_MAX || (long long)hi_v - lo_v <= 1;
    const bool all_narrow = __all_sync(0xffffffffu, narrow);
    __syncwarp();
    // window extents: columns over lanes 0..15, rows over lanes 16..31
    int mn = lo_v, mx = hi_v;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
        mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const int cmin = __shfl_sync(0xffffffffu, mn, 0), cmax = __shfl_sync(0xffffffffu, mx, 0);
    const int rmin = __shfl_sync(0xffffffffu, mn, 16), rmax = __shfl_sync(0xffffffffu, mx, 16);
    GridWindow &W = s.win[gi];
    const bool nonempty = cmin <= cmax && rmin <= rmax;
    const int ww = nonempty ? cmax - cmin + 4 : 0, wh = nonempty ? rmax - rmin + 4 : 0;
    const bool ok = nonempty && ww <= kMaxWin && wh <= kMaxWin;
    if (lane == 0) {
        W.x0 = cmin - 1;
        W.y0 = rmin - 1;
        W.w = ok ? ww : 0;
        W.h = ok ? wh : 0;
    }
    if (!ok) {
        if (lane == 0) {
            W.span = 0;
            W.sweep_ok = 0;
        }
        return;
    }
    // candidate cells of window column tx: lattice columns c with colmin[c] <= tx + 1 and
    // colmax[c] >= tx - 2 (both monotonic in c, so the set is a contiguous range)
    int span = 0;
    for (int k = lane; k < kMaxWin * 2; k += 32) {
        const bool isx_span = k < kMaxWin;
        const bool isx = k < kMaxWin;
        const int idx = isx ? k : k - kMaxWin;
        if (idx >= (isx ? ww : wh)) continue;
        const int tcoord = (isx ? cmin : rmin) - 1 + idx;
        int lo = kTileSide, hi = -1;
        const int *fmin = s.fin[gi][isx ? 0 : 2], *fmax = s.fin[gi][isx ? 1 : 3];
        for (int c = 0; c < kTileSide; ++c) {
            if (fmin[c] <= tcoord + 1 && fmax[c] >= tcoord - 2) {
                lo = min(lo, c);
                hi = max(hi, c);
            }
        }
        (isx ? W.cand_x : W.cand_y)[idx] = lo | (hi << 16);
        if (isx_span) span = max(span, hi - lo + 1);
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) span = max(span, __shfl_xor_sync(0xffffffffu, span, o));
    if (lane == 0) {
        W.span = span;
        W.sweep_ok = all_narrow;
    }
}

// Latent-gradient column sweep.  Task = (grid, pair of lattice rows, window column tx).
// For lattice row cj the footprints of its samples cover texel rows fy .. fy + 4 with
// fy = min base row - 1 (each sample's base row is fy + 1 or fy + 2).  The task walks its
// candidate cells (the lattice columns whose footprints can cover tx, at most L of them),
// forms w_x * dX once per candidate and adds w_y * (w_x * dX) into a 5-row register window
// R aligned to fy; moving to the next lattice row shifts R by the change of fy and flushes
// the rows that no later lattice row can reach.  Every flush is one float4 reduction per 4
// channels into the global gradient.  Loads are unconditional (weights are zero where a
// candidate does not cover the texel), so all candidates of a row are independent.
template <int C>
__device__ __forceinline__ void sweep_flush_row(const TrainLaunch &p, int gi, int tx, int ty, const float (&row)[C])
{
    bool any = false;
#pragma unroll
    for (int c = 0; c < C; ++c) any |= row[c] != 0.f;
    if (!any) return;
    const int gw = p.gw[gi], gh = p.gh[gi];
    const float sc = p.inv_num_samples;
    float4 *dst = reinterpret_cast<float4 *>(p.ggrid[gi] + ((size_t)wrap_coord(ty, gh) * gw + wrap_coord(tx, gw)) * C);
#pragma unroll
    for (int q = 0; q < C / 4; ++q)
        atomicAdd(dst + q, make_float4(row[4 * q] * sc, row[4 * q + 1] * sc, row[4 * q + 2] * sc, row[4 * q + 3] * sc));
}

template <int C>
__device__ __forceinline__ void sweep_shift(const TrainLaunch &p, int gi, int tx, int fy, float (&R)[5][C])
{
    sweep_flush_row<C>(p, gi, tx, fy, R[0]);
#pragma unroll
    for (int m = 0; m < 4; ++m)
#pragma unroll
        for (int c = 0; c < C; ++c) R[m][c] = R[m + 1][c];
#pragma unroll
    for (int c = 0; c < C; ++c) R[4][c] = 0.f;
}

template <int C, int L>
__device__ __forceinline__ void latent_bwd_sweep(const TrainSmem &s, const TrainLaunch &p, int tid)
{
    constexpr int kRowsPerTask = 2;
    constexpr int kChunks = kTileSide / kRowsPerTask;
    const float *dx = reinterpret_cast<const float *>(s.DH2);
    const int nt0 = s.win[0].w * kChunks;
    const int ntot = nt0 + s.win[1].w * kChunks;
    for (int k = tid; k < ntot; k += kThreads) {
        const int gi = k < nt0 ? 0 : 1;
        const GridWindow &W = s.win[gi];
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
        for (int r = 0; r < kRowsPerTask; ++r) {
            const int cj = chunk * kRowsPerTask + r;
            const int rmin = s.fin[gi][2][cj];
            if (rmin == INT_MAX) continue;  // no valid sample in this lattice row
            const int fy = rmin - 1;
            if (fy_cur == INT_MIN) fy_cur = fy;
            while (fy > fy_cur) {  // rows below fy are complete (lattice rows are monotonic)
                sweep_shift<C>(p, gi, tx, fy_cur, R);
                ++fy_cur;
            }
#pragma unroll
            for (int b = 0; b < L; ++b) {
                const int ci = min(lo + b, kTileSide - 1);
                const bool inr = lo + b <= hi;
                const int sidx = cj * kTileSide + ci;
                const short2 bs = s.base[gi][sidx];
                const int kx = tx - bs.x + 1;
                const float wxv = (inr && (unsigned)kx <= 3u) ? s.wts[gi][sidx][kx & 3] : 0.f;
                const float4 wy = *reinterpret_cast<const float4 *>(&s.wts[gi][sidx][4]);
                const bool e1 = bs.y - 1 - fy != 0;  // base row fy + 2 (else fy + 1)
                float wxd[C];
                const float4 *d4 = reinterpret_cast<const float4 *>(dx + sidx * kDxStride + gi * C);
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
        for (int m = 0; m < 5; ++m) sweep_flush_row<C>(p, gi, tx, fy_cur + m, R[m]);
    }
}

// Dual gather with a fixed candidate stencil of L x L cells (L >= the longest candidate
// range of the tile): fully unrolled, loads independent of one another, the fp32 dX rows
// read only for candidates whose footprint covers the texel.  Texels of both grids share
// one index space so that all threads stay busy.
template <int C, int L>
__device__ __forceinline__ void window_accumulate_stencil(const TrainSmem &s, const TrainLaunch &p, int tid)
{
    const float *dx = reinterpret_cast<const float *>(s.DH2);
    const int n0 = s.win[0].w * s.win[0].h;
    const int n = n0 + s.win[1].w * s.win[1].h;
    for (int k = tid; k < n; k += kThreads) {
        const int gi = k < n0 ? 0 : 1;
        const GridWindow &W = s.win[gi];
        const int kk = gi ? k - n0 : k;
        const int lx = kk % W.w, ly = kk / W.w;
        const int tx = W.x0 + lx, ty = W.y0 + ly;
        const int cx = W.cand_x[lx], cy = W.cand_y[ly];
        const int cx0 = cx & 0xffff, cx1 = cx >> 16, cy0 = cy & 0xffff, cy1 = cy >> 16;
        float acc[C];
#pragma unroll
        for (int c = 0; c < C; ++c) acc[c] = 0.f;
#pragma unroll
        for (int a = 0; a < L; ++a) {
            const int cj = cy0 + a;
            const bool rowok = cj <= cy1;
            const int cjc = min(rowok ? cj : cy0, kTileSide - 1);
#pragma unroll
            for (int b = 0; b < L; ++b) {
                const int ci = cx0 + b;
                const bool ok = rowok && ci <= cx1;
                const int sidx = cjc * kTileSide + min(ok ? ci : cx0, kTileSide - 1);
                const short2 bs = s.base[gi][sidx];
                const int jx = tx - bs.x + 1, jy = ty - bs.y + 1;
                const bool hit = ok && (unsigned)jx <= 3u && (unsigned)jy <= 3u;
                if (hit) {
                    const float wgt = s.wts[gi][sidx][jx] * s.wts[gi][sidx][4 + jy];
                    const float4 *d4 = reinterpret_cast<const float4 *>(dx + sidx * kDxStride + gi * C);
#pragma unroll
                    for (int q = 0; q < C / 4; ++q) {
                        const float4 d = d4[q];
                        acc[4 * q + 0] = fmaf(wgt, d.x, acc[4 * q + 0]);
                        acc[4 * q + 1] = fmaf(wgt, d.y, acc[4 * q + 1]);
                        acc[4 * q + 2] = fmaf(wgt, d.z, acc[4 * q + 2]);
                        acc[4 * q + 3] = fmaf(wgt, d.w, acc[4 * q + 3]);
                    }
                }
            }
        }
        if (cx1 < cx0 || cy1 < cy0) continue;
        const int gw = p.gw[gi], gh = p.gh[gi];
        const float scale = p.inv_num_samples;
        float4 *dst = reinterpret_cast<float4 *>(p.ggrid[gi] + ((size_t)wrap_coord(ty, gh) * gw + wrap_coord(tx, gw)) * C);
#pragma unroll
        for (int q = 0; q < C / 4; ++q)
            atomicAdd(dst + q, make_float4(acc[4 * q] * scale, acc[4 * q + 1] * scale, acc[4 * q + 2] * scale,
                                           acc[4 * q + 3] * scale));
    }
}

template <int C>
__device__ __forceinline__ void window_accumulate(const TrainSmem &s, int gi, float *__restrict__ ggrid, int gw,
                                                  int gh, float scale, int tid)
{
    const GridWindow &W = s.win[gi];
    const float *dx = reinterpret_cast<const float *>(s.DH2);
    const int n = W.w * W.h;
    for (int k = tid; k < n; k += kThreads) {
        const int lx = k % W.w, ly = k / W.w;
        const int tx = W.x0 + lx, ty = W.y0 + ly;
        const int cx = W.cand_x[lx], cy = W.cand_y[ly];
        const int cx0 = cx & 0xffff, cx1 = cx >> 16, cy0 = cy & 0xffff, cy1 = cy >> 16;
        float acc[C];
#pragma unroll
        for (int c = 0; c < C; ++c) acc[c] = 0.f;
        bool any = false;
        for (int cj = cy0; cj <= cy1; ++cj) {
            for (int ci = cx0; ci <= cx1; ++ci) {
                const int sidx = cj * kTileSide + ci;
                const short2 b = s.base[gi][sidx];
                const int jx = tx - b.x + 1, jy = ty - b.y + 1;
                if ((unsigned)jx > 3u || (unsigned)jy > 3u) continue;
                const float wgt = s.wts[gi][sidx][jx] * s.wts[gi][sidx][4 + jy];
                const float4 *d4 = reinterpret_cast<const float4 *>(dx + sidx * kDxStride + gi * C);
#pragma unroll
                for (int q = 0; q < C / 4; ++q) {
                    const float4 d = d4[q];
                    acc[4 * q + 0] = fmaf(wgt, d.x, acc[4 * q + 0]);
                    acc[4 * q + 1] = fmaf(wgt, d.y, acc[4 * q + 1]);
                    acc[4 * q + 2] = fmaf(wgt, d.z, acc[4 * q + 2]);
                    acc[4 * q + 3] = fmaf(wgt, d.w, acc[4 * q + 3]);
                }
                any = true;
            }
        }
        if (!any) continue;
        float4 *dst = reinterpret_cast<float4 *>(ggrid + ((size_t)wrap_coord(ty, gh) * gw + wrap_coord(tx, gw)) * C);
#pragma unroll
        for (int q = 0; q < C / 4; ++q)
            atomicAdd(dst + q, make_float4(acc[4 * q] * scale, acc[4 * q + 1] * scale, acc[4 * q + 2] * scale,
                                           acc[4 * q + 3] * scale));
    }
}

// Fallback for footprints wider than the window cap: per-sample, per-tap vector atomics.
template <int C>
__device__ __forceinline__ void scatter_taps(const TrainSmem &s, int gi, float *__restrict__ ggrid, int gw, int gh,
                                             float scale, int tid, bool valid)
{
    if (!valid) return;
    const float *dxr = reinterpret_cast<const float *>(s.DH2) + tid * kDxStride + gi * C;
    const short2 b = s.base[gi][tid];
    for (int j = 0; j < 4; ++j) {
        const int yy = wrap_coord(b.y - 1 + j, gh);
        for (int i = 0; i < 4; ++i) {
            const int xx = wrap_coord(b.x - 1 + i, gw);
            const float wgt = s.wts[gi][tid][i] * s.wts[gi][tid][4 + j] * scale;
            float4 *dst = reinterpret_cast<float4 *>(ggrid + ((size_t)yy * gw + xx) * C);
#pragma unroll
            for (int q = 0; q < C / 4; ++q)
                atomicAdd(dst + q, make_float4(wgt * dxr[4 * q], wgt * dxr[4 * q + 1], wgt * dxr[4 * q + 2],
                                               wgt * dxr[4 * q + 3]));
        }
    }
}

template <int C, int NT3>
__global__ void __launch_bounds__(kThreads, 1) train_kernel(const TrainLaunch p)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    TrainSmem &s = *reinterpret_cast<TrainSmem *>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    constexpr int NTX = ((2 * C + 15) / 16) * 2;  // n8 tiles of dL/dX covering the latents

    stage_weights(s.mlp, p.net);

    float aw2[4][4], aw3[4], aw1[2][4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        aw3[e] = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) aw2[q][e] = 0.f;
        aw1[0][e] = aw1[1][e] = 0.f;
    }
    float adb1 = 0.f, adb2 = 0.f, adb3 = 0.f, sse = 0.f;
    __syncthreads();

    const uint32_t sX = smem_addr(s.X), sH1 = smem_addr(s.H1), sH2 = smem_addr(s.H2);
    const uint32_t sDY = smem_addr(s.DY), sDH2 = smem_addr(s.DH2);
    const int ntiles = p.tiles_x * p.tiles_y;
    const int r0 = warp * 32;

    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int ix = (tile % p.tiles_x) * kTileSide + (tid & (kTileSide - 1));
        const int iy = (tile / p.tiles_x) * kTileSide + tid / kTileSide;
        const bool valid = ix < p.sampler.lattice_w && iy < p.sampler.lattice_h;
        float tgt[16];

        // ---- gather: one sample per thread -------------------------------------------
        {
            uint32_t packed[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) packed[k] = 0u;
#pragma unroll
            for (int k = 0; k < 16; ++k) tgt[k] = 0.f;
            float u = 0.f, v = 0.f;
            if (valid) sample_uv(p.sampler, ix, iy, u, v);
#pragma unroll
            for (int gi = 0; gi < 2; ++gi) {
                Footprint fp;
                footprint(u, v, p.gw[gi], p.gh[gi], fp);
                if (valid) {
                    float f[C];
                    gather_cr<C>(p.grid[gi], p.gw[gi], fp, f);
#pragma unroll
                    for (int k = 0; k < C / 2; ++k) packed[gi * (C / 2) + k] = pack_half2(f[2 * k], f[2 * k + 1]);
                }
                s.base[gi][tid] = make_short2((short)fp.bx, (short)fp.by);
                float4 *wr = reinterpret_cast<float4 *>(s.wts[gi][tid]);
                wr[0] = make_float4(fp.wx[0], fp.wx[1], fp.wx[2], fp.wx[3]);
                wr[1] = make_float4(fp.wy[0], fp.wy[1], fp.wy[2], fp.wy[3]);
                footprint_extents(s, gi, fp.bx, fp.by, valid && !p.finalize, warp, lane);
            }
            if (valid) {
                float pe[8];
                posenc(u, v, pe);
#pragma unroll
                for (int k = 0; k < 4; ++k) packed[C + k] = pack_half2(pe[2 * k], pe[2 * k + 1]);
                Footprint fp;
                footprint(u, v, p.tw, p.th, fp);
                gather_target(p.target, p.tw, p.net.cout, fp, tgt);
            }
            uint4 *xr = reinterpret_cast<uint4 *>(s.X + tid * kStrideK32);
#pragma unroll
            for (int q = 0; q < 4; ++q)
                xr[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
        __syncwarp();

        // ---- forward (this warp's 32 rows) ----------------------------------------------
        {
            float acc3[2][NT3][4];
            warp_forward<NT3>(s.mlp, s.X, s.H1, s.H2, r0, lane, acc3);
            store_out16<NT3>(acc3, s.DY, r0, lane);
        }
        __syncwarp();

        // ---- loss: weighted L2 (train.cu:876-888), gradient 2 w err kept unscaled ------
        {
            uint4 *dyr = reinterpret_cast<uint4 *>(s.DY + tid * kStrideK16);
            uint4 yv[2] = {dyr[0], dyr[1]};
            const uint32_t *yw = reinterpret_cast<const uint32_t *>(yv);
            uint32_t out[8];
#pragma unroll
            for (int c2 = 0; c2 < 8; ++c2) {
                const float2 y = unpack_half2(yw[c2]);
                float d[2] = {0.f, 0.f};
                const float yy[2] = {y.x, y.y};
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int c = 2 * c2 + e;
                    if (valid && c < NT3 * 8 && c < p.net.cout) {
                        const float err = yy[e] - tgt[c];
                        sse = fmaf(p.cw[c] * err, err, sse);
                        d[e] = 2.f * p.cw[c] * err;
                    }
                }
                out[c2] = pack_half2(d[0], d[1]);
            }
            dyr[0] = make_uint4(out[0], out[1], out[2], out[3]);
            dyr[1] = make_uint4(out[4], out[5], out[6], out[7]);
        }
        __syncwarp();

        // ---- backward 1: dH2 = (dY W3^T) * [H2 > 0] -------------------------------------
        {
            uint32_t da[2][1][4];
            load_a<2, 1>(da, sDY, kStrideK16, r0, lane);
            float acc[2][8][4];
            acc_init_bias<2, 8>(acc, nullptr, lane);
            warp_gemm_wt<2, 1, 8>(acc, da, smem_addr(s.mlp.W3), kStrideK64, lane);
            uint32_t dh2a[2][4][4];
            mask_relu_store<8>(acc, s.H2, s.DH2, dh2a, r0, lane);
        }
        __syncthreads();

        // ---- phase A: dW2 += H1^T dH2, dW3 += H2^T dY, db2, db3 (all 256 samples) -------
        {
            if (warp < 2 && !p.finalize) finalize_window(s, warp, lane);
            const int mi = warp & 3, nj0 = (warp >> 2) * 4;
#pragma unroll 4
            for (int ks = 0; ks < kTileSamples / 16; ++ks) {
                uint32_t a[4], b[4];
                ldsm_x4_t(a, at_frag_addr(sH1, kStrideK64, ks * 16, mi * 16, lane));
                ldsm_x4_t(b, bt_frag2n_addr(sDH2, kStrideK64, ks * 16, nj0 * 8, lane));
                mma16816(aw2[0], a, b[0], b[1]);
                mma16816(aw2[1], a, b[2], b[3]);
                ldsm_x4_t(b, bt_frag2n_addr(sDH2, kStrideK64, ks * 16, (nj0 + 2) * 8, lane));
                mma16816(aw2[2], a, b[0], b[1]);
                mma16816(aw2[3], a, b[2], b[3]);
            }
            if (warp < 4 * NT3) {
                const int mi3 = warp & 3, nc = warp >> 2;
#pragma unroll 4
                for (int ks = 0; ks < kTileSamples / 16; ++ks) {
                    uint32_t a[4], b[2];
                    ldsm_x4_t(a, at_frag_addr(sH2, kStrideK64, ks * 16, mi3 * 16, lane));
                    const int row = ks * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
                    ldsm_x2_t(b, sDY + 2u * (uint32_t)(row * kStrideK16 + nc * 8));
                    mma16816(aw3, a, b[0], b[1]);
                }
            }
            {
                const int col = tid & 63, rbase = (tid >> 6) * 64;
                float sacc = 0.f;
#pragma unroll 8
                for (int r = 0; r < 64; ++r) sacc += __half2float(s.DH2[(rbase + r) * kStrideK64 + col]);
                adb2 += sacc;
            }
            {
                const int col = tid & 15, rbase = (tid >> 4) * 16;
                float sacc = 0.f;
#pragma unroll 8
                for (int r = 0; r < 16; ++r) sacc += __half2float(s.DY[(rbase + r) * kStrideK16 + col]);
                adb3 += sacc;
            }
        }
        __syncthreads();

        // ---- backward 2: dH1 = (dH2 W2^T) * [H1 > 0] -> H2 buffer; dX = dH1 W1^T --------
        {
            uint32_t da[2][4][4];
            load_a<2, 4>(da, sDH2, kStrideK64, r0, lane);
            float acc[2][8][4];
            acc_init_bias<2, 8>(acc, nullptr, lane);
            warp_gemm_wt<2, 4, 8>(acc, da, smem_addr(s.mlp.W2), kStrideK64, lane);
            uint32_t dh1a[2][4][4];
            mask_relu_store<8>(acc, s.H1, s.H2, dh1a, r0, lane);
            float ax[2][NTX][4];
            acc_init_bias<2, NTX>(ax, nullptr, lane);
            warp_gemm_wt<2, 4, NTX>(ax, dh1a, smem_addr(s.mlp.W1), kStrideK32, lane);
            __syncwarp();
            float *dx = reinterpret_cast<float *>(s.DH2);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < NTX; ++nt) {
                    float *q0 = dx + (r0 + mt * 16 + g) * kDxStride + nt * 8 + 2 * t;
                    *reinterpret_cast<float2 *>(q0) = make_float2(ax[mt][nt][0], ax[mt][nt][1]);
                    *reinterpret_cast<float2 *>(q0 + 8 * kDxStride) = make_float2(ax[mt][nt][2], ax[mt][nt][3]);
                }
        }
        __syncthreads();

        // ---- phase B: dW1 += X^T dH1, db1 -------------------------------------------------
        {
            const int mi = warp & 1, nj0 = (warp >> 1) * 2;
#pragma unroll 4
            for (int ks = 0; ks < kTileSamples / 16; ++ks) {
                uint32_t a[4], b[4];
                ldsm_x4_t(a, at_frag_addr(sX, kStrideK32, ks * 16, mi * 16, lane));
                ldsm_x4_t(b, bt_frag2n_addr(sH2, kStrideK64, ks * 16, nj0 * 8, lane));
                mma16816(aw1[0], a, b[0], b[1]);
                mma16816(aw1[1], a, b[2], b[3]);
            }
            const int col = tid & 63, rbase = (tid >> 6) * 64;
            float sacc = 0.f;
#pragma unroll 8
            for (int r = 0; r < 64; ++r) sacc += __half2float(s.H2[(rbase + r) * kStrideK64 + col]);
            adb1 += sacc;
        }

        // ---- latent gradients: dual gather over the tile's footprint windows --------------
        if (!p.finalize) {
            const bool both = s.win[0].w > 0 && s.win[1].w > 0 && s.win[0].sweep_ok && s.win[1].sweep_ok;
            const int span = max(s.win[0].span, s.win[1].span);
            if (both && span <= 5) {
                latent_bwd_sweep<C, 5>(s, p, tid);
            } else if (both && span <= 10) {
                latent_bwd_sweep<C, 10>(s, p, tid);
            } else {
#pragma unroll
                for (int gi = 0; gi < 2; ++gi) {
                    if (s.win[gi].w > 0)
                        window_accumulate<C>(s, gi, p.ggrid[gi], p.gw[gi], p.gh[gi], p.inv_num_samples, tid);
                    else
                        scatter_taps<C>(s, gi, p.ggrid[gi], p.gw[gi], p.gh[gi], p.inv_num_samples, tid, valid);
                }
            }
        }
        __syncthreads();
    }

    // ---- flush the per-CTA partial gradients (scaled by 1 / num_samples) ------------------
    const float sc = p.inv_num_samples;
    {
        const int mi = warp & 3, nj0 = (warp >> 2) * 4;
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int in = mi * 16 + g + 8 * (e >> 1);
                const int out = (nj0 + q) * 8 + 2 * t + (e & 1);
                atomicAdd(p.gW[1] + out * 64 + in, aw2[q][e] * sc);
            }
    }
    if (warp < 4 * NT3) {
        const int mi3 = warp & 3, nc = warp >> 2;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int hid = mi3 * 16 + g + 8 * (e >> 1);
            const int out = nc * 8 + 2 * t + (e & 1);
            if (out < p.net.cout) atomicAdd(p.gW[2] + out * 64 + hid, aw3[e] * sc);
        }
    }
    {
        const int mi = warp & 1, nj0 = (warp >> 1) * 2;
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int in = mi * 16 + g + 8 * (e >> 1);
                const int hid = (nj0 + q) * 8 + 2 * t + (e & 1);
                atomicAdd(p.gW[0] + hid * 32 + in, aw1[q][e] * sc);
            }
    }
    atomicAdd(p.gb[0] + (tid & 63), adb1 * sc);
    atomicAdd(p.gb[1] + (tid & 63), adb2 * sc);
    if ((tid & 15) < p.net.cout) atomicAdd(p.gb[2] + (tid & 15), adb3 * sc);
    if (p.loss_accum) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sse += __shfl_xor_sync(0xffffffffu, sse, o);
        if (lane == 0) s.red[warp] = sse;
        __syncthreads();
        if (tid == 0) {
            float tot = 0.f;
            for (int w = 0; w < kThreads / 32; ++w) tot += s.red[w];
            atomicAdd(p.loss_accum, tot);
        }
    }
}

template <int C, int NT3>
static cudaError_t launch_train_t(const TrainLaunch &p, cudaStream_t stream)
{
    const size_t smem = sizeof(TrainSmem);
    cudaError_t e = set_smem_limit(reinterpret_cast<const void *>(train_kernel<C, NT3>), smem);
    if (e != cudaSuccess) return e;
    const int ntiles = p.tiles_x * p.tiles_y;
    const int grid = ntiles < sm_count() ? ntiles : sm_count();
    train_kernel<C, NT3><<<grid, kThreads, smem, stream>>>(p);
    count_launch();
    return cudaGetLastError();
}

int train_engine()
{
    static const int engine = [] {
        const char *e = getenv("NT_TRAIN_ENGINE");
        return (e && strcmp(e, "mma") == 0) ? 0 : 1;
    }();
    return engine;
}

cudaError_t launch_train(const TrainLaunch &p, int channels, cudaStream_t stream)
{
    if (train_engine() == 1) return launch_train_tc(p, channels, stream);
    const bool wide = p.net.cout > 8;
    if (channels == 8) return wide ? launch_train_t<8, 2>(p, stream) : launch_train_t<8, 1>(p, stream);
    if (channels == 12) return wide ? launch_train_t<12, 2>(p, stream) : launch_train_t<12, 1>(p, stream);
    return cudaErrorInvalidValue;
}

}  // namespace nt

// nt_train_tc.cu -- fused training pass on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Contract (TrainLoopPass / TrainLoop,
// mavenkim2/neural_textures train.cu:818-915, :979-983; mlp.h:101-257 backward; the latent
// scatter of train.cu:460-509): one jittered sample per lattice cell, weighted L2 loss,
// weight / bias / latent gradients accumulated (x 1 / num_samples) into fp32 buffers.
//
// Work decomposition.  A CTA of 8 warps owns one tile of 16 x 8 lattice cells (128
// samples, M = 128, sample s = TMEM lane s) at a time; two CTAs share an SM, so one CTA's
// gathers and epilogues overlap the other's tensor-core products.  Thread t works on sample
// t % 128; the two threads of a sample split the gathers (latent grids / target and
// positional features) and the epilogue columns (warps w and w + 4 read the same TMEM
// lanes).  Per tile:
//     gather -> F1 -> E1 -> F2 -> E2 -> F3 -> E3 (loss) -> B3 -> E4 -> B2 -> E5 -> B1 -> E6
// Fk / Bk are tensor-core products that thread 0 issues after a CTA barrier (operands in
// shared memory, fenced to the async proxy); Ek are epilogues (TMEM -> registers -> fp16
// operand tiles in shared memory).
//
// Tensor-core products per tile (fp16 x fp16 -> fp32; operands in the no-swizzle
// core-matrix layout of nt_umma.cuh):
//   F1  Z1   = X  W1e^T          M128 N64  K=XW   (X carries a constant-1 column, W1e the
//                                                  bias b1 in that column)
//   F2  Z2   = H1e W2e^T         M128 N64  K80    (H1e = [relu(Z1) | 1 | 0...])
//   F3  Y    = H2e W3e^T         M128 N16  K80
//   B3  dH2  = dY W3             M128 N64  K16    (W3e read MN-major: no transpose)
//       dW3^T += H2e^T dY        M128 N16  K128   (row 64 of the result is db3)
//   B2  dH1  = dZ2 W2            M128 N64  K64
//       dW2  += dZ2^T H1e        M64  N72  K128   (column 64 is db2)
//   B1  dX   = dZ1 W1            M128 NX   K64
//       dW1  += dZ1^T X          M64  N=XW K128   (column 2C + 8 is db1)
// The weight-gradient accumulators stay in TMEM for the whole kernel and each CTA adds
// them to global memory once at the end (float4 reductions).  The activation tiles are
// stored once as [samples][features] and read K-major by the forward products and
// MN-major by the gradient products.
//
// Latent gradients: dX rows go to shared memory and a column sweep over the tile's
// footprint window accumulates them per texel before one float4 reduction per 4 channels
// (per-tap vector atomics when a window does not fit).  Block features (BLK) take the same
// per-texel sums through the BC6 backward into the block records, once per window texel
// instead of once per tap.
//
// Every wait is bounded.  A timeout sets bit 0 of the device status word (read back by
// nt_read_device_status); the CTA agrees on it at its next barrier, stops issuing work,
// waits (bounded) for the products in flight and releases its tensor memory.
#include <climits>
#include <cmath>

#include "nt_kernels.cuh"
#include "nt_mma.cuh"
#include "nt_bc6f.cuh"
#include "nt_tc_common.cuh"
#include "nt_umma.cuh"

#include "nt_train_tc.cuh"

namespace nt {

namespace tc {

template <int C>
struct Smem {
    alignas(128) uint8_t W1[64 * Cfg<C>::XW * 2];  // [out][in | b1 | 0]
    alignas(128) uint8_t W2[64 * kHW * 2];         // [out][in | b2 | 0]
    alignas(128) uint8_t W3[16 * kHW * 2];         // [out (zero rows past cout)][in | b3 | 0]
    union {
        struct {  // the network's operand tiles
            alignas(128) uint8_t X[kTileN * Cfg<C>::XW * 2];
            alignas(128) uint8_t H1[kTileN * kHW * 2];  // H1e, then dZ1 (in place)
            alignas(128) uint8_t H2[kTileN * kHW * 2];  // H2e, then dZ2 (in place), then dX (fp32)
            alignas(128) uint8_t DY[kTileN * 16 * 2];   // follows H2: the M = 128 read of H2 runs 768 B past it
        } m;
        struct {  // latent scatter operands: Q_g = wy dX over window rows, A_g = wx over window columns
            // (each Q tile is followed by another operand: its M = 128 / 64 read runs past its end)
            alignas(128) uint8_t Q0[kTileN * sc_qa(0) * 16];
            alignas(128) uint8_t Q1[kTileN * sc_qa(1) * 16];
            alignas(128) uint8_t A0[kTileN * sc_w(0) * 2];
            alignas(128) uint8_t A1[kTileN * sc_w(1) * 2];
        } q;
        struct {  // the scattered window sums, fp32 [row][column (+1 pad)][channel]
            float g0[sc_h(0) * (sc_w(0) + 1) * C];
            float g1[sc_h(1) * (sc_w(1) + 1) * C];
        } f;
    } t;
    short2 base[2][kTileN];
    float wts[2][kTileN][8];
    int32_t part[2][4][4][kTileW];  // [grid][col min, col max, row min, row max][warp][index]
    int32_t colext[2][2][kTileW];
    int32_t rowmin[2][kTileH];
    Window win[2];
    alignas(8) uint64_t done, dwdone;  // stage products; weight-gradient products of B3 / B2 / B1
    uint32_t tmem_base;
    int32_t next_tile;  // with a tile counter: the CTA's next tile (written by the last thread)
    float red[kThreadsTC / 32];
};

// TMEM -> fp32 staging of the window sums (thread: one (row, channel) lane, 16 columns).
// Channels 0-7: grid 0 M = 128 (lane m = 8 y + c), grid 1 M = 64 (row m = 16 q + lane);
// channels 8-11 (C = 12): M = 64 rows m = 8 (y / 2) + 4 (y % 2) + c - 8.
template <int C>
__device__ __forceinline__ void scatter_stage_out(Smem<C> &s, uint32_t tmem, int warp, int lane, int half)
{
    const int q = warp & 3;
    const uint32_t lanes = (uint32_t)(32 * q) << 16;
    {  // grid 0, channels 0-7: half h takes x in [16 h, 16 h + 16)
        uint32_t v[16];
        umma::ld16(tmem + kColTile + lanes + 16 * half, v);
        umma::wait_ld();
        const int m = 32 * q + lane, y = m >> 3, c = m & 7;
        if (y < sc_h(0)) {
            float *o = s.t.f.g0 + (y * (sc_w(0) + 1) + 16 * half) * C + c;
#pragma unroll
            for (int j = 0; j < 16; ++j) o[C * j] = __uint_as_float(v[j]);
        }
    }
    if (half) {  // grid 1, channels 0-7: rows m = 16 q + lane (lanes 0..15), columns x
        uint32_t v[16];
        umma::ld16(tmem + kColTile + sc_w(0) + lanes, v);
        umma::wait_ld();
        const int m = 16 * q + lane, y = m >> 3, c = m & 7;
        if (lane < 16) {
            float *o = s.t.f.g1 + (y * (sc_w(1) + 1)) * C + c;
#pragma unroll
            for (int j = 0; j < 16; ++j) o[C * j] = __uint_as_float(v[j]);
        }
    }
    if constexpr (C == 12) {
        const int m = 16 * q + lane, y = 2 * (m >> 3) + ((m >> 2) & 1), c = 8 + (m & 3);
        {  // grid 0, channels 8-11: half h takes x in [16 h, 16 h + 16)
            uint32_t v[16];
            umma::ld16(tmem + Cols<C>::ScatB0 + lanes + 16 * half, v);
            umma::wait_ld();
            if (lane < 16 && y < sc_h(0)) {
                float *o = s.t.f.g0 + (y * (sc_w(0) + 1) + 16 * half) * C + c;
#pragma unroll
                for (int j = 0; j < 16; ++j) o[C * j] = __uint_as_float(v[j]);
            }
        }
        if (half) {  // grid 1, channels 8-11
            uint32_t v[16];
            umma::ld16(tmem + Cols<C>::ScatB1 + lanes, v);
            umma::wait_ld();
            if (lane < 16 && y < sc_h(1)) {
                float *o = s.t.f.g1 + (y * (sc_w(1) + 1)) * C + c;
#pragma unroll
                for (int j = 0; j < 16; ++j) o[C * j] = __uint_as_float(v[j]);
            }
        }
    }
}

// Staged window sums of block features -> the BC6 backward of every window texel.
template <int C>
__device__ __forceinline__ void scatter_reduce_blocks(const Smem<C> &s, const TrainLaunch &p, int tid)
{
    constexpr int n0 = sc_h(0) * sc_w(0), n1 = sc_h(1) * sc_w(1);  // (row, column) slots
    static_assert((n0 + n1) % kThreadsTC == 0, "whole slots per thread");
#pragma unroll 1
    for (int it = 0; it < (n0 + n1) / kThreadsTC; ++it) {
        const int k = tid + it * kThreadsTC;
        const int g = k < n0 ? 0 : 1;
        const int kk = g ? k - n0 : k;
        const int x = g ? kk & (sc_w(1) - 1) : kk & (sc_w(0) - 1);
        const int y = g ? kk >> 4 : kk >> 5;
        const Window &W = s.win[g];
        if (x >= W.w || y >= W.h) continue;
        const float *src = g ? s.t.f.g1 + (y * (sc_w(1) + 1) + x) * C : s.t.f.g0 + (y * (sc_w(0) + 1) + x) * C;
        float row[C];
#pragma unroll
        for (int q = 0; q < C / 4; ++q) {
            const float4 v = *reinterpret_cast<const float4 *>(src + 4 * q);
            row[4 * q] = v.x;
            row[4 * q + 1] = v.y;
            row[4 * q + 2] = v.z;
            row[4 * q + 3] = v.w;
        }
        flush_row<C, true>(p, g, W.x0 + x, W.y0 + y, row);
    }
}

template <int C>
__device__ __forceinline__ Descs<C> make_descs(const Smem<C> &s)
{
    using K = Cfg<C>;
    using umma::desc;
    constexpr uint32_t XG = K::XC * 128, HG = kHC * 128;
    Descs<C> d;
    d.x = desc(smem_addr(s.t.m.X), 128, XG);
    d.h1 = desc(smem_addr(s.t.m.H1), 128, HG);
    d.h2 = desc(smem_addr(s.t.m.H2), 128, HG);
    d.dy = desc(smem_addr(s.t.m.DY), 128, 256);
    d.w1 = desc(smem_addr(s.W1), 128, XG);
    d.w2 = desc(smem_addr(s.W2), 128, HG);
    d.w3 = desc(smem_addr(s.W3), 128, HG);
    d.x_mn = desc(smem_addr(s.t.m.X), XG, 128);
    d.h1_mn = desc(smem_addr(s.t.m.H1), HG, 128);
    d.h2_mn = desc(smem_addr(s.t.m.H2), HG, 128);
    d.dy_mn = desc(smem_addr(s.t.m.DY), 256, 128);
    d.w1_mn = desc(smem_addr(s.W1), XG, 128);
    d.w2_mn = desc(smem_addr(s.W2), HG, 128);
    d.w3_mn = desc(smem_addr(s.W3), HG, 128);
    d.q0 = desc(smem_addr(s.t.q.Q0), sc_qa(0) * 128, 128);
    d.q1 = desc(smem_addr(s.t.q.Q1), sc_qa(1) * 128, 128);
    d.q0b = desc(smem_addr(s.t.q.Q0), sc_qb(0) * 128, 128);
    d.q1b = desc(smem_addr(s.t.q.Q1), sc_qb(1) * 128, 128);
    d.a0 = desc(smem_addr(s.t.q.A0), sc_w(0) / 8 * 128, 128);
    d.a1 = desc(smem_addr(s.t.q.A1), sc_w(1) / 8 * 128, 128);
    return d;
}

// Stage boundary: the operands written since the last one become visible to the tensor
// core, the CTA agrees on failure, thread 0 issues the stage, every thread waits for it.
// Returns false (the same answer on every thread) when the CTA must stop; a wait that
// times out is recorded and reaches the other threads at the next barrier.
template <int C>
__device__ __forceinline__ bool run_stage(int stage, const Descs<C> &d, uint32_t tmem, bool first, uint32_t done,
                                          uint32_t dwdone, uint32_t &ph, bool &failed, int tid)
{
    umma::fence_async_smem();
    umma::fence_before();
    if (__syncthreads_or(failed)) {
        failed = true;
        return false;
    }
    umma::fence_after();
    // the stage's product by thread 0; the weight-gradient products of B3 / B2 / B1 by the last
    // thread (another warp and scheduler), so that neither issue delays one warp's epilogue twice
    if (tid == 0) issue_stage<C>(stage, d, tmem, done);
    if (tid == kThreadsTC - 1 && stage >= 3 && stage <= 5) issue_dw<C>(stage, d, tmem, first, dwdone);
    if (!umma::mbar_wait(done, ph, kSpinLimit)) {
        failed = true;
        atomicOr(&g_device_status, 1u);
        umma::mbar_wait(done, ph, kSpinLimit);  // one more bounded wait for the products in flight
    }
    ph ^= 1u;
    umma::fence_after();
    return true;
}

// ---- second mip level of a fractional mip coordinate (MIP) ---------------------------------
//
// After the first level's scatter, each sample's footprint in the second level replaces the
// first level's in shared memory, the tile's windows are rebuilt from it, and the same scatter
// (tensor-core or column sweep) runs on the second level's gradients with the weight-t share of
// dX.  A grid whose t is 0 (its chain ended) contributes nothing.  Returns false when a stage
// failed (the caller leaves the tile loop).
template <int C>
__device__ bool scatter_second_level(Smem<C> &s, const TrainLaunch &p, const Descs<C> &d, uint32_t tmem, bool &first,
                                     uint32_t done, uint32_t dwdone, uint32_t &ph, bool &failed, int tid, int warp,
                                     int lane, int r, int half, int ix, int iy, bool sample_valid, const float (&dxo)[C])
{
    using K = Cfg<C>;
    const float t = p.mip_t[half];
    const bool valid = sample_valid && t > 0.f;
    float dxb[C];
#pragma unroll
    for (int k = 0; k < C; ++k) dxb[k] = valid ? __fmul_rn(dxo[k], t) : 0.f;
    {
        float u = 0.f, v = 0.f;
        if (valid) sample_uv(p.sampler, ix, iy, u, v);
        Footprint fb;
        footprint(u, v, max(p.gw_b[half], 1), max(p.gh_b[half], 1), fb);
        s.base[half][r] = make_short2((short)fb.bx, (short)fb.by);
        float4 *wr = reinterpret_cast<float4 *>(s.wts[half][r]);
        wr[0] = make_float4(fb.wx[0], fb.wx[1], fb.wx[2], fb.wx[3]);
        wr[1] = make_float4(fb.wy[0], fb.wy[1], fb.wy[2], fb.wy[3]);
        extents_partial(s.part[half], fb.bx, fb.by, valid, warp & 3, lane);
    }
    if (__syncthreads_or(failed)) return false;
    if (warp < 2) finalize_window_tc(s, warp, lane);
    if (__syncthreads_or(failed)) return false;
    bool tc = false;
    if constexpr (C == 8) tc = (s.win[0].tc || s.win[0].w == 0) && (s.win[1].tc || s.win[1].w == 0);
    if (tc) {
        if constexpr (C == 8) {
            if (half) scatter_rows<C, 1>(s, s.t.q, r, valid, dxb);
            else scatter_rows<C, 0>(s, s.t.q, r, valid, dxb);
        }
        if (!run_stage<C>(6, d, tmem, first, done, dwdone, ph, failed, tid)) return false;
        scatter_stage_out<C>(s, tmem, warp, lane, half);
        if (__syncthreads_or(failed)) return false;
        scatter_reduce<C, true>(s, s.t.f, p, tid);
    } else {
        float *dxr = reinterpret_cast<float *>(s.t.m.H2) + r * K::DXS + half * C;
#pragma unroll
        for (int q = 0; q < C / 4; ++q)
            *reinterpret_cast<float4 *>(dxr + 4 * q) = make_float4(dxb[4 * q], dxb[4 * q + 1], dxb[4 * q + 2], dxb[4 * q + 3]);
        if (warp < 2) window_cands(s, warp, lane);
        if (__syncthreads_or(failed)) return false;
        const bool both = s.win[0].ok && s.win[1].ok;
        const int span = max(s.win[0].span, s.win[1].span);
        if (both && span <= 5) {
            sweep_tc<C, 5, false, true>(s, reinterpret_cast<const float *>(s.t.m.H2), p, tid);
        } else if (both && span <= 10) {
            sweep_tc<C, 10, false, true>(s, reinterpret_cast<const float *>(s.t.m.H2), p, tid);
        } else if (valid) {
            scatter_taps_tc<C, false, true>(s, reinterpret_cast<const float *>(s.t.m.H2), p, half, r);
        }
    }
    umma::fence_before();
    return !__syncthreads_or(failed);  // the next tile (or pass) overwrites the footprints and windows
}

// ---- block-feature gather through a decoded window ----------------------------------------
//
// The 128 samples of a tile read about 290 distinct texels of the two grids (config 1) but
// 4,096 taps.  Each window texel is decoded from its block records once per tile into shared
// memory (over the H1 / H2 / DY tiles, idle until F1 completes), and the samples gather from
// there in gather_bc6f's order, so the features are bit-identical to the direct decode.

template <int C>
__device__ __forceinline__ float *blk_window(Smem<C> &s) { return reinterpret_cast<float *>(s.t.m.H1); }

template <int C>
__host__ __device__ constexpr int blk_window_floats()
{
    return (int)((sizeof(Smem<C>::t.m.H1) + sizeof(Smem<C>::t.m.H2) + sizeof(Smem<C>::t.m.DY)) / sizeof(float));
}

// Decode the windows of both grids (all threads); false when they do not fit.
template <int C>
__device__ __forceinline__ bool blk_decode_windows(Smem<C> &s, const TrainLaunch &p, int tid)
{
    constexpr int T = (C + 2) / 3;
    const Window &W0 = s.win[0], &W1 = s.win[1];
    const long long n0 = (long long)W0.w * W0.h, n1 = (long long)W1.w * W1.h;
    if ((n0 + n1) * C > blk_window_floats<C>()) return false;
    float *buf = blk_window<C>(s);
    const int items0 = (int)n0 * T, items = items0 + (int)n1 * T;
    for (int k = tid; k < items; k += kThreadsTC) {
        const int g = k < items0 ? 0 : 1;
        const int kk = g ? k - items0 : k;
        const int n = g ? (int)n1 : (int)n0;
        const int t = kk / n, idx = kk - t * n;  // consecutive threads: consecutive texels of a row
        const Window &W = s.win[g];
        const int ly = idx / W.w, lx = idx - ly * W.w;
        const int gw = p.gw[g], gh = p.gh[g];
        float v[3];
        bc6f_texel_triple(reinterpret_cast<const float *>(p.grid[g]), gw, T, wrap_coord(W.x0 + lx, gw),
                          wrap_coord(W.y0 + ly, gh), t, v);
        float *dst = buf + (g ? (int)n0 * C : 0) + idx * C + 3 * t;
#pragma unroll
        for (int c = 0; c < 3; ++c)
            if (3 * t + c < C) dst[c] = v[c];
    }
    return true;
}

// Catmull-Rom gather of sample r from a decoded window (gather_bc6f's fmaf order).
template <int C>
__device__ __forceinline__ void blk_gather_window(const Smem<C> &s, const float *win, int g, int r, float (&out)[C])
{
    const Window &W = s.win[g];
    const short2 b = s.base[g][r];
    const float4 wx4 = *reinterpret_cast<const float4 *>(&s.wts[g][r][0]);
    const float4 wy4 = *reinterpret_cast<const float4 *>(&s.wts[g][r][4]);
    const float wx[4] = {wx4.x, wx4.y, wx4.z, wx4.w}, wy[4] = {wy4.x, wy4.y, wy4.z, wy4.w};
#pragma unroll
    for (int k = 0; k < C; ++k) out[k] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float *rp = win + ((b.y - 1 + j - W.y0) * W.w + (b.x - 1 - W.x0)) * C;
        float row[C];
#pragma unroll
        for (int k = 0; k < C; ++k) row[k] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int q = 0; q < C / 4; ++q) {
                const float4 v = *reinterpret_cast<const float4 *>(rp + i * C + 4 * q);
                row[4 * q] = fmaf(wx[i], v.x, row[4 * q]);
                row[4 * q + 1] = fmaf(wx[i], v.y, row[4 * q + 1]);
                row[4 * q + 2] = fmaf(wx[i], v.z, row[4 * q + 2]);
                row[4 * q + 3] = fmaf(wx[i], v.w, row[4 * q + 3]);
            }
        }
#pragma unroll
        for (int k = 0; k < C; ++k) out[k] = fmaf(wy[j], row[k], out[k]);
    }
}

// ---- gather of one latent grid (fp16 grids) ---------------------------------------------------

// Sample r's Catmull-Rom gather of grid G (second level blended in at a fractional mip
// coordinate), its footprint for the latent scatter, and its latents in the X operand:
// grid 0 takes X elements 0 .. C - 1, grid 1 elements C .. 2C - 1.
template <int C, int G, bool MIP>
__device__ __forceinline__ void gather_grid(Smem<C> &s, const TrainLaunch &p, int r, bool valid, float u, float v,
                                            int warp, int lane)
{
    using K = Cfg<C>;
    Footprint fp;
    footprint(u, v, p.gw[G], p.gh[G], fp);
    if (valid) shard_rows(p, G, p.gh[G], fp);
    uint32_t packed[C / 2];
#pragma unroll
    for (int k = 0; k < C / 2; ++k) packed[k] = 0u;
    if (valid) {
        float f[C];
        gather_cr<C>(p.grid[G], p.gw[G], fp, f);
        if constexpr (MIP) {
            const float t = p.mip_t[G];
            if (t > 0.f) {  // (1 - t) level m0 + t level m1 (train.cu:303-304)
                Footprint fb;
                footprint(u, v, p.gw_b[G], p.gh_b[G], fb);
                float fl[C];
                gather_cr<C>(p.grid_b[G], p.gw_b[G], fb, fl);
                const float omt = __fsub_rn(1.f, t);
#pragma unroll
                for (int k = 0; k < C; ++k) f[k] = __fadd_rn(__fmul_rn(omt, f[k]), __fmul_rn(t, fl[k]));
            }
        }
#pragma unroll
        for (int k = 0; k < C / 2; ++k) packed[k] = pack_half2(f[2 * k], f[2 * k + 1]);
    }
    if (!p.finalize) {
        s.base[G][r] = make_short2((short)fp.bx, (short)fp.by);
        float4 *wr = reinterpret_cast<float4 *>(s.wts[G][r]);
        wr[0] = make_float4(fp.wx[0], fp.wx[1], fp.wx[2], fp.wx[3]);
        wr[1] = make_float4(fp.wy[0], fp.wy[1], fp.wy[2], fp.wy[3]);
        extents_partial(s.part[G], fp.bx, fp.by, valid, warp & 3, lane);
    }
    // X elements G * C .. G * C + C - 1 in 4-element (8-byte) pieces
#pragma unroll
    for (int e = 0; e < C; e += 4) {
        const int k = G * C + e;
        if ((k & 7) == 0 && e + 8 <= C) {
            st16(s.t.m.X, umma::cm_offset(r, k, K::XC), packed[e / 2], packed[e / 2 + 1], packed[e / 2 + 2],
                 packed[e / 2 + 3]);
            e += 4;
        } else {
            *reinterpret_cast<uint2 *>(s.t.m.X + umma::cm_offset(r, k, K::XC)) =
                make_uint2(packed[e / 2], packed[e / 2 + 1]);
        }
    }
}

// ---- the kernel ---------------------------------------------------------------------------------

// C: latent channels per grid; TC: target channels when they have a vector gather (4, 8,
// 12 or 16), 0 for the generic per-channel gather; BLK: the latents are BC6 block features
// (nt_bc6f.cuh: float records sampled through the BC6 decode, gradients into the records);
// MIP: a fractional mip coordinate, so a grid or the target also reads a second level
// (weight mip_t / target_t): features and target blend the two, the first level's gradient
// takes the usual scatter at weight 1 - t and the second level per-tap atomics at weight t.
// DYN: tiles after the first come from the tile counter p.tile_counter (a separate
// instantiation: the claim code measured 6 % slower on the fixed-share path of config 1).
template <int C, int TC, bool BLK, bool MIP, bool DYN>
__global__ void __launch_bounds__(kThreadsTC, 2) train_tc_kernel(const TrainLaunch p)
{
    using K = Cfg<C>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    Smem<C> &s = *reinterpret_cast<Smem<C> *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r = tid & (kTileN - 1), half = tid >> 7;  // sample, role

    stage_weights_tc<C>(s, p.net, tid, kThreadsTC);
    if (warp == 0) umma::alloc(smem_addr(&s.tmem_base), kTmemCols);
    if (tid == 0) {
        umma::mbar_init(smem_addr(&s.done), 1);
        umma::mbar_init(smem_addr(&s.dwdone), 1);
        umma::mbar_fence_init();
    }
    umma::fence_async_smem();
    umma::fence_before();
    __syncthreads();
    umma::fence_after();
    const uint32_t tmem = s.tmem_base;
    const uint32_t Rl = tmem + kColTile + ((uint32_t)(32 * (warp & 3)) << 16);  // this warp's lanes
    const uint32_t done = smem_addr(&s.done), dwdone = smem_addr(&s.dwdone);
    uint32_t dph = 0;  // parity of the next weight-gradient completion
    const Descs<C> d = make_descs<C>(s);
    const int ntiles = p.tiles_x * p.tiles_y;
    const int cout = p.net.cout;
    uint32_t ph = 0;
    bool failed = false, first = true;
    float sse = 0.f;

    // Tiles: every CTA starts on tile blockIdx.x.  With a tile counter it then takes the next
    // unclaimed tile past the first gridDim.x (claimed during the tile before, published after
    // B1, read by all after a later barrier); without one, tiles blockIdx.x + gridDim.x, ...
    for (int tile = blockIdx.x; tile < ntiles; tile = DYN ? s.next_tile : tile + gridDim.x) {
        const int cx0 = (tile % p.tiles_x) * kTileW, cy0 = (tile / p.tiles_x) * kTileH;
        const int ix = cx0 + (r & (kTileW - 1));
        const int iy = p.lat_row0 + cy0 + (r >> 4);  // full lattice row (sharded calls train a band)
        const bool valid = ix < p.sampler.lattice_w && iy < p.lat_row0 + p.lat_rows && iy < p.sampler.lattice_h;
        float tgt[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) tgt[k] = 0.f;

        // ---- gather.  8-channel grids with an fp16 target buffer: half 0 = grid 0 + positional
        // features, half 1 = grid 1 + target.  12-channel grids (whose half-1 registers would
        // not hold a grid gather beside the target) and the generic target (reference textures:
        // 9 texture fetches per texture and level): half 0 = both grids, half 1 = target +
        // positional features.  Block features: half 0 = both footprints (the records are
        // gathered after the window decode below), half 1 = target + positional features.
        {
            constexpr bool kSplitGrids = C == 8 && TC > 0 && !BLK;
            float u = 0.f, v = 0.f;
            if (valid) sample_uv(p.sampler, ix, iy, u, v);
            if constexpr (kSplitGrids) {
                if (half == 0) gather_grid<C, 0, MIP>(s, p, r, valid, u, v, warp, lane);
                else gather_grid<C, 1, MIP>(s, p, r, valid, u, v, warp, lane);
            } else if constexpr (!BLK) {
                if (half == 0) {
                    uint32_t packed[K::LC * 4];
#pragma unroll
                    for (int k = 0; k < K::LC * 4; ++k) packed[k] = 0u;
#pragma unroll
                    for (int gi = 0; gi < 2; ++gi) {
                        Footprint fp;
                        footprint(u, v, p.gw[gi], p.gh[gi], fp);
                        if (valid) shard_rows(p, gi, p.gh[gi], fp);
                        if (valid) {
                            float f[C];
                            gather_cr<C>(p.grid[gi], p.gw[gi], fp, f);
                            if constexpr (MIP) {
                                const float t = p.mip_t[gi];
                                if (t > 0.f) {  // (1 - t) level m0 + t level m1 (train.cu:303-304)
                                    Footprint fb;
                                    footprint(u, v, p.gw_b[gi], p.gh_b[gi], fb);
                                    float fl[C];
                                    gather_cr<C>(p.grid_b[gi], p.gw_b[gi], fb, fl);
                                    const float omt = __fsub_rn(1.f, t);
#pragma unroll
                                    for (int k = 0; k < C; ++k)
                                        f[k] = __fadd_rn(__fmul_rn(omt, f[k]), __fmul_rn(t, fl[k]));
                                }
                            }
#pragma unroll
                            for (int k = 0; k < C / 2; ++k) packed[gi * (C / 2) + k] = pack_half2(f[2 * k], f[2 * k + 1]);
                        }
                        if (!p.finalize) {
                            s.base[gi][r] = make_short2((short)fp.bx, (short)fp.by);
                            float4 *wr = reinterpret_cast<float4 *>(s.wts[gi][r]);
                            wr[0] = make_float4(fp.wx[0], fp.wx[1], fp.wx[2], fp.wx[3]);
                            wr[1] = make_float4(fp.wy[0], fp.wy[1], fp.wy[2], fp.wy[3]);
                            extents_partial(s.part[gi], fp.bx, fp.by, valid, warp, lane);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < K::LC; ++j)
                        st16(s.t.m.X, umma::cm_offset(r, 8 * j, K::XC), packed[4 * j], packed[4 * j + 1],
                             packed[4 * j + 2], packed[4 * j + 3]);
                }
            }
            if (BLK && half == 0) {
#pragma unroll
                for (int gi = 0; gi < 2; ++gi) {
                    Footprint fp;
                    footprint(u, v, p.gw[gi], p.gh[gi], fp);
                    if (valid) shard_rows(p, gi, p.gh[gi], fp);
                    s.base[gi][r] = make_short2((short)fp.bx, (short)fp.by);
                    float4 *wr = reinterpret_cast<float4 *>(s.wts[gi][r]);
                    wr[0] = make_float4(fp.wx[0], fp.wx[1], fp.wx[2], fp.wx[3]);
                    wr[1] = make_float4(fp.wy[0], fp.wy[1], fp.wy[2], fp.wy[3]);
                    extents_partial(s.part[gi], fp.bx, fp.by, valid, warp, lane);
                }
            }
            const bool pe_half = kSplitGrids ? half == 0 : half == 1;  // writes the positional features
            if (pe_half) {
                uint32_t packed[4] = {0u, 0u, 0u, 0u};
                if (valid) {
                    float pe[8];
                    posenc(u, v, pe);
#pragma unroll
                    for (int k = 0; k < 4; ++k) packed[k] = pack_half2(pe[2 * k], pe[2 * k + 1]);
                }
                static_assert(K::XC == K::LC + 2 || K::XC == K::LC + 3, "X row: latents, posenc, 1, [0]");
                st16(s.t.m.X, umma::cm_offset(r, 8 * K::LC, K::XC), packed[0], packed[1], packed[2], packed[3]);
                st16(s.t.m.X, umma::cm_offset(r, 8 * (K::LC + 1), K::XC), pack_half2(1.f, 0.f), 0u, 0u, 0u);
                if constexpr (K::XC > K::LC + 2)
                    st16(s.t.m.X, umma::cm_offset(r, 8 * (K::LC + 2), K::XC), 0u, 0u, 0u, 0u);
            }
            if (half == 1 && valid) {  // the target (the loss epilogue runs on half 1)
                Footprint fp;
                footprint(u, v, p.tw, p.th, fp);
                shard_rows(p, 2, p.th, fp);
                if constexpr (TC > 0)
                    gather_cr<TC>(p.target, p.tw, fp, tgt);
                else if (p.num_ref > 0)  // reference textures (train.cu:105-157)
                    ref_expected(p.ref, p.num_ref, u, v, p.ref_lod, tgt);
                else
                    gather_cr_any(p.target, p.tw, cout, fp, tgt);
                if constexpr (MIP) {
                    const float t = p.target_t;
                    if (t > 0.f) {  // train.cu:102: sample0 (1 - t) + sample1 t
                        float tb[16];
                        footprint(u, v, p.tw_b, p.th_b, fp);
                        if constexpr (TC > 0) {
#pragma unroll
                            for (int k = TC; k < 16; ++k) tb[k] = 0.f;
                            gather_cr<TC>(p.target_b, p.tw_b, fp, tb);
                        } else {
                            gather_cr_any(p.target_b, p.tw_b, cout, fp, tb);
                        }
                        const float omt = __fsub_rn(1.f, t);
#pragma unroll
                        for (int k = 0; k < 16; ++k) tgt[k] = __fadd_rn(__fmul_rn(omt, tgt[k]), __fmul_rn(t, tb[k]));
                    }
                }
            }
        }
        if constexpr (BLK) {
            __syncthreads();  // footprints and extents
            if (warp < 2) finalize_window_tc(s, warp, lane);
            __syncthreads();  // windows
            const bool windowed = blk_decode_windows<C>(s, p, tid);
            __syncthreads();  // decoded window texels
            if (half == 0) {
                uint32_t packed[K::LC * 4];
#pragma unroll
                for (int k = 0; k < K::LC * 4; ++k) packed[k] = 0u;
                if (valid) {
#pragma unroll
                    for (int gi = 0; gi < 2; ++gi) {
                        float f[C];
                        if (windowed) {
                            const float *win = blk_window<C>(s) + (gi ? s.win[0].w * s.win[0].h * C : 0);
                            blk_gather_window<C>(s, win, gi, r, f);
                        } else {
                            float u = 0.f, v = 0.f;
                            sample_uv(p.sampler, ix, iy, u, v);
                            Footprint fp;
                            footprint(u, v, p.gw[gi], p.gh[gi], fp);
                            gather_bc6f<C>(reinterpret_cast<const float *>(p.grid[gi]), p.gw[gi], fp, f);
                        }
#pragma unroll
                        for (int k = 0; k < C / 2; ++k) packed[gi * (C / 2) + k] = pack_half2(f[2 * k], f[2 * k + 1]);
                    }
                }
#pragma unroll
                for (int j = 0; j < K::LC; ++j)
                    st16(s.t.m.X, umma::cm_offset(r, 8 * j, K::XC), packed[4 * j], packed[4 * j + 1], packed[4 * j + 2],
                         packed[4 * j + 3]);
            }
        }
        if (!run_stage<C>(0, d, tmem, first, done, dwdone, ph, failed, tid)) break;  // F1
        // the next tile is claimed by the last thread (not thread 0, which issues the products),
        // and its number is only needed after B1, so the atomic's latency is hidden
        uint32_t claim = 0;
        if (DYN && tid == kThreadsTC - 1) claim = gridDim.x + atomicAdd(p.tile_counter, 1u);

        // ---- E1: H1e = [relu(Z1) | 1 | 0] -----------------------------------------------
        relu_store32(Rl + 32 * half, s.t.m.H1, r, 4 * half);
        if (half)
            st16(s.t.m.H1, umma::cm_offset(r, 64, kHC), pack_half2(1.f, 0.f), 0u, 0u, 0u);
        else
            st16(s.t.m.H1, umma::cm_offset(r, 72, kHC), 0u, 0u, 0u, 0u);
        if (!run_stage<C>(1, d, tmem, first, done, dwdone, ph, failed, tid)) break;  // F2

        // ---- E2: H2e ------------------------------------------------------------------------
        relu_store32(Rl + 32 * half, s.t.m.H2, r, 4 * half);
        if (half)
            st16(s.t.m.H2, umma::cm_offset(r, 64, kHC), pack_half2(1.f, 0.f), 0u, 0u, 0u);
        else
            st16(s.t.m.H2, umma::cm_offset(r, 72, kHC), 0u, 0u, 0u, 0u);
        if (!run_stage<C>(2, d, tmem, first, done, dwdone, ph, failed, tid)) break;  // F3

        // ---- E3: weighted L2 (train.cu:876-888); dY = 2 w err (fp16, unscaled) -------------
        // (half 0 meanwhile finalises the footprint windows published by the gather barrier)
        if (!BLK && !half && !p.finalize && warp < 2) finalize_window_tc(s, warp, lane);  // BLK: in the gather
        if (half) {
            uint32_t v[16];
            umma::ld16(Rl, v);
            umma::wait_ld();
            uint32_t out[8];
#pragma unroll
            for (int c2 = 0; c2 < 8; ++c2) {
                float dd[2] = {0.f, 0.f};
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int c = 2 * c2 + e;
                    if (valid && c < cout) {
                        const float y = round_half(__uint_as_float(v[c]));
                        const float err = y - tgt[c];
                        sse = fmaf(p.cw[c] * err, err, sse);
                        dd[e] = 2.f * p.cw[c] * err;
                    }
                }
                out[c2] = pack_half2(dd[0], dd[1]);
            }
            st16(s.t.m.DY, umma::cm_offset(r, 0, 2), out[0], out[1], out[2], out[3]);
            st16(s.t.m.DY, umma::cm_offset(r, 8, 2), out[4], out[5], out[6], out[7]);
        }
        if (!run_stage<C>(3, d, tmem, first, done, dwdone, ph, failed, tid)) break;  // B3

        // ---- E4: dZ2 = dH2 * [H2 > 0] (in place of H2) -----------------------------------
        mask_store32(Rl + 32 * half, s.t.m.H2, r, 4 * half, dwdone, dph, failed);  // after dW3 (reads H2)
        dph ^= 1u;
        if (!run_stage<C>(4, d, tmem, first, done, dwdone, ph, failed, tid)) break;  // B2

        // ---- E5: dZ1 = dH1 * [H1 > 0] (in place of H1) -----------------------------------
        mask_store32(Rl + 32 * half, s.t.m.H1, r, 4 * half, dwdone, dph, failed);  // after dW2 (reads H1)
        dph ^= 1u;
        if (!run_stage<C>(5, d, tmem, first, done, dwdone, ph, failed, tid)) break;  // B1
        if (DYN && tid == kThreadsTC - 1) s.next_tile = (int)claim;  // read after the next barrier

        // ---- E6: dX -> shared (fp32 rows over the dead H2 tile) -> latent gradients ------
        // dW1 (reads X and dZ1) must finish before anything below or the next tile writes them
        if (!umma::mbar_wait(dwdone, dph, kSpinLimit)) {
            failed = true;
            atomicOr(&g_device_status, 1u);
        }
        dph ^= 1u;
        float dxo[C];  // MIP: dX of grid `half` before the split between the two levels
        if (!p.finalize) {
            // dX columns [half * C, half * C + C): the latents of grid `half`
            float dxv[C];
            {
                uint32_t v[32];
                umma::ld16(Rl, *reinterpret_cast<uint32_t(*)[16]>(v));
                if constexpr (K::NX > 16) umma::ld16(Rl + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
                umma::wait_ld();
#pragma unroll
                for (int e = 0; e < C; ++e) dxv[e] = __uint_as_float(half ? v[C + e] : v[e]);
            }
            if constexpr (MIP) {
#pragma unroll
                for (int k = 0; k < C; ++k) dxo[k] = dxv[k];
                const float t = p.mip_t[half];
                if (t > 0.f) {  // level m0 takes weight 1 - t here, level m1 weight t after it
                    const float omt = __fsub_rn(1.f, t);
#pragma unroll
                    for (int k = 0; k < C; ++k) dxv[k] = __fmul_rn(dxv[k], omt);
                }
            }
            bool tc_scatter = false;
            if constexpr (C == 8 || !BLK) tc_scatter = s.win[0].tc && s.win[1].tc;
            if (tc_scatter) {
                if (half) scatter_rows<C, 1>(s, s.t.q, r, valid, dxv);
                else scatter_rows<C, 0>(s, s.t.q, r, valid, dxv);
                if (!run_stage<C>(6, d, tmem, first, done, dwdone, ph, failed, tid)) break;  // scatter product
                if constexpr (C == 12) {  // channels 8-11 through the same operand tiles
                    if (half) scatter_rows<C, 1, 1>(s, s.t.q, r, valid, dxv);
                    else scatter_rows<C, 0, 1>(s, s.t.q, r, valid, dxv);
                    if (!run_stage<C>(7, d, tmem, first, done, dwdone, ph, failed, tid)) break;
                }
                scatter_stage_out<C>(s, tmem, warp, lane, half);
                if (__syncthreads_or(failed)) {
                    failed = true;
                    break;
                }
                if constexpr (BLK)
                    scatter_reduce_blocks<C>(s, p, tid);
                else
                    scatter_reduce<C>(s, s.t.f, p, tid);
                first = false;
                umma::fence_before();
                if (__syncthreads_or(failed)) {
                    failed = true;
                    break;
                }
                if constexpr (MIP) {
                    if ((p.mip_t[0] > 0.f || p.mip_t[1] > 0.f) &&
                        !scatter_second_level<C>(s, p, d, tmem, first, done, dwdone, ph, failed, tid, warp, lane, r,
                                                 half, ix, iy, valid, dxo)) {
                        failed = true;
                        break;
                    }
                }
                continue;
            }
            float *dxr = reinterpret_cast<float *>(s.t.m.H2) + r * K::DXS + half * C;
#pragma unroll
            for (int q = 0; q < C / 4; ++q)
                *reinterpret_cast<float4 *>(dxr + 4 * q) = make_float4(dxv[4 * q], dxv[4 * q + 1], dxv[4 * q + 2], dxv[4 * q + 3]);
            if (warp < 2) window_cands(s, warp, lane);
            if (__syncthreads_or(failed)) {
                failed = true;
                break;
            }
            const bool both = s.win[0].ok && s.win[1].ok;
            const int span = max(s.win[0].span, s.win[1].span);
            if (both && span <= 5) {
                sweep_tc<C, 5, BLK>(s, reinterpret_cast<const float *>(s.t.m.H2), p, tid);
            } else if (both && span <= 10) {
                sweep_tc<C, 10, BLK>(s, reinterpret_cast<const float *>(s.t.m.H2), p, tid);
            } else if (valid) {
                scatter_taps_tc<C, BLK>(s, reinterpret_cast<const float *>(s.t.m.H2), p, half, r);
            }
        }
        first = false;
        umma::fence_before();
        // the next tile overwrites the footprints, the windows, X and H
        if (__syncthreads_or(failed)) {
            failed = true;
            break;
        }
        if constexpr (MIP) {
            if (!p.finalize && (p.mip_t[0] > 0.f || p.mip_t[1] > 0.f) &&
                !scatter_second_level<C>(s, p, d, tmem, first, done, dwdone, ph, failed, tid, warp, lane, r, half, ix,
                                         iy, valid, dxo)) {
                failed = true;
                break;
            }
        }
    }

    // every product of this CTA (the weight-gradient accumulators included) has completed:
    // each stage was waited for before the loop moved on

    // ---- flush the weight / bias gradients (x 1 / num_samples) --------------------------
    const float sc = p.inv_num_samples;
    if (!first && !failed) {
        const uint32_t lanes = (uint32_t)(32 * (warp & 3)) << 16;
        if (half == 0) {
            // dW1 (M = 64: row 16 (warp & 3) + lane for lane < 16) and dW3^T (M = 128)
            const int o = 16 * (warp & 3) + lane;
#pragma unroll
            for (int c0 = 0; c0 < K::XW; c0 += 16) {
                uint32_t v[16];
                umma::ld16(tmem + kColW1 + lanes + c0, v);
                umma::wait_ld();
                if (lane < 16) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int in = c0 + 4 * q;
                        if (in + 3 < K::kBias1)
                            red_add_v4(p.gW[0] + o * 32 + in, __uint_as_float(v[4 * q]) * sc,
                                       __uint_as_float(v[4 * q + 1]) * sc, __uint_as_float(v[4 * q + 2]) * sc,
                                       __uint_as_float(v[4 * q + 3]) * sc);
                        else if (in == K::kBias1)
                            atomicAdd(p.gb[0] + o, __uint_as_float(v[4 * q]) * sc);
                    }
                }
            }
            const int f = 32 * (warp & 3) + lane;  // hidden feature of dW3^T
            uint32_t v[16];
            umma::ld16(tmem + Cols<C>::W3 + lanes, v);
            umma::wait_ld();
#pragma unroll
            for (int o3 = 0; o3 < 16; ++o3) {
                if (o3 >= cout) continue;
                const float g = __uint_as_float(v[o3]) * sc;
                if (f < 64) atomicAdd(p.gW[2] + o3 * 64 + f, g);
                else if (f == 64) atomicAdd(p.gb[2] + o3, g);
            }
        } else {  // dW2 (M = 64, 72 columns)
            const int o = 16 * (warp & 3) + lane;
#pragma unroll
            for (int c0 = 0; c0 < 72; c0 += 8) {
                uint32_t v[8];
                umma::ld8(tmem + kColW2 + lanes + c0, v);
                umma::wait_ld();
                if (lane < 16) {
                    if (c0 < 64) {
#pragma unroll
                        for (int q = 0; q < 2; ++q)
                            red_add_v4(p.gW[1] + o * 64 + c0 + 4 * q, __uint_as_float(v[4 * q]) * sc,
                                       __uint_as_float(v[4 * q + 1]) * sc, __uint_as_float(v[4 * q + 2]) * sc,
                                       __uint_as_float(v[4 * q + 3]) * sc);
                    } else {
                        atomicAdd(p.gb[1] + o, __uint_as_float(v[0]) * sc);
                    }
                }
            }
        }
    }
    if (p.loss_accum) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sse += __shfl_xor_sync(0xffffffffu, sse, o);
        if (lane == 0) s.red[warp] = sse;
    }
    umma::fence_before();
    __syncthreads();
    if (p.loss_accum && tid == 0) {
        float tot = 0.f;
        for (int w = 0; w < kThreadsTC / 32; ++w) tot += s.red[w];
        atomicAdd(p.loss_accum, tot);
    }
    if (DYN && tid == 0) {  // the last CTA to finish (every CTA has made its last claim) zeroes the counters
        __threadfence();
        if (atomicAdd(p.tile_counter + 1, 1u) == gridDim.x - 1) {
            atomicExch(p.tile_counter, 0u);
            atomicExch(p.tile_counter + 1, 0u);
        }
    }
    if (warp == 0) {
        umma::fence_after();
        umma::dealloc(tmem, kTmemCols);
    }
}

template <int C, int TC, bool BLK, bool MIP = false>
static cudaError_t launch_t(TrainLaunch p, cudaStream_t stream)
{
    const size_t smem = sizeof(Smem<C>);
    static_assert(sizeof(Smem<C>) <= 113 * 1024, "two CTAs per SM");
    p.tiles_x = (p.sampler.lattice_w + kTileW - 1) / kTileW;
    p.tiles_y = (p.lat_rows + kTileH - 1) / kTileH;
    const int ntiles = p.tiles_x * p.tiles_y;
    const int cap = 2 * sm_count();
    const int grid = ntiles < cap ? ntiles : cap;
    // Tile counters (single-level fp16 grids): below 8 tiles per CTA the fixed shares are
    // balanced to within a tile and measured faster; from there on the counter wins (5 % at 27
    // tiles per CTA)
    if constexpr (!BLK && !MIP) {
        if (p.tile_counter && ntiles >= 8 * grid) {
            cudaError_t e = set_smem_limit(reinterpret_cast<const void *>(train_tc_kernel<C, TC, BLK, MIP, true>), smem);
            if (e != cudaSuccess) return e;
            train_tc_kernel<C, TC, BLK, MIP, true><<<grid, kThreadsTC, smem, stream>>>(p);
            count_launch();
            return cudaGetLastError();
        }
    }
    cudaError_t e = set_smem_limit(reinterpret_cast<const void *>(train_tc_kernel<C, TC, BLK, MIP, false>), smem);
    if (e != cudaSuccess) return e;
    p.tile_counter = nullptr;
    train_tc_kernel<C, TC, BLK, MIP, false><<<grid, kThreadsTC, smem, stream>>>(p);
    count_launch();
    return cudaGetLastError();
}

}  // namespace tc

cudaError_t launch_train_tc(const TrainLaunch &p, int channels, cudaStream_t stream)
{
    const int cout = p.net.cout;
    if (p.blocks) {  // BC6 block features
        if (channels == 8)
            return cout == 8 && !p.num_ref ? tc::launch_t<8, 8, true>(p, stream) : tc::launch_t<8, 0, true>(p, stream);
        if (channels == 12)
            return cout == 12 && !p.num_ref ? tc::launch_t<12, 12, true>(p, stream)
                                            : tc::launch_t<12, 0, true>(p, stream);
        return cudaErrorInvalidValue;
    }
    if (p.mip_t[0] > 0.f || p.mip_t[1] > 0.f || p.target_t > 0.f) {  // two mip levels
        if (channels == 8)
            return cout == 8 && !p.num_ref ? tc::launch_t<8, 8, false, true>(p, stream)
                                           : tc::launch_t<8, 0, false, true>(p, stream);
        if (channels == 12)
            return cout == 12 && !p.num_ref ? tc::launch_t<12, 12, false, true>(p, stream)
                                            : tc::launch_t<12, 0, false, true>(p, stream);
        return cudaErrorInvalidValue;
    }
    // reference textures come through the generic target path (TC = 0)
    if (channels == 8)
        return cout == 8 && !p.num_ref ? tc::launch_t<8, 8, false>(p, stream) : tc::launch_t<8, 0, false>(p, stream);
    if (channels == 12)
        return cout == 12 && !p.num_ref ? tc::launch_t<12, 12, false>(p, stream)
                                        : tc::launch_t<12, 0, false>(p, stream);
    return cudaErrorInvalidValue;
}

}  // namespace nt

namespace nt {

// An mbarrier (count 1) that nothing arrives on: the bounded wait gives up after `tries` polls
// and reports through the status word like the kernels' waits.
__global__ void wait_timeout_kernel(uint32_t tries)
{
    __shared__ alignas(8) uint64_t bar;
    if (threadIdx.x == 0) {
        umma::mbar_init(smem_addr(&bar), 1);
        umma::mbar_fence_init();
        if (!umma::mbar_wait(smem_addr(&bar), 0, tries)) atomicOr(&g_device_status, 1u);
    }
}

}  // namespace nt

extern "C" nt_status nt_wait_timeout_selftest(uint32_t tries)
{
    if (tries < 1 || tries > 1000000) return NT_ERR_INVALID_ARG;
    nt::wait_timeout_kernel<<<1, 32>>>(tries);
    nt::count_launch();
    if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) return NT_ERR_CUDA;
    return NT_OK;
}

extern "C" nt_status nt_read_device_status(uint32_t *status, int32_t clear)
{
    if (!status) return NT_ERR_INVALID_ARG;
    uint32_t train = 0, decode = 0;
    if (cudaMemcpyFromSymbol(&train, nt::g_device_status, sizeof(uint32_t)) != cudaSuccess) return NT_ERR_CUDA;
    if (nt::read_decode_status(&decode, clear != 0) != cudaSuccess) return NT_ERR_CUDA;
    if (clear) {
        const uint32_t zero = 0;
        if (cudaMemcpyToSymbol(nt::g_device_status, &zero, sizeof(uint32_t)) != cudaSuccess) return NT_ERR_CUDA;
    }
    *status = train | decode;
    return NT_OK;
}

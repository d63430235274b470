// nt_train.cu -- fused training pass: sample -> MLP forward -> weighted L2 -> MLP backward
// -> weight/bias gradient reduction -> latent-gradient scatter, in one persistent kernel.
//
// Replaces TrainLoopPass / TrainLoop (mavenkim2/neural_textures train.cu:818-915, :979-983)
// and the per-warp gradient reductions of mlp.h:101-220.
//
// Work decomposition.  A CTA of 8 warps owns a 16 x 16 tile of lattice cells (one jittered
// sample per cell, 256 samples) at a time and loops over tiles (persistent grid, one CTA
// per SM).  Every thread gathers one sample (both latent grids + the target, Catmull-Rom,
// 16-byte loads); every warp runs the three layers forward and backward for its 32 rows
// with fp16 tensor-core MMAs and fp32 accumulation; then the CTA cooperatively reduces
// the weight gradients over its 256 samples: each warp owns a fixed slice of dW1 / dW2 /
// dW3 and accumulates it in registers across all tiles it processes, so the global
// weight-gradient buffers see one atomic add per element per CTA (the reference issues one
// per element per warp per step, mlp.h:212-218).
#include "nt_mlp_smem.cuh"

namespace nt {

struct TrainSmem {
    MlpSmem mlp;
    __half X[kTileSamples * kStrideK32];    // MLP input
    __half H1[kTileSamples * kStrideK64];   // layer-1 output (post-ReLU)
    __half H2[kTileSamples * kStrideK64];   // layer-2 output, later dL/dH1
    __half DY[kTileSamples * kStrideK16];   // fp16 output, later dL/dY (x num_samples)
    __half DH2[kTileSamples * kStrideK64];  // dL/dH2, later dL/dX (fp32, 36 floats per row)
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
        float u = 0.f, v = 0.f;
        float tgt[16];

        // ---- gather: one sample per thread -------------------------------------------
        {
            uint32_t packed[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) packed[k] = 0u;
#pragma unroll
            for (int k = 0; k < 16; ++k) tgt[k] = 0.f;
            if (valid) {
                sample_uv(p.sampler, ix, iy, u, v);
                float f[C];
                Footprint fp;
#pragma unroll
                for (int gi = 0; gi < 2; ++gi) {
                    footprint(u, v, p.gw[gi], p.gh[gi], fp);
                    gather_cr<C>(p.grid[gi], p.gw[gi], fp, f);
#pragma unroll
                    for (int k = 0; k < C / 2; ++k) packed[gi * (C / 2) + k] = pack_half2(f[2 * k], f[2 * k + 1]);
                }
                float pe[8];
                posenc(u, v, pe);
#pragma unroll
                for (int k = 0; k < 4; ++k) packed[C + k] = pack_half2(pe[2 * k], pe[2 * k + 1]);
                footprint(u, v, p.sampler.image_w, p.sampler.image_h, fp);
                gather_cr_any(p.target, p.sampler.image_w, p.net.cout, fp, tgt);
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

        // ---- latent-gradient scatter (train.cu:460-509 with the Catmull-Rom footprint) ----
        if (!p.finalize && valid) {
            const float *dxr = reinterpret_cast<const float *>(s.DH2) + tid * kDxStride;
            float d[2 * C];
#pragma unroll
            for (int k = 0; k < 2 * C; ++k) d[k] = dxr[k] * p.inv_num_samples;
#pragma unroll
            for (int gi = 0; gi < 2; ++gi) {
                Footprint fp;
                footprint(u, v, p.gw[gi], p.gh[gi], fp);
                float *gg = p.ggrid[gi];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float *rowp = gg + (size_t)fp.ys[j] * (size_t)p.gw[gi] * C;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float wgt = fp.wy[j] * fp.wx[i];
                        float4 *dst = reinterpret_cast<float4 *>(rowp + (size_t)fp.xs[i] * C);
#pragma unroll
                        for (int q = 0; q < C / 4; ++q)
                            atomicAdd(dst + q, make_float4(wgt * d[gi * C + 4 * q], wgt * d[gi * C + 4 * q + 1],
                                                           wgt * d[gi * C + 4 * q + 2], wgt * d[gi * C + 4 * q + 3]));
                    }
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

cudaError_t launch_train(const TrainLaunch &p, int channels, cudaStream_t stream)
{
    const bool wide = p.net.cout > 8;
    if (channels == 8) return wide ? launch_train_t<8, 2>(p, stream) : launch_train_t<8, 1>(p, stream);
    if (channels == 12) return wide ? launch_train_t<12, 2>(p, stream) : launch_train_t<12, 1>(p, stream);
    return cudaErrorInvalidValue;
}

}  // namespace nt

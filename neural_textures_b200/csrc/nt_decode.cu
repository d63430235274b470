// nt_decode.cu -- decode (inference) of every texel centre of the image.
//
// Replaces Inference / RunInference (mavenkim2/neural_textures train.cu:917-961, :974-977):
// texel centres u = (x + 0.5) / W, latent sampling, MLP forward, outputs written per texel,
// optional squared error against a target.  The reference issues one thread per texel with
// per-thread weight loads and a single global SSE atomic per thread (train.cu:960); here a
// persistent CTA owns 16 x 16 texel tiles, keeps the weights in shared memory, runs the
// layers on tensor cores per warp and reduces the SSE once per CTA.
#include "nt_mlp_smem.cuh"

namespace nt {

struct DecodeSmem {
    MlpSmem mlp;
    __half X[kTileSamples * kStrideK32];
    __half Y[kTileSamples * kStrideK16];
    float red[kThreads / 32];
};

template <int C, int NT3>
__global__ void __launch_bounds__(kThreads, 2) decode_kernel(const DecodeLaunch p)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    DecodeSmem &s = *reinterpret_cast<DecodeSmem *>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    stage_weights(s.mlp, p.net);
    __syncthreads();
    const int ntiles = p.tiles_x * p.tiles_y;
    const int cout = p.net.cout;
    float sse = 0.f;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int x = (tile % p.tiles_x) * kTileSide + (tid & (kTileSide - 1));
        const int y = (tile / p.tiles_x) * kTileSide + tid / kTileSide;
        const bool valid = x < p.image_w && y < p.image_h;
        {
            uint32_t packed[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) packed[k] = 0u;
            if (valid) {
                float u, v;
                texel_uv(x, y, p.image_w, p.image_h, u, v);
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
            }
            uint4 *xr = reinterpret_cast<uint4 *>(s.X + tid * kStrideK32);
#pragma unroll
            for (int q = 0; q < 4; ++q)
                xr[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
        __syncwarp();
        {
            float acc3[2][NT3][4];
            warp_forward<NT3>(s.mlp, s.X, nullptr, nullptr, warp * 32, lane, acc3);
            store_out16<NT3>(acc3, s.Y, warp * 32, lane);
        }
        __syncwarp();
        if (valid) {
            const __half *yr = s.Y + tid * kStrideK16;
            const size_t texel = (size_t)y * p.image_w + x;
            if (!p.out_f32 && cout == 8) {
                *reinterpret_cast<uint4 *>(reinterpret_cast<__half *>(p.out) + texel * 8) =
                    *reinterpret_cast<const uint4 *>(yr);
            } else if (!p.out_f32) {
                __half *o = reinterpret_cast<__half *>(p.out) + texel * cout;
                for (int c = 0; c < cout; ++c) o[c] = yr[c];
            } else {
                float *o = reinterpret_cast<float *>(p.out) + texel * cout;
                for (int c = 0; c < cout; ++c) o[c] = __half2float(yr[c]);
            }
            if (p.target) {
                const __half *tr = p.target + texel * cout;
                for (int c = 0; c < cout; ++c) {
                    const float e = __half2float(yr[c]) - __half2float(tr[c]);
                    sse = fmaf(e, e, sse);
                }
            }
        }
    }
    if (p.mse_accum) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sse += __shfl_xor_sync(0xffffffffu, sse, o);
        if (lane == 0) s.red[warp] = sse;
        __syncthreads();
        if (tid == 0) {
            float tot = 0.f;
            for (int w = 0; w < kThreads / 32; ++w) tot += s.red[w];
            atomicAdd(p.mse_accum, tot);
        }
    }
}

template <int C, int NT3>
static cudaError_t launch_decode_t(const DecodeLaunch &p, cudaStream_t stream)
{
    const size_t smem = sizeof(DecodeSmem);
    cudaError_t e = set_smem_limit(reinterpret_cast<const void *>(decode_kernel<C, NT3>), smem);
    if (e != cudaSuccess) return e;
    const int ntiles = p.tiles_x * p.tiles_y;
    const int cap = 2 * sm_count();
    const int grid = ntiles < cap ? ntiles : cap;
    decode_kernel<C, NT3><<<grid, kThreads, smem, stream>>>(p);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_decode(const DecodeLaunch &p, int channels, cudaStream_t stream)
{
    if (decode_engine() == 1) return launch_decode_tc(p, channels, stream);
    const bool wide = p.net.cout > 8;
    if (channels == 8) return wide ? launch_decode_t<8, 2>(p, stream) : launch_decode_t<8, 1>(p, stream);
    if (channels == 12) return wide ? launch_decode_t<12, 2>(p, stream) : launch_decode_t<12, 1>(p, stream);
    return cudaErrorInvalidValue;
}

}  // namespace nt

// nt_kernels.cuh -- launch descriptors shared by the C-ABI layer and the kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "nt_common.cuh"
#include "nt_reftex.cuh"

namespace nt {

constexpr int kTileSide = 16;        // lattice cells / texels per tile side
constexpr int kTileSamples = 256;    // = kTileSide^2, one per thread
constexpr int kThreads = 256;        // 8 warps

struct NetView {
    const __half *W[3];  // global, padded column-major
    const __half *b[3];  // global, {64, 64, cout}
    int32_t cout;
};

struct TrainLaunch {
    const __half *grid[2];
    float *ggrid[2];
    int32_t gw[2], gh[2];
    NetView net;
    float *gW[3];
    float *gb[3];
    const __half *target;
    float cw[16];
    SamplerView sampler;
    float inv_num_samples;
    float *loss_accum;
    int32_t finalize;
    int32_t tiles_x, tiles_y;
    // Row sharding: lattice rows [lat_row0, lat_row0 + lat_rows) are trained; source s
    // (0, 1: latent grids, 2: target) stores rows_s rows from full row org[s] (wrapping).
    int32_t lat_row0, lat_rows;
    int32_t org[3], rows[3];
    int32_t blocks;  // 1: grid / ggrid hold BC6 block-feature records (float), not fp16 texels
    // Mip chains.  grid / ggrid / gw / gh above are the level m0 that every sample reads; with
    // mip_t[g] > 0 grid g also reads level m1 (grid_b ...): feature (1 - t) a + t b.  The target
    // level m0 is tw x th texels; target_t > 0 adds level m1.
    const __half *grid_b[2];
    float *ggrid_b[2];
    int32_t gw_b[2], gh_b[2];
    float mip_t[2];
    int32_t tw, th;
    const __half *target_b;
    int32_t tw_b, th_b;
    float target_t;
    // reference textures (num_ref > 0): the target comes from them, at mip coordinate ref_lod
    RefTexView ref[kMaxRefTextures];
    int32_t num_ref;
    float ref_lod;
    // optional tile counter pair (next tile, CTAs finished) in the caller's workspace: NULL for
    // a fixed share of the tiles per CTA
    uint32_t *tile_counter;
};

// Bytes of NtKernelParams.workspace (two 32-bit counters, padded).
constexpr size_t kWorkspaceBytes = 256;

struct DecodeLaunch {
    const __half *grid[2];
    int32_t gw[2], gh[2];
    NetView net;
    void *out;
    int32_t out_f32;
    int32_t out_stride;    // elements per texel of out (>= cout; channels past cout are written as 0)
    const __half *target;  // optional, fp16 [h][w][cout]
    float *mse_accum;      // optional
    int32_t image_w, image_h;
    int32_t tiles_x, tiles_y;
    // second mip level of grid g when mip_t[g] > 0 (TrainLaunch)
    const __half *grid_b[2];
    int32_t gw_b[2], gh_b[2];
    float mip_t[2];
    // reference textures for the MSE (num_ref > 0 and mse_accum)
    RefTexView ref[kMaxRefTextures];
    int32_t num_ref;
    float ref_lod;
};

constexpr int kMaxAdamSegments = 8;
constexpr int kAdamChunk = 1024;  // parameters per Adam CTA

struct AdamSegment {
    __half *w;
    float *w32;  // fp32 parameters instead of w (BC6 block-feature records)
    float *g, *m, *v;
    int64_t n;
    float lr, beta1, beta2, eps, bc1, bc2;
    int32_t first_block;
};

struct AdamLaunch {
    AdamSegment seg[kMaxAdamSegments];
    int32_t nseg;
    int32_t total_blocks;
};

// tcgen05 / TMEM training kernel (16 x 8 tiles; recomputes tiles_x / tiles_y itself)
cudaError_t launch_train_tc(const TrainLaunch &p, int channels, cudaStream_t stream);
// tcgen05 / TMEM decode kernel (16 x 8 tiles; recomputes tiles_x / tiles_y itself)
cudaError_t launch_decode_tc(const DecodeLaunch &p, int channels, cudaStream_t stream);
// Status word of the decode kernel's bounded waits (host read, optionally cleared).
cudaError_t read_decode_status(uint32_t *status, bool clear);
cudaError_t launch_adam(const AdamLaunch &p, cudaStream_t stream);
int sm_count();
// Raise the dynamic shared-memory limit of `kernel` once per device.
cudaError_t set_smem_limit(const void *kernel, size_t bytes);

}  // namespace nt

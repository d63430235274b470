/*
 * nt_capi.h -- C-ABI boundary of the B200 neural-texture trainer / decoder.
 *
 * Everything here is plain C: POD structs, raw device pointers, sizes and an opaque
 * stream handle.  No C++ or torch type crosses this boundary.  All device buffers are
 * owned by the caller (the reference allocates every buffer in its driver,
 * main.cpp:657-793); the library allocates no device memory of its own.
 *
 * Reference interface replaced (mavenkim2/neural_textures):
 *   train.h:120-157   struct KernelParams            -> NtKernelParams
 *   train.h:22-27     enum TrainingKernelType        -> NtTrainingKernelType
 *   train.h:29-35     struct AdamConstants           -> NtAdamConstants
 *   train.h:51-67     struct Feature                 -> NtFeature
 *   train.h:158       InvokeOptimizeNetwork          -> nt_invoke_optimize_network
 *   train.h:159       InvokeOptimizeFeatures         -> nt_invoke_optimize_features
 *   train.h:160       InvokeTraining                 -> nt_invoke_training
 *   train.h:161       InvokeInference                -> nt_invoke_inference
 *   tests/forward_pass_test.h:6  RunForwardPassTest  -> nt_run_forward_pass_test
 * The reference's entry points return void and surface errors at the next device
 * synchronisation (main.cpp:103-110); every entry point here returns an nt_status and
 * never throws.
 *
 * Network (fixed by the build, not by macros as in train.h:9-20):
 *   input  32 = 2 x C latent channels + 8 positional features, zero padded
 *   hidden 64 (ReLU) -> 64 (ReLU) -> output_channels (linear, <= 16)
 * Weights are fp16, column-major and padded to multiples of 16 exactly as the reference
 * stores them (train.h:84-112, main.cpp:195): layer l has W[col * padIn + row] with
 * padIn = {32, 64, 64} and padOut = {64, 64, 16}.  Biases are fp16 with one entry per
 * output (train.h:114-118).  Padded weight entries must be zero.
 */
#ifndef NT_CAPI_H
#define NT_CAPI_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NT_API __attribute__((visibility("default")))
#else
#define NT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define NT_CAPI_VERSION 1

#define NT_NUM_FEATURES 2        /* latent grids; the reference has 4 float3 features (train.h:18) */
#define NT_NUM_NETWORK_LAYERS 3  /* train.h:17 */
#define NT_MLP_INPUT 32
#define NT_MLP_HIDDEN 64
#define NT_MAX_OUTPUT 16         /* train.h:11 NT_OUTPUT_SIZE */
#define NT_POSENC_FEATURES 8     /* 2 frequencies x (u, v) x (sin, cos) */

typedef enum nt_status {
    NT_OK = 0,
    NT_ERR_INVALID_ARG = 1,
    NT_ERR_CUDA = 2,
    NT_ERR_NCCL = 3,
    NT_ERR_TIMEOUT = 4,
    NT_ERR_BOUNDS = 5,
    NT_ERR_UNSUPPORTED = 6,
    NT_ERR_IO = 7               /* a checkpoint file could not be read or written, or is corrupt */
} nt_status;

/* train.h:22-27 */
typedef enum NtTrainingKernelType {
    NT_TRAIN_UNCONSTRAINED = 0, /* latents are free fp16 grids */
    NT_TRAIN_BLOCK_FEATURES = 1, /* BC6 block latents (latent_format NT_LATENT_BC6_BLOCKS) */
    NT_TRAIN_FINALIZE = 2        /* network gradients only, latents frozen */
} NtTrainingKernelType;

typedef enum NtDtype { NT_DTYPE_F16 = 0, NT_DTYPE_F32 = 1, NT_DTYPE_U8 = 2, NT_DTYPE_I32 = 3 } NtDtype;

/* Opaque CUDA stream (cudaStream_t); NULL means the legacy default stream. */
typedef void *nt_stream_t;

/* train.h:29-35 */
typedef struct NtAdamConstants {
    float beta1;
    float beta2;
    float learning_rate;
    float epsilon;
} NtAdamConstants;

/* train.h:51-67, reduced to one mip level of fp16 channel-interleaved latents:
 * grid[(y * width + x) * channels + c].  gradients / moment1 / moment2 are fp32 with the
 * same layout (they may be NULL for decode-only use). */
typedef struct NtFeature {
    void *grid;         /* fp16 */
    float *gradients;
    float *moment1;
    float *moment2;
    int32_t width;
    int32_t height;
    int32_t num_mips;   /* train.h:61; 0 or 1: one level (see NtKernelParams.lod) */
} NtFeature;

/* train.h:69-77.  A reference texture: a CUDA texture object over an fp32 mip chain
 * (nt_reference_texture_create), sampled like the reference: Catmull-Rom through 9 hardware
 * bilinear fetches per level (filter/catmull_rom.h:39-89), the two levels of the mip coordinate
 * blended (train.cu:78-103).  Its channels fill the next output channels of the target, each
 * with the texture's loss weight (train.cu:105-157). */
#define NT_MAX_REFERENCE_TEXTURES 16 /* train.h:20 */
typedef struct NtReferenceTexture {
    uint64_t texture;      /* cudaTextureObject_t; 0: skipped */
    uint64_t storage;      /* the cudaMipmappedArray behind it (freed by nt_reference_texture_destroy) */
    int32_t width, height; /* level 0 */
    int32_t num_channels;  /* 1 .. 4 */
    int32_t num_mips;
    float loss_weight;
    int32_t reserved;
} NtReferenceTexture;

/* train.h:120-157.  Passed by pointer; the library copies what it needs at launch, so the
 * struct may be modified or freed as soon as the call returns. */
/* Latent representations (NtKernelParams.latent_format). */
#define NT_LATENT_GRID_F16 0
#define NT_LATENT_BC6_BLOCKS 1
/* Floats per channel triple of a 4x4 block in NT_LATENT_BC6_BLOCKS records. */
#define NT_BC6F_RECORD_FLOATS 32

typedef struct NtKernelParams {
    NtFeature features[NT_NUM_FEATURES];
    int32_t latent_channels;   /* C per grid: 8 or 12 */
    int32_t output_channels;   /* used outputs (train.h:147 usedOutputChannels), 1..16 */

    void *network_weights[NT_NUM_NETWORK_LAYERS];          /* fp16, padded column-major */
    float *network_weight_gradients[NT_NUM_NETWORK_LAYERS];
    float *network_weight_moment1[NT_NUM_NETWORK_LAYERS];
    float *network_weight_moment2[NT_NUM_NETWORK_LAYERS];
    void *network_biases[NT_NUM_NETWORK_LAYERS];           /* fp16, {64, 64, output_channels} */
    float *network_bias_gradients[NT_NUM_NETWORK_LAYERS];
    float *network_bias_moment1[NT_NUM_NETWORK_LAYERS];
    float *network_bias_moment2[NT_NUM_NETWORK_LAYERS];

    NtAdamConstants network_adam;
    NtAdamConstants feature_adam;

    /* Training target (stands in for train.h:69-77 ReferenceTexture): fp16
     * [image_height][image_width][output_channels], sampled with Catmull-Rom and wrap
     * addressing like filter/catmull_rom.h:39-89.  May be NULL for decode without MSE. */
    const void *target;
    float channel_loss_weights[NT_MAX_OUTPUT]; /* train.cu:876-888 channelWeights */

    /* Decode output [image_height * image_width][output_channels] (train.cu:950-955). */
    void *inference_output;
    int32_t inference_output_dtype;  /* NtDtype */
    float *inference_mse_accum;      /* optional: += sum of squared error vs target */

    int32_t image_width;
    int32_t image_height;

    /* Training samples: one jittered sample per cell of a lattice_width x lattice_height
     * lattice laid over the image (train.cu:827-844 uses one cell per texel of a 512^2
     * region; sample_stride_* generalises the cell size in texels). */
    int32_t lattice_width;
    int32_t lattice_height;
    float sample_stride_x;
    float sample_stride_y;
    int32_t texel_offset_x;          /* train.h:153-154 */
    int32_t texel_offset_y;
    int32_t num_samples;             /* must equal lattice_width * lattice_height */
    int32_t step;                    /* train.h:156; Adam uses t = max(step, 1) */
    uint32_t seed;                   /* 0 reproduces the reference's per-sample seeds */

    float *loss_accum;               /* optional: += sum over samples and channels of err^2 */

    /* Row sharding of one material over several calls (no reference counterpart; all zero
     * means the whole material).  nt_invoke_training trains lattice rows
     * [lattice_row0, lattice_row0 + lattice_rows) only (lattice_rows 0: all rows); num_samples
     * stays the whole lattice, so every call scales by the global batch.  Source s (0, 1: the
     * latent grids with their gradients, 2: the target) may hold only stored_rows[s] rows of
     * its full height, starting at full row row_origin[s] and wrapping: full row r lives at
     * stored row (r - row_origin[s]) mod height (stored_rows 0: the full height, origin 0).
     * The stored rows must cover every row the trained samples' footprints reach; a row
     * outside them is skipped and sets bit 1 of the device status word. */
    int32_t lattice_row0, lattice_rows;
    int32_t row_origin[3], stored_rows[3];

    /* Latent representation (train.h:29-64 keeps both in Feature): NT_LATENT_GRID_F16 (0)
     * fp16 channel-interleaved grids, or NT_LATENT_BC6_BLOCKS (1) BC6 block features: per
     * 4x4 block, ceil(C / 3) channel triples of 32 floats (endpoints e0..e3 xyz, 16 pixel
     * indices, partition and mode as int32 bits, 2 unused), gradients and moments in the same
     * layout, decoded with the reference's float BC6 decode (train.cu:161-261, :436-454).
     * UNCONSTRAINED trains grids, BLOCK_FEATURES trains blocks, FINALIZE samples either. */
    int32_t latent_format;

    /* Mip chains (train.h:61 numMips; level choice train.cu:78-103, blend :264-314).  A grid
     * with features[f].num_mips = n > 1 stores its n levels one after another in grid,
     * gradients and moments: level m has max(width >> m, 1) x max(height >> m, 1) texels
     * (train.cu:214-218), or, for block features, max(w_m >> 2, 1) x max(h_m >> 2, 1) blocks
     * of records (train.cu:220-231).  Every sample reads its latents and its target at mip
     * coordinate lod (the reference's uvs.z, 0 in its driver): lod is clamped to [0, n - 1],
     * m0 = floor(lod), m1 = min(m0 + 1, n - 1), and the value is (1 - t) level m0 + t level
     * m1 with t = lod - m0 (t = 0: one level).  Gradients reach the levels read, with the same
     * weights.  The target is a chain of target_num_mips levels of a target_width x
     * target_height image (0: the image size).  A fractional lod needs the tcgen05 engines and
     * fp16 grids; sharded calls need lod 0; inference_mse_accum compares with the target level
     * of an integer lod, which must have the image's size. */
    float lod;
    int32_t target_num_mips;
    int32_t target_width, target_height;

    /* Reference textures (train.h:139-140).  With num_reference_textures > 0 the training target
     * and the inference MSE come from them instead of `target`: texture i fills the next
     * num_channels output channels (train.cu:105-157), each weighted by its loss_weight, and
     * output channels past the textures' are trained towards 0 with weight 1 (train.cu:112-119);
     * channel_loss_weights is then unused.  Needs an unsharded call. */
    NtReferenceTexture reference_textures[NT_MAX_REFERENCE_TEXTURES];
    int32_t num_reference_textures;

    /* Elements per texel in inference_output (0: output_channels).  A larger stride writes
     * channels output_channels .. stride - 1 as 0, so a caller laid out like the reference
     * (train.cu:950-955: NT_OUTPUT_SIZE = 16 fp32 values per texel) reads its layout. */
    int32_t inference_output_stride;

    /* Optional workspace of nt_invoke_training (no reference counterpart): at least
     * nt_workspace_bytes() device bytes, 16-byte aligned, zeroed once by the caller.  With it,
     * the training kernel hands out its tiles through a counter there (each CTA starts on its
     * own tile, then takes the next unclaimed one as it finishes a tile, instead of a fixed
     * share; lattices of fewer than 8 tiles of 128 samples per CTA, BC6 block features and
     * fractional mip levels keep the fixed shares), and the last CTA to finish sets the
     * counter back to zero, so the workspace is zero again after every call.  NULL: fixed
     * shares.  Calls that run at the same time on the GPU must not share a workspace. */
    void *workspace;
    int64_t workspace_bytes;
} NtKernelParams;

/* ---- library ------------------------------------------------------------------------ */
NT_API int32_t nt_version(void);
NT_API const char *nt_get_last_error_string(void);
NT_API size_t nt_kernel_params_size(void);
/* Offset of a named field of NtKernelParams (for binding checks), or (size_t)-1. */
NT_API size_t nt_kernel_params_offset(const char *field);
/* Device bytes of NtKernelParams.workspace (nt_invoke_training's tile counter). */
NT_API size_t nt_workspace_bytes(void);
/* Kernels launched by this library on the calling thread since load (for launch accounting). */
NT_API uint64_t nt_launch_count(void);

/* ---- train.h:158-161 ------------------------------------------------------------------ */

/* train.h:160.  One fused pass over params->num_samples samples: sample latents and
 * target, MLP forward, weighted L2 loss, MLP backward.  ACCUMULATES into the network
 * weight/bias gradients and (UNCONSTRAINED) the latent gradients; the optimizers consume
 * and zero them, as in the reference (train.cu:586, :621, :638). */
NT_API nt_status nt_invoke_training(const NtKernelParams *params, NtTrainingKernelType type,
                             nt_stream_t stream);

/* No counterpart in the reference.  nt_invoke_training for callers that cannot allocate device
 * memory when they train: an engine that reserves its device memory at start-up and may not
 * call cudaMalloc / cudaFree later (they can stall the device and break its memory budget), or
 * a binding that passes parameter blocks only and has no allocator to make a workspace with.
 * The tile counters live in a 256-byte array of device memory owned by the library (the most
 * scratch this call may use; a pass that would need more is rejected with NT_ERR_INVALID_ARG),
 * and params->workspace must be NULL.  It calls no cudaMalloc, cudaFree or other allocating
 * routine.  The first call on a device, with that device current, looks up the array's address
 * (cudaGetSymbolAddress) and keeps it: make that first call before any stream capture starts.
 * All calls on a device share the array and it keeps the last call's contents, so each call
 * zeroes the counters on its stream before the pass; calls whose work overlaps on the GPU (other
 * streams, other host threads) race on the counters and must be ordered on one stream. */
NT_API nt_status nt_invoke_training_static_scratch(const NtKernelParams *params, NtTrainingKernelType type,
                                                   nt_stream_t stream);

/* train.h:158.  Adam over the three weight matrices and bias vectors (train.cu:681-726). */
NT_API nt_status nt_invoke_optimize_network(const NtKernelParams *params, nt_stream_t stream);

/* train.h:159.  Adam over every latent texel of both grids (train.cu:764-803). */
NT_API nt_status nt_invoke_optimize_features(const NtKernelParams *params, NtTrainingKernelType type,
                                      nt_stream_t stream);

/* One launch doing the work of nt_invoke_optimize_network + nt_invoke_optimize_features
 * (no reference counterpart; the reference makes two launches, main.cpp:1072-1076). */
NT_API nt_status nt_invoke_optimize_all(const NtKernelParams *params, nt_stream_t stream);

/* train.h:161.  Decode every texel centre of the image (train.cu:917-961). */
NT_API nt_status nt_invoke_inference(const NtKernelParams *params, nt_stream_t stream);

/* One training step as the reference driver runs it (main.cpp:1071-1077):
 * training pass, then fused Adam over network and latents.  The training type follows
 * latent_format (UNCONSTRAINED for fp16 grids, BLOCK_FEATURES for BC6 block records).
 * The caller increments step. */
NT_API nt_status nt_train_step(const NtKernelParams *params, nt_stream_t stream);

/* ---- tests/forward_pass_test.h:6 ------------------------------------------------------ */

/* Known-answer test of the 12 -> 16 (ReLU) -> 16 network (tests/forward_pass_test.cu:152-275):
 * returns 1 on pass, 0 on fail, and prints the first mismatch.  Runs on the current device. */
NT_API int32_t nt_run_forward_pass_test(void);
/* Same network on caller data: inputs [32][12] fp16, W0/W1 [16][16] column-major fp16,
 * b0/b1 [16] fp16, outputs [32][16] fp16 (all device pointers). */
NT_API nt_status nt_forward_pass_12x16x16(const void *inputs, const void *w0, const void *w1,
                                   const void *b0, const void *b1, void *outputs,
                                   nt_stream_t stream);

/* ---- BC6H latent block codec (train.cu:20-34, :161-202 hold the reference's BC6 pieces) -- */

/* A strided fp16 surface: element (channel c, row y, texel x) lives at
 * data[c * channel_stride + y * row_stride + x * texel_stride] (strides in elements), so
 * planar [C][H][W] latents and channel-interleaved [H][W][C] grids are both addressable.
 * Channels are coded in triples (a missing third channel holds the bias). */
typedef struct NtBc6hSurface {
    void *data;
    int32_t width;
    int32_t height;
    int32_t channels;
    int64_t channel_stride;
    int64_t row_stride;
    int64_t texel_stride;
} NtBc6hSurface;

/* Bytes of the block array of a surface: ceil(channels/3) x ceil(h/4) x ceil(w/4) x 16,
 * stored [triple][block row][block column]. */
NT_API size_t nt_bc6h_blocks_bytes(int32_t width, int32_t height, int32_t channels);
/* Encode half(value + bias) as BC6H UF16 blocks (bias 4 suits latents in [-4, 4]);
 * partial edge blocks replicate the last texel. */
NT_API nt_status nt_bc6h_encode(const NtBc6hSurface *src, void *blocks, float bias,
                                nt_stream_t stream);
/* Decode to half(decoded - bias) into the surface (only texels inside it are written). */
NT_API nt_status nt_bc6h_decode(const void *blocks, const NtBc6hSurface *dst, float bias,
                                nt_stream_t stream);
/* Raw decode of num_blocks blocks to 48 fp16 bit patterns each (16 texels x 3 channels),
 * interpreted as SF16 (is_signed = 1) or UF16. */
NT_API nt_status nt_bc6h_decode_raw(const void *blocks, int64_t num_blocks, int32_t is_signed,
                                    void *texels, nt_stream_t stream);
/* Decode through the GPU texture unit instead: uploads the blocks of one blocks_w x
 * blocks_h surface into a BC6H CUDA array, fetches every texel with point sampling and
 * writes [blocks_h*4][blocks_w*4][4] floats.  Synchronous; allocates and frees the array. */
NT_API nt_status nt_bc6h_decode_hardware(const void *blocks, int32_t blocks_w, int32_t blocks_h,
                                         int32_t is_signed, float *rgba);

/* ---- reference textures (main.cpp:558-637: UploadTexture) -------------------------------- */

/* Texture object over an fp32 chain of num_mips levels (0 or 1: one level), level after level,
 * each [h_m][w_m][c] with c = num_channels, or 4 for 3 channels (the reference uploads RGB as
 * RGBA, main.cpp:216-224, :547), in host or device memory.  The texture uses the reference's
 * descriptor: wrap addressing, linear filtering, normalized coordinates, linear mipmap
 * filtering (main.cpp:609-619).  Allocates device memory: not for use inside a captured graph. */
NT_API nt_status nt_reference_texture_create(const float *chain, int32_t width, int32_t height,
                                             int32_t num_channels, int32_t num_mips, float loss_weight,
                                             NtReferenceTexture *out);
NT_API nt_status nt_reference_texture_destroy(NtReferenceTexture *texture);
/* Samples texture at n coordinates (uv: n x 2 floats, device) and mip coordinate lod with the
 * reference's filter (SampleReferenceTextureTrilinear, train.cu:78-103): out gets n x 4 floats
 * (device; channels past num_channels are 0). */
NT_API nt_status nt_reference_texture_sample(const NtReferenceTexture *texture, const float *uv, int64_t n,
                                             float lod, float *out, nt_stream_t stream);

/* ---- mip chains (no reference counterpart: the reference loads its chains from EXR files,
 * main.cpp:360-433) ------------------------------------------------------------------------ */

/* Texels of an n-level chain of a width x height image (NtKernelParams.lod). */
NT_API int64_t nt_mip_chain_texels(int32_t width, int32_t height, int32_t num_mips);
/* Levels 1 .. num_mips - 1 of an fp16 [texel][channels] chain from its level 0: texel (x, y) of
 * level m is ((a + b) + (c + d)) / 4 in fp32 over texels (2x, 2y), (2x + 1, 2y), (2x, 2y + 1),
 * (2x + 1, 2y + 1) of level m - 1 (clamped to its size), rounded to fp16. */
NT_API nt_status nt_build_mips(void *chain, int32_t width, int32_t height, int32_t channels, int32_t num_mips,
                               nt_stream_t stream);

/* ---- on-disk format (no reference counterpart: the reference's driver reads and writes EXR
 * images, main.cpp:360-556, :855-904, and keeps no training state on disk) -----------------
 *
 * A checkpoint file is a set of named, typed sections in host memory order: an 64-byte header
 * ("NTB2CKPT", version 1, section count, index offset and the index's FNV-1a 64 checksum),
 * the payloads at 64-byte aligned offsets, then the index (per section: name, dtype, shape,
 * offset, bytes and the payload's FNV-1a 64 checksum).  nt_checkpoint_write writes
 * path + ".tmp" and renames it over path, so a reader never sees a partial file.  Reads verify
 * the checksums and return NT_ERR_IO for a missing, truncated or corrupt file.  All buffers are
 * host memory; neural_textures_b200.NeuralTexture.save / load map a material onto sections. */
#define NT_CKPT_NAME_LEN 32
#define NT_CKPT_MAX_SECTIONS 4096
typedef struct NtCheckpointSection {
    char name[NT_CKPT_NAME_LEN]; /* NUL-terminated, non-empty, unique within a file */
    int32_t dtype;               /* NtDtype */
    int32_t ndim;                /* 0 .. 4 */
    int64_t shape[4];
    int64_t bytes;               /* product of the shape x element size */
    const void *data;            /* payload (nt_checkpoint_write); NULL in an index */
} NtCheckpointSection;

NT_API nt_status nt_checkpoint_write(const char *path, const NtCheckpointSection *sections, int32_t count);
/* Fills up to capacity entries (data NULL) and *count with the file's section count; sections
 * may be NULL with capacity 0 to query the count. */
NT_API nt_status nt_checkpoint_index(const char *path, NtCheckpointSection *sections, int32_t capacity,
                                     int32_t *count);
/* Reads section `name` into dst, which must hold exactly its bytes. */
NT_API nt_status nt_checkpoint_read(const char *path, const char *name, void *dst, int64_t bytes);

/* ---- block records <-> BC6H blocks (no reference counterpart: the reference's
 * BLOCK_FEATURES path, train.cu:316-458, starts from and ends in float records) ----------- */

/* Floats of the NT_LATENT_BC6_BLOCKS records of a width x height x channels grid
 * ([height/4][width/4][ceil(channels/3)][NT_BC6F_RECORD_FLOATS]); 0 unless width and height
 * are positive multiples of 4. */
NT_API size_t nt_bc6f_records_floats(int32_t width, int32_t height, int32_t channels);
/* Records from BC6H UF16 blocks in nt_bc6h_encode's layout: e = (31 u 2^b / 64 - 32768) / 31744
 * for unquantized endpoints u, x = weight / 512, partition and mode kept for modes 1-10;
 * one-region blocks give equal regions.  Each record's float decode is within one fp16 ulp
 * of the block's integer decode (the texel values are value + the encoder's bias). */
NT_API nt_status nt_bc6f_from_bc6h(const void *blocks, int32_t width, int32_t height, int32_t channels,
                                   float *records, nt_stream_t stream);
/* BC6H UF16 blocks from records: the record's partition, the best-fitting mode (its own
 * first), nearest palette indices.  A record made by nt_bc6f_from_bc6h returns a block that
 * decodes to the same texels. */
NT_API nt_status nt_bc6f_to_bc6h(const float *records, int32_t width, int32_t height, int32_t channels,
                                 void *blocks, nt_stream_t stream);

/* ---- row-sharded training from one host thread (no reference counterpart) -----------------
 *
 * The reference trains one material on one device (main.cpp:1071-1077).  A material split
 * into bands of lattice rows, one band per shard, trains here with one call per step; the
 * shards may share a device or sit on several.  Shard r of n stores, for each latent grid,
 * `halo_rows` rows above its owned band, the band, and `halo_rows` rows below (its training
 * pass reads and accumulates into all of them); shard r + 1's band follows shard r's, and
 * shard 0's follows shard n - 1's (the grids wrap).  A step is:
 *   1. every shard's training pass (nt_invoke_training with its params);
 *   2. per shard, one kernel that reads its neighbours' memory: the gradients they left in
 *      their halo rows are added to this shard's band edges, and Adam updates this shard's
 *      copy of the network with the sum, in shard order, of every shard's network gradients
 *      (so the copies stay bit-identical); then Adam over the owned band (zero-skip and
 *      gradient zeroing as nt_invoke_optimize_features);
 *   3. per shard, one kernel that copies the neighbours' updated band edges into its halo
 *      rows and zeroes its halo and network gradients.
 * The phases are ordered by events between the shards' streams; no kernel waits on another
 * device.  Shards on different devices need peer access between them, which the call enables
 * (NT_ERR_CUDA if the devices cannot reach each other).  Every shard's buffers must be on its
 * device.  As with nt_train_step the caller advances params.step (main.cpp:1077); all shards
 * must carry the same step, network Adam constants and network shape. */
#define NT_DIST_MAX_SHARDS 16
typedef struct NtShard {
    NtKernelParams params;  /* the band's training pass: lattice_row0 / lattice_rows, and per source
                             * row_origin / stored_rows, as for nt_invoke_training */
    int32_t halo_rows[NT_NUM_FEATURES]; /* per latent grid: stored_rows = owned + 2 * halo_rows */
    int32_t device;         /* CUDA device holding the shard's buffers */
    nt_stream_t stream;     /* a stream on that device (NULL: its default stream) */
} NtShard;

/* The band split used for shards: lattice rows [rank * H / world, (rank + 1) * H / world) of
 * an H-row lattice reach rows [lo, hi) of a source of `height` rows (the range scaled and
 * rounded to the nearest row, so consecutive ranks partition the source).  NT_ERR_INVALID_ARG
 * if a band would be thinner than 2 x `halo` rows (nt_dist_train_step adds halo gradients to
 * both band edges at once) or its stored rows taller than the source. */
NT_API nt_status nt_dist_band(int32_t rank, int32_t world, int32_t lattice_height, int32_t height, int32_t halo,
                              int32_t *lo, int32_t *hi);
/* One training step of a row-sharded material (count 1 .. NT_DIST_MAX_SHARDS; count 1 is
 * nt_train_step).  Returns once every phase is queued; the current device is restored.  Every
 * shard owns its buffers (two shards passing the same buffer are rejected).  The argument
 * checks run before anything is queued; an error returned after that (a failed launch or
 * event record) can leave some shards stepped and others not: the material must then be
 * reloaded (from a checkpoint) before training goes on. */
NT_API nt_status nt_dist_train_step(const NtShard *shards, int32_t count);

/* ---- row-sharded training with one process (or host thread) per GPU over NCCL (no reference
 * counterpart: the reference trains on one device, main.cpp:1071-1077) -----------------------
 *
 * The same band layout as nt_dist_train_step (an NtShard per rank: halo rows above and below the
 * owned band of each latent grid, bands in a ring), but every rank steps only its own shard and
 * the exchanges run over NCCL (NVLink / NVSwitch between the GPUs of a node):
 *   1. the training pass of the band;
 *   2. the gradients of the halo rows go to the neighbours that own those rows (the halo above to
 *      rank - 1, the halo below to rank + 1; NCCL send / receive into the workspace), the
 *      network gradients are summed over the ranks (NCCL all-reduce, in place);
 *   3. the received halo gradients are added to the band's first / last halo_rows rows and the
 *      halo gradients zeroed; Adam on the network (identical on every rank) and on the owned band;
 *   4. the updated first / last halo_rows rows of the band go to the neighbours' halo rows
 *      (NCCL send / receive straight into them).
 * Everything is queued on the shard's stream; nt_nccl_train_step returns once it is queued.  The
 * library loads NCCL (libnccl.so.2) at the first call; NT_ERR_NCCL when it cannot.  The caller
 * passes a workspace of nt_nccl_workspace_bytes(shard) device bytes on the shard's device (the
 * library allocates no device memory; NCCL allocates its own buffers for the communicator). */
#define NT_NCCL_UNIQUE_ID_BYTES 128
typedef struct NtNcclComm NtNcclComm; /* opaque */

/* The communicator id: one rank creates it and hands the 128 bytes to every rank. */
NT_API nt_status nt_nccl_unique_id(void *id);
/* Joins the `world`-rank communicator as `rank` on CUDA device `device` (a collective call: every
 * rank makes it, each from its own process or thread).  *comm is NULL on failure. */
NT_API nt_status nt_nccl_comm_create(const void *id, int32_t world, int32_t rank, int32_t device,
                                     NtNcclComm **comm);
/* Releases the communicator (after its work completed, or after nt_nccl_comm_wait gave up). */
NT_API nt_status nt_nccl_comm_destroy(NtNcclComm *comm);
/* Device bytes of the workspace of nt_nccl_train_step for this shard (16-byte multiple). */
NT_API size_t nt_nccl_workspace_bytes(const NtShard *shard);
/* One training step of this rank's shard (see above); shard->device must be the communicator's
 * device.  All ranks must call it with the same step and the same band plan.  An argument error
 * returns before anything is queued. */
NT_API nt_status nt_nccl_train_step(NtNcclComm *comm, const NtShard *shard, void *workspace,
                                    size_t workspace_bytes);
/* Waits at most timeout_ms for the work queued by this communicator's last nt_nccl_train_step,
 * polling NCCL's asynchronous error state: NT_OK when it completed, NT_ERR_NCCL on an NCCL error
 * and NT_ERR_TIMEOUT when the time ran out; in both error cases the communicator is aborted (its
 * ranks' pending operations end with an error) and must be destroyed. */
NT_API nt_status nt_nccl_comm_wait(NtNcclComm *comm, int32_t timeout_ms);

/* ---- tensor-core self-test (no reference counterpart) ---------------------------------- */

/* Runs the tcgen05 operand layouts of the fused kernels on small known matrices (device
 * pointers): a [128][32], b [64][32], h [128][64] fp16 row-major; writes d1 = a b^T
 * ([128][64] fp32) and d2 = h^T a ([64][32] fp32); *status (device int) gets bit 0 set if
 * the tensor core did not complete within the bounded wait. */
NT_API nt_status nt_umma_selftest(const void *a, const void *b, const void *h, float *d1, float *d2,
                                  int32_t *status, nt_stream_t stream);

/* Device status word of the training kernels (no reference counterpart: the reference has
 * no bounded waits).  Bit 0 is set when a bounded wait inside a kernel gave up; the kernel
 * then stops issuing work and returns.  Synchronises with the device; clear != 0 resets
 * the word. */
NT_API nt_status nt_read_device_status(uint32_t *status, int32_t clear);
/* Exercises the bounded-wait path without a fault: one thread waits on an mbarrier that
 * nothing arrives on, gives up after `tries` polls (1 .. 1,000,000) and sets bit 0 of the
 * status word, as the kernels do on a timeout.  Synchronous. */
NT_API nt_status nt_wait_timeout_selftest(uint32_t tries);

/* ---- seeded set-up helpers (not in the reference: it loads EXR files, main.cpp:436-556) -- */

/* Synthetic target: per channel the sigmoid of a sum of 16 seeded sinusoids with
 * 1..64 cycles per texture and random direction and phase; fp16 [height][width][channels].
 * pbr_normals with 12 channels: channels 3..5 hold the normal of the height channel 9. */
NT_API nt_status nt_generate_target(void *target, int32_t width, int32_t height, int32_t channels,
                             uint32_t seed, int32_t pbr_normals, nt_stream_t stream);
/* Latent grid ~ U(-1, 1), fp16, hash-seeded. */
NT_API nt_status nt_init_latents(void *grid, int64_t count, uint32_t seed, nt_stream_t stream);
/* Device-side L2 flush helper: writes `bytes` of `scratch` (caller-owned). */
NT_API nt_status nt_flush_l2(void *scratch, size_t bytes, nt_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* NT_CAPI_H */

/*
 * nt_oracle.h -- CPU restatement of the reference's neural-texture hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA path and the
 * timed CPU baseline of bench.py; the product never links, loads or calls it.  Only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm use it.
 *
 * Every function cites the reference file:line (mavenkim2/neural_textures) whose behaviour
 * it restates.  Where the build deliberately differs from the reference (Catmull-Rom on
 * the latents instead of bilinear, fp32 accumulation, loss-gradient scaling), the
 * function says so.  Compiled with -ffp-contract=off so that every float expression
 * rounds exactly as written.
 */
#ifndef NT_ORACLE_H
#define NT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- fp16 ------------------------------------------------------------------------ */
uint16_t nto_f2h(float f);  /* round to nearest even, like __float2half */
float nto_h2f(uint16_t h);  /* exact, like __half2float */
void nto_f2h_array(const float *in, uint16_t *out, int64_t n);
void nto_h2f_array(const uint16_t *in, float *out, int64_t n);

/* ---- per-sample RNG and sample placement (train.cu:37-58, :827-844) --------------- */
uint32_t nto_rng_seed(uint32_t sample_index, uint32_t step, uint32_t seed);
uint32_t nto_rng_next(uint32_t *state);
float nto_rng_uniform(uint32_t *state);

typedef struct nto_sampler {
    int32_t image_w, image_h;
    int32_t lattice_w, lattice_h;
    float stride_x, stride_y;
    int32_t offset_x, offset_y;
    int32_t step;
    uint32_t seed;
} nto_sampler;
void nto_sample_uv(const nto_sampler *s, int64_t index, float *u, float *v);
void nto_sample_uv_array(const nto_sampler *s, float *uv /* [n][2] */);

/* ---- Catmull-Rom latent sampling ---------------------------------------------------- */
void nto_catmull_rom_weights(float f, float w[4]);
int32_t nto_wrap(int32_t coord, int32_t size);
/* Sample a channel-interleaved fp16 grid at uv (texel-centre convention, wrap).
 * taps_out (optional): base texel (x, y) and the 4 + 4 weights. */
void nto_sample_grid(const uint16_t *grid, int32_t w, int32_t h, int32_t c, float u, float v,
                     float *out, int32_t base_out[2], float wx_out[4], float wy_out[4]);
void nto_posenc(float u, float v, float out[8]);

/* ---- network -------------------------------------------------------------------------- */
/* ---- BC6 block features (train.cu:161-182, :240-261, :436-454) -------------------------
 * A grid of C channels in block form: per 4x4 block (row-major, width / 4 blocks per row)
 * ceil(C / 3) channel triples of 32 floats: endpoints e0..e3 (xyz, 12 floats), 16 pixel
 * indices, partition (int32 bits), mode (int32 bits, 0..9), 2 unused.  Texel (x, y) of triple
 * t uses region r = partition bit ((y & 3) * 4 + (x & 3)), endpoints e[2r], e[2r + 1], pixel
 * index [(y & 3) * 4 + (x & 3)] and the mode's endpoint precision. */
#define NTO_BC6F_FLOATS 32
void nto_bc6f_decode(const float e0[3], const float e1[3], int32_t bits, float x, float out[3]);
void nto_bc6f_texel(const float *blocks, int32_t w, int32_t channels, int32_t x, int32_t y, float *out);

typedef struct nto_model {
    int32_t channels;       /* C per grid */
    int32_t cout;           /* output channels, <= 16 */
    int32_t gw[2], gh[2];
    const uint16_t *grid[2];
    const float *blocks[2]; /* block-feature form of grid g (NULL: the fp16 grid) */
    const uint16_t *W[3];   /* padded column-major fp16: [64][32], [64][64], [16][64] */
    const uint16_t *b[3];   /* fp16: 64, 64, cout */
    /* Second mip level of grid g (nto_mip_select): features = (1 - t) level + t level_b;
     * mip_t[g] = 0 or grid_b[g] = NULL: one level. */
    const uint16_t *grid_b[2];
    int32_t gw_b[2], gh_b[2];
    float mip_t[2];
} nto_model;

typedef struct nto_fwd {
    float x[32];
    float h1[64];
    float h2[64];
    float y[16];     /* fp16-rounded outputs */
    int32_t base[2][2];
    float wx[2][4], wy[2][4];
    int32_t base_b[2][2];   /* second mip level's footprint (mip_t > 0) */
    float wx_b[2][4], wy_b[2][4];
} nto_fwd;

void nto_forward_sample(const nto_model *m, float u, float v, nto_fwd *f);

/* Decode all texel centres; out is fp16 (out_f32 = 0) or fp32 [h*w][cout].
 * target (optional, fp16 [h][w][cout]) accumulates the SSE into *sse. */
void nto_decode(const nto_model *m, int32_t w, int32_t h, void *out, int32_t out_f32,
                const uint16_t *target, double *sse, int32_t threads);
/* Decode only texel indices [first, first + count) (used for bounded CPU baselines). */
void nto_decode_range(const nto_model *m, int32_t w, int32_t h, int64_t first, int64_t count,
                      void *out, int32_t out_f32, int32_t threads);

/* ---- reference textures (train.cu:78-157, filter/catmull_rom.h:39-89) -----------------
 * An fp32 chain, level after level, [h_m][w_m][cc] with cc = channels (4 for 3 channels).
 * The texture unit's bilinear filter is emulated: wrap addressing of normalized coordinates,
 * texel position x W - 0.5, weights of the two texels per axis from its fraction; the fraction
 * is exact (mode 0), rounded to the nearest 1/256 (1) or truncated to 1/256 (2) -- the CUDA
 * documentation gives 9-bit fixed-point weights with 8 fractional bits. */
typedef struct nto_ref_texture {
    const float *chain;
    int32_t w, h, channels, num_mips;
    float loss_weight;
} nto_ref_texture;
void nto_set_texture_filter_mode(int32_t mode);
void nto_ref_trilinear(const nto_ref_texture *t, float u, float v, float lod, float out[4]);
/* train.cu:105-157: the textures' channels fill expected[] in order, weights = loss_weight (1
 * past the textures) */
void nto_ref_expected(const nto_ref_texture *t, int32_t n, float u, float v, float lod, float expected[16],
                      float weights[16]);

typedef struct nto_train_args {
    const uint16_t *target;    /* fp16 [target_h][target_w][cout] */
    const float *channel_weights; /* [cout] or NULL */
    nto_sampler sampler;
    int32_t finalize;          /* 1: no latent gradients */
    /* mip chains (all zero: one level, target of the image's size) */
    int32_t target_w, target_h;          /* 0: the sampler's image size */
    const uint16_t *target_b;            /* second target level, weight target_t */
    int32_t target_w_b, target_h_b;
    float target_t;
    float *ggrid_b[2];                   /* gradients of the grids' second levels */
    const nto_ref_texture *ref;          /* reference textures (num_ref > 0 replaces target) */
    int32_t num_ref;
    float lod;                           /* their mip coordinate */
} nto_train_args;

/* One training pass: accumulates network and latent gradients (fp32, already scaled by
 * 1 / num_samples) and returns the weighted sum of squared errors. */
double nto_train_pass(const nto_model *m, const nto_train_args *a, float *gW[3], float *gb[3],
                      float *ggrid[2], int32_t threads);
/* Same, restricted to samples [first, first + count) of the lattice (bounded baselines). */
double nto_train_pass_range(const nto_model *m, const nto_train_args *a, int64_t first,
                            int64_t count, float *gW[3], float *gb[3], float *ggrid[2],
                            int32_t threads);

/* ---- mip chains ------------------------------------------------------------------------
 * A chain of n levels stores level m (max(w >> m, 1) x max(h >> m, 1) texels, train.cu:214-218)
 * after level m - 1.  nto_mip_select gives the levels a sample at mip coordinate lod reads
 * (train.cu:78-103, :264-314): lod clamped to [0, n - 1] (NaN: 0), m0 = floor, m1 =
 * min(m0 + 1, n - 1), t = lod - m0 when m1 > m0, else 0; the sample is (1 - t) s(m0) + t s(m1). */
void nto_mip_select(int32_t num_mips, float lod, int32_t *m0, int32_t *m1, float *t);
int32_t nto_mip_dim(int32_t size, int32_t m);
int64_t nto_mip_offset(int32_t w, int32_t h, int32_t m); /* texels before level m */
/* Levels 1 .. n - 1 of an fp16 chain from level 0: 2x2 box average in fp32 ((a + b) + (c + d))
 * * 0.25, source texels clamped to the level below, rounded to fp16. */
void nto_build_mips(uint16_t *chain, int32_t w, int32_t h, int32_t c, int32_t num_mips);

/* ---- Adam (train.cu:521-564, :566-588) ---------------------------------------------- */
void nto_adam_bias_correction(float beta1, float beta2, int32_t step, float *bc1, float *bc2);
void nto_adam_f16(uint16_t *w, float *g, float *m, float *v, int64_t n, float lr, float beta1,
                  float beta2, float eps, float bc1, float bc2);
void nto_adam_f32(float *w, float *g, float *m, float *v, int64_t n, float lr, float beta1,
                  float beta2, float eps, float bc1, float bc2);

/* ---- synthetic target --------------------------------------------------------------- */
void nto_target_params(uint32_t seed, int32_t channel, int32_t k, int32_t *fu, int32_t *fv,
                       float *phase, float *amp);
void nto_generate_target(uint16_t *out, int32_t w, int32_t h, int32_t channels, uint32_t seed,
                         int32_t pbr_normals, int32_t threads);

/* ---- BC6H-style latent block codec (nt_oracle_codec.c) ------------------------------- */
int nto_bc6h_mode_index(const uint8_t block[16]);
/* out: 16 texels x 3 channels of fp16 bits, texels in raster order */
void nto_bc6h_decode_block(const uint8_t block[16], int is_signed, uint16_t out[48]);
/* UF16 encoder: texels are non-negative halves (16 texels x 3 channels) */
void nto_bc6h_encode_block(const uint16_t texels[48], uint8_t out[16]);
/* Surfaces: element (channel c, row y, texel x) at data[c*cstride + y*rstride + x*tstride];
 * channels grouped in triples (a missing third channel encodes as the bias); blocks
 * [ceil(channels/3)][ceil(h/4)][ceil(w/4)] x 16 B of BC6H UF16 holding value + bias;
 * partial blocks replicate the edge texels. */
void nto_bc6h_encode_surface(const uint16_t *data, int32_t w, int32_t h, int32_t channels,
                             int64_t cstride, int64_t rstride, int64_t tstride, float bias,
                             uint8_t *blocks, int32_t threads);
void nto_bc6h_decode_surface(const uint8_t *blocks, int32_t w, int32_t h, int32_t channels,
                             int64_t cstride, int64_t rstride, int64_t tstride, float bias,
                             uint16_t *data, int32_t threads);
/* Float BC6 block records (32 floats per triple, NTO_BC6F_FLOATS) <-> BC6H UF16 blocks;
 * surfaces need w and h multiples of 4: records [h/4][w/4][ceil(channels/3)][32], blocks as
 * above. */
void nto_bc6f_from_bc6h_block(const uint8_t block[16], float rec[32]);
void nto_bc6f_to_bc6h_block(const float rec[32], uint8_t out[16]);
void nto_bc6f_from_bc6h_surface(const uint8_t *blocks, int32_t w, int32_t h, int32_t channels, float *records);
void nto_bc6f_to_bc6h_surface(const float *records, int32_t w, int32_t h, int32_t channels, uint8_t *blocks);

/* ---- tests/forward_pass_test.cu:45-150 known-answer test ---------------------------- */
void nto_fwdtest_generate(uint16_t inputs[32 * 12], uint16_t w0[256], uint16_t w1[256],
                          uint16_t b0[16], uint16_t b1[16]);
void nto_fwdtest_reference(const uint16_t inputs[32 * 12], const uint16_t w0[256],
                           const uint16_t w1[256], const uint16_t b0[16], const uint16_t b1[16],
                           float out[32 * 16]);

#ifdef __cplusplus
}
#endif

#endif

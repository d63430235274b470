// nt_capi.cu -- the extern "C" boundary (include/nt_capi.h): argument validation, launch
// descriptors, per-step Adam constants and error reporting.  No exception crosses the ABI;
// every entry point returns an nt_status and records a message for
// nt_get_last_error_string().
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <utility>

#include "nt_capi.h"
#include "nt_kernels.cuh"

namespace nt {

static std::atomic<uint64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// SM count of the current device, cached per device (host threads may drive devices
// concurrently: the cache is atomic, and a race only repeats the same query).
int sm_count()
{
    static std::atomic<int> cached[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    int n = cached[dev].load(std::memory_order_relaxed);
    if (!n) {
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        n = n > 0 ? n : 148;
        cached[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

cudaError_t set_smem_limit(const void *kernel, size_t bytes)
{
    static std::mutex mu;
    static std::set<std::pair<const void *, int>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({kernel, dev})) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) done.insert({kernel, dev});
    return e;
}

cudaError_t launch_bc6h(const NtBc6hSurface *s, const void *blocks, float bias, bool encode, cudaStream_t st);
cudaError_t launch_bc6h_raw(const void *blocks, int64_t n, int is_signed, void *out, cudaStream_t st);
cudaError_t launch_bc6f_convert(const void *blocks, float *records, int32_t w, int32_t h, int32_t channels,
                                bool to_records, cudaStream_t st);
cudaError_t hardware_decode(const void *blocks, int bw, int bh, int is_signed, float *rgba);
cudaError_t launch_target(void *out, int32_t w, int32_t h, int32_t c, uint32_t seed, int32_t pbr, cudaStream_t st);
cudaError_t launch_init_latents(void *grid, int64_t count, uint32_t seed, cudaStream_t st);
cudaError_t launch_flush(void *scratch, size_t bytes, cudaStream_t st);
cudaError_t launch_build_mips(__half *chain, int32_t w, int32_t h, int32_t c, int32_t num_mips, cudaStream_t st);
cudaError_t ref_texture_create(const float *chain, int w, int h, int ch, int mips, NtReferenceTexture *out);
cudaError_t ref_texture_destroy(NtReferenceTexture *t);
RefTexView ref_view(const NtReferenceTexture &t);
cudaError_t launch_ref_sample(const NtReferenceTexture &t, const float *uv, int64_t n, float lod, float *out,
                              cudaStream_t st);

}  // namespace nt

using namespace nt;

static thread_local std::string g_last_error;

static nt_status fail(nt_status st, const char *fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return st;
}

namespace nt {
// The last-error string for code outside this file (the checkpoint reader and writer).
nt_status set_error(nt_status st, const char *fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return st;
}
}  // namespace nt

static nt_status check_cuda(cudaError_t e, const char *what)
{
    if (e == cudaSuccess) return NT_OK;
    return fail(NT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

#define NT_REQUIRE(cond, ...)                                     \
    do {                                                          \
        if (!(cond)) return fail(NT_ERR_INVALID_ARG, __VA_ARGS__); \
    } while (0)

static nt_status validate_network(const NtKernelParams *p)
{
    NT_REQUIRE(p->latent_channels == 8 || p->latent_channels == 12,
               "latent_channels must be 8 or 12 (got %d)", p->latent_channels);
    NT_REQUIRE(p->output_channels >= 1 && p->output_channels <= NT_MAX_OUTPUT,
               "output_channels must be in [1, %d] (got %d)", NT_MAX_OUTPUT, p->output_channels);
    for (int l = 0; l < NT_NUM_NETWORK_LAYERS; ++l) {
        NT_REQUIRE(p->network_weights[l] && aligned16(p->network_weights[l]),
                   "network_weights[%d] must be a non-null 16-byte aligned device pointer", l);
        NT_REQUIRE(p->network_biases[l], "network_biases[%d] is null", l);
    }
    for (int f = 0; f < NT_NUM_FEATURES; ++f) {
        const NtFeature &ft = p->features[f];
        NT_REQUIRE(ft.grid && aligned16(ft.grid), "features[%d].grid must be a non-null 16-byte aligned pointer", f);
        NT_REQUIRE(ft.width >= 1 && ft.height >= 1, "features[%d] has empty size %dx%d", f, ft.width, ft.height);
        NT_REQUIRE(ft.width <= 32767 && ft.height <= 32767, "features[%d] is wider than 32767 texels", f);
        NT_REQUIRE((int64_t)ft.width * ft.height * p->latent_channels < (int64_t)1 << 31,
                   "features[%d] is too large", f);
        NT_REQUIRE(ft.num_mips >= 0 && ft.num_mips <= 16, "features[%d].num_mips must be in [0, 16] (got %d)", f,
                   ft.num_mips);
        NT_REQUIRE(p->latent_format == NT_LATENT_GRID_F16 ||
                       (p->latent_format == NT_LATENT_BC6_BLOCKS && ft.width % 4 == 0 && ft.height % 4 == 0),
                   "latent_format %d: features[%d] must be %s", p->latent_format, f,
                   p->latent_format == NT_LATENT_BC6_BLOCKS ? "a multiple of 4 texels in each direction"
                                                             : "a known latent format");
    }
    return NT_OK;
}

// ---- mip chains (train.h:61, train.cu:78-103, :214-231, :264-314) --------------------------

static int mip_dim(int size, int m)
{
    const int d = m < 31 ? size >> m : 0;
    return d > 0 ? d : 1;
}

// Units of level m: texels, or 4x4 blocks of records (train.cu:220-231).
static int64_t mip_units(int w, int h, int m, bool blocks)
{
    const int lw = mip_dim(w, m), lh = mip_dim(h, m);
    if (!blocks) return (int64_t)lw * lh;
    return (int64_t)std::max(lw >> 2, 1) * std::max(lh >> 2, 1);
}

static int64_t mip_offset(int w, int h, int m, bool blocks)
{
    int64_t off = 0;
    for (int k = 0; k < m; ++k) off += mip_units(w, h, k, blocks);
    return off;
}

struct MipSel {
    int m0, m1;
    float t;  // weight of level m1; 0: level m0 alone
};

// train.cu:83-87: lod clamped to the chain, levels floor(lod) and the next one.
static MipSel mip_select(int num_mips, float lod)
{
    const int last = num_mips > 1 ? num_mips - 1 : 0;
    float c = lod > 0.f ? lod : 0.f;  // NaN -> 0
    if (c > (float)last) c = (float)last;
    MipSel s;
    s.m0 = std::min((int)floorf(c), last);
    s.m1 = std::min(s.m0 + 1, last);
    s.t = s.m1 > s.m0 ? c - (float)s.m0 : 0.f;
    return s;
}

static int feature_mips(const NtFeature &ft) { return ft.num_mips > 1 ? ft.num_mips : 1; }

// Elements (fp16 texel channels, or record floats) per unit of a latent chain.
static int64_t unit_elems(const NtKernelParams *p)
{
    return p->latent_format == NT_LATENT_BC6_BLOCKS ? (int64_t)((p->latent_channels + 2) / 3) * NT_BC6F_RECORD_FLOATS
                                                     : p->latent_channels;
}

// Level pointers and sizes of grid f at p->lod (training and decode share them).
struct LevelView {
    const void *grid, *grid_b;
    float *grad, *grad_b;
    int w, h, w_b, h_b;
    float t;
    int m0;
};

static LevelView feature_levels(const NtKernelParams *p, int f)
{
    const NtFeature &ft = p->features[f];
    const bool blocks = p->latent_format == NT_LATENT_BC6_BLOCKS;
    const size_t esz = blocks ? sizeof(float) : sizeof(__half);
    const int64_t per = unit_elems(p);
    const MipSel ms = mip_select(feature_mips(ft), p->lod);
    LevelView v;
    const int64_t oa = mip_offset(ft.width, ft.height, ms.m0, blocks) * per;
    const int64_t ob = mip_offset(ft.width, ft.height, ms.m1, blocks) * per;
    v.grid = static_cast<const char *>(ft.grid) + oa * esz;
    v.grid_b = static_cast<const char *>(ft.grid) + ob * esz;
    v.grad = ft.gradients ? ft.gradients + oa : nullptr;
    v.grad_b = ft.gradients ? ft.gradients + ob : nullptr;
    v.w = mip_dim(ft.width, ms.m0);
    v.h = mip_dim(ft.height, ms.m0);
    v.w_b = mip_dim(ft.width, ms.m1);
    v.h_b = mip_dim(ft.height, ms.m1);
    v.t = ms.t;
    v.m0 = ms.m0;
    return v;
}

// Reference textures of the call (train.h:139-140); returns the number used.
static nt_status reference_views(const NtKernelParams *p, RefTexView (&ref)[kMaxRefTextures], int &n)
{
    NT_REQUIRE(p->num_reference_textures >= 0 && p->num_reference_textures <= NT_MAX_REFERENCE_TEXTURES,
               "num_reference_textures must be in [0, %d]", NT_MAX_REFERENCE_TEXTURES);
    n = p->num_reference_textures;
    for (int i = 0; i < n; ++i) {
        const NtReferenceTexture &t = p->reference_textures[i];
        NT_REQUIRE(!t.texture || (t.num_channels >= 1 && t.num_channels <= 4 && t.width >= 1 && t.height >= 1 &&
                                  t.num_mips >= 0 && t.num_mips <= 16),
                   "reference_textures[%d]: 1 .. 4 channels, a positive size and 0 .. 16 mips are required", i);
        ref[i] = ref_view(t);
    }
    return NT_OK;
}

static NetView net_view(const NtKernelParams *p)
{
    NetView n;
    for (int l = 0; l < 3; ++l) {
        n.W[l] = reinterpret_cast<const __half *>(p->network_weights[l]);
        n.b[l] = reinterpret_cast<const __half *>(p->network_biases[l]);
    }
    n.cout = p->output_channels;
    return n;
}

static AdamSegment make_segment(void *w, float *g, float *m, float *v, int64_t n, const NtAdamConstants &c,
                                int32_t step)
{
    AdamSegment s;
    s.w = reinterpret_cast<__half *>(w);
    s.w32 = nullptr;
    s.g = g;
    s.m = m;
    s.v = v;
    s.n = n;
    s.lr = c.learning_rate;
    s.beta1 = c.beta1;
    s.beta2 = c.beta2;
    s.eps = c.epsilon;
    const int t = step > 0 ? step : 1;  // train.cu:528
    s.bc1 = 1.0f - powf(c.beta1, (float)t);
    s.bc2 = 1.0f - powf(c.beta2, (float)t);
    s.first_block = 0;
    return s;
}

static void finalize_adam(AdamLaunch &a)
{
    int blocks = 0;
    for (int i = 0; i < a.nseg; ++i) {
        a.seg[i].first_block = blocks;
        blocks += (int)((a.seg[i].n + kAdamChunk - 1) / kAdamChunk);
    }
    a.total_blocks = blocks;
}

static nt_status add_network_segments(const NtKernelParams *p, AdamLaunch &a)
{
    static const int64_t wcount[3] = {64 * 32, 64 * 64, 16 * 64};
    const int64_t bcount[3] = {64, 64, p->output_channels};
    for (int l = 0; l < 3; ++l) {
        NT_REQUIRE(p->network_weight_gradients[l] && p->network_weight_moment1[l] && p->network_weight_moment2[l],
                   "network weight gradient / moment buffers of layer %d are required", l);
        NT_REQUIRE(p->network_bias_gradients[l] && p->network_bias_moment1[l] && p->network_bias_moment2[l],
                   "network bias gradient / moment buffers of layer %d are required", l);
        a.seg[a.nseg++] = make_segment(p->network_weights[l], p->network_weight_gradients[l],
                                       p->network_weight_moment1[l], p->network_weight_moment2[l], wcount[l],
                                       p->network_adam, p->step);
        a.seg[a.nseg++] = make_segment(p->network_biases[l], p->network_bias_gradients[l],
                                       p->network_bias_moment1[l], p->network_bias_moment2[l], bcount[l],
                                       p->network_adam, p->step);
    }
    return NT_OK;
}

static nt_status add_feature_segments(const NtKernelParams *p, AdamLaunch &a)
{
    for (int f = 0; f < NT_NUM_FEATURES; ++f) {
        const NtFeature &ft = p->features[f];
        NT_REQUIRE(ft.gradients && ft.moment1 && ft.moment2,
                   "features[%d] gradient / moment buffers are required", f);
        // every level of the chain (train.cu:990-1026 runs Adam over all mips)
        const bool blocks = p->latent_format == NT_LATENT_BC6_BLOCKS;
        const int64_t n = mip_offset(ft.width, ft.height, feature_mips(ft), blocks) * unit_elems(p);
        if (blocks) {
            // fp32 block records; partition / mode slots keep a zero gradient and are skipped
            AdamSegment sg = make_segment(nullptr, ft.gradients, ft.moment1, ft.moment2, n, p->feature_adam, p->step);
            sg.w32 = reinterpret_cast<float *>(ft.grid);
            a.seg[a.nseg++] = sg;
        } else {
            a.seg[a.nseg++] = make_segment(ft.grid, ft.gradients, ft.moment1, ft.moment2, n, p->feature_adam, p->step);
        }
    }
    return NT_OK;
}

extern "C" {

int32_t nt_version(void) { return NT_CAPI_VERSION; }

const char *nt_get_last_error_string(void) { return g_last_error.c_str(); }

size_t nt_kernel_params_size(void) { return sizeof(NtKernelParams); }

size_t nt_kernel_params_offset(const char *field)
{
    if (!field) return (size_t)-1;
#define NT_FIELD(name) \
    if (!strcmp(field, #name)) return offsetof(NtKernelParams, name);
    NT_FIELD(features)
    NT_FIELD(latent_channels)
    NT_FIELD(output_channels)
    NT_FIELD(network_weights)
    NT_FIELD(network_weight_gradients)
    NT_FIELD(network_weight_moment1)
    NT_FIELD(network_weight_moment2)
    NT_FIELD(network_biases)
    NT_FIELD(network_bias_gradients)
    NT_FIELD(network_bias_moment1)
    NT_FIELD(network_bias_moment2)
    NT_FIELD(network_adam)
    NT_FIELD(feature_adam)
    NT_FIELD(target)
    NT_FIELD(channel_loss_weights)
    NT_FIELD(inference_output)
    NT_FIELD(inference_output_dtype)
    NT_FIELD(inference_mse_accum)
    NT_FIELD(image_width)
    NT_FIELD(image_height)
    NT_FIELD(lattice_width)
    NT_FIELD(lattice_height)
    NT_FIELD(sample_stride_x)
    NT_FIELD(sample_stride_y)
    NT_FIELD(texel_offset_x)
    NT_FIELD(texel_offset_y)
    NT_FIELD(num_samples)
    NT_FIELD(step)
    NT_FIELD(seed)
    NT_FIELD(loss_accum)
    NT_FIELD(lattice_row0)
    NT_FIELD(lattice_rows)
    NT_FIELD(row_origin)
    NT_FIELD(stored_rows)
    NT_FIELD(latent_format)
    NT_FIELD(lod)
    NT_FIELD(target_num_mips)
    NT_FIELD(target_width)
    NT_FIELD(target_height)
    NT_FIELD(reference_textures)
    NT_FIELD(num_reference_textures)
    NT_FIELD(inference_output_stride)
    NT_FIELD(workspace)
    NT_FIELD(workspace_bytes)
#undef NT_FIELD
    return (size_t)-1;
}

uint64_t nt_launch_count(void) { return g_launches.load(); }

size_t nt_workspace_bytes(void) { return kWorkspaceBytes; }

nt_status nt_invoke_training(const NtKernelParams *p, NtTrainingKernelType type, nt_stream_t stream)
{
    NT_REQUIRE(p, "params is null");
    NT_REQUIRE(type == NT_TRAIN_UNCONSTRAINED || type == NT_TRAIN_BLOCK_FEATURES || type == NT_TRAIN_FINALIZE,
               "unknown training kernel type %d", (int)type);
    nt_status st = validate_network(p);
    if (st != NT_OK) return st;
    NT_REQUIRE(p->num_reference_textures > 0 || (p->target && aligned16(p->target)),
               "target must be a non-null 16-byte aligned device pointer (or reference textures given)");
    NT_REQUIRE(p->image_width >= 1 && p->image_height >= 1, "image size must be positive");
    NT_REQUIRE(p->lattice_width >= 1 && p->lattice_height >= 1, "lattice size must be positive");
    NT_REQUIRE((int64_t)p->lattice_width * p->lattice_height == p->num_samples,
               "num_samples (%d) must equal lattice_width * lattice_height (%d x %d)", p->num_samples,
               p->lattice_width, p->lattice_height);
    NT_REQUIRE(p->sample_stride_x > 0.f && p->sample_stride_y > 0.f, "sample strides must be positive");
    for (int l = 0; l < 3; ++l)
        NT_REQUIRE(p->network_weight_gradients[l] && aligned16(p->network_weight_gradients[l]) &&
                       p->network_bias_gradients[l],
                   "network gradient buffers of layer %d are required (weights 16-byte aligned)", l);
    if (type == NT_TRAIN_UNCONSTRAINED)
        for (int f = 0; f < NT_NUM_FEATURES; ++f)
            NT_REQUIRE(p->features[f].gradients && aligned16(p->features[f].gradients),
                       "features[%d].gradients must be a 16-byte aligned device pointer", f);

    TrainLaunch L;
    memset(&L, 0, sizeof L);
    for (int f = 0; f < 2; ++f) {
        const LevelView v = feature_levels(p, f);
        L.grid[f] = reinterpret_cast<const __half *>(v.grid);
        L.ggrid[f] = v.grad;
        L.gw[f] = v.w;
        L.gh[f] = v.h;
        NT_REQUIRE(p->latent_format != NT_LATENT_BC6_BLOCKS || (v.w % 4 == 0 && v.h % 4 == 0 && v.t == 0.f),
                   "block features sample one mip level whose size is a multiple of 4 (features[%d], lod %g)", f,
                   (double)p->lod);
        if (v.t > 0.f) {
            L.grid_b[f] = reinterpret_cast<const __half *>(v.grid_b);
            L.ggrid_b[f] = v.grad_b;
            L.gw_b[f] = v.w_b;
            L.gh_b[f] = v.h_b;
            L.mip_t[f] = v.t;
        }
    }
    L.net = net_view(p);
    for (int l = 0; l < 3; ++l) {
        L.gW[l] = p->network_weight_gradients[l];
        L.gb[l] = p->network_bias_gradients[l];
    }
    if ((st = reference_views(p, L.ref, L.num_ref)) != NT_OK) return st;
    L.ref_lod = p->lod;
    if (L.num_ref > 0) {  // train.cu:105-157: texture channels in order, each with its loss weight
        int oc = 0;
        for (int c = 0; c < 16; ++c) L.cw[c] = 1.f;
        for (int i = 0; i < L.num_ref && oc < 16; ++i) {
            const NtReferenceTexture &t = p->reference_textures[i];
            if (!t.texture) continue;
            for (int c = 0; c < t.num_channels && oc < 16; ++c) L.cw[oc++] = t.loss_weight;
        }
        L.tw = p->image_width;
        L.th = p->image_height;
    } else {  // target chain at the same lod
        NT_REQUIRE(p->target_num_mips >= 0 && p->target_num_mips <= 16 && p->target_width >= 0 && p->target_height >= 0,
                   "target_num_mips must be in [0, 16] and the target size non-negative");
        const int tw = p->target_width ? p->target_width : p->image_width;
        const int th = p->target_height ? p->target_height : p->image_height;
        const MipSel ts = mip_select(p->target_num_mips, p->lod);
        const __half *t0 = reinterpret_cast<const __half *>(p->target);
        L.target = t0 + mip_offset(tw, th, ts.m0, false) * p->output_channels;
        L.tw = mip_dim(tw, ts.m0);
        L.th = mip_dim(th, ts.m0);
        if (ts.t > 0.f) {
            L.target_b = t0 + mip_offset(tw, th, ts.m1, false) * p->output_channels;
            L.tw_b = mip_dim(tw, ts.m1);
            L.th_b = mip_dim(th, ts.m1);
            L.target_t = ts.t;
        }
    }  // target
    if (!L.num_ref)
        for (int c = 0; c < 16; ++c) L.cw[c] = c < p->output_channels ? p->channel_loss_weights[c] : 0.f;
    L.sampler.image_w = p->image_width;
    L.sampler.image_h = p->image_height;
    L.sampler.lattice_w = p->lattice_width;
    L.sampler.lattice_h = p->lattice_height;
    L.sampler.stride_x = p->sample_stride_x;
    L.sampler.stride_y = p->sample_stride_y;
    L.sampler.offset_x = p->texel_offset_x;
    L.sampler.offset_y = p->texel_offset_y;
    L.sampler.step = (uint32_t)p->step;
    L.sampler.seed = p->seed;
    L.inv_num_samples = 1.0f / (float)p->num_samples;
    L.loss_accum = p->loss_accum;
    if (p->workspace) {
        NT_REQUIRE(p->workspace_bytes >= (int64_t)kWorkspaceBytes && aligned16(p->workspace),
                   "workspace must hold nt_workspace_bytes() = %zu bytes, 16-byte aligned (got %lld)",
                   kWorkspaceBytes, (long long)p->workspace_bytes);
        L.tile_counter = static_cast<uint32_t *>(p->workspace);
    }
    L.finalize = type == NT_TRAIN_FINALIZE;
    // row sharding (all zero: the whole material)
    NT_REQUIRE(p->lattice_row0 >= 0 && p->lattice_rows >= 0 &&
                   (int64_t)p->lattice_row0 + p->lattice_rows <= p->lattice_height,
               "lattice rows [%d, %d + %d) are outside the %d-row lattice", p->lattice_row0, p->lattice_row0,
               p->lattice_rows, p->lattice_height);
    L.lat_row0 = p->lattice_row0;
    L.lat_rows = p->lattice_rows ? p->lattice_rows : p->lattice_height - p->lattice_row0;
    bool sharded = p->lattice_row0 != 0 || L.lat_rows != p->lattice_height;
    for (int s = 0; s < 3; ++s) {
        const int h = s < 2 ? L.gh[s] : L.th;
        NT_REQUIRE(p->stored_rows[s] >= 0 && p->stored_rows[s] <= h && p->row_origin[s] >= 0 && p->row_origin[s] < h,
                   "source %d: stored rows %d from row %d do not fit its %d rows", s, p->stored_rows[s],
                   p->row_origin[s], h);
        L.org[s] = p->stored_rows[s] ? p->row_origin[s] : 0;
        L.rows[s] = p->stored_rows[s] ? p->stored_rows[s] : h;
        sharded = sharded || L.rows[s] != h;
    }
    NT_REQUIRE(!sharded || (p->lod == 0.f && L.th == p->image_height),
               "row sharding needs lod 0 and a target of the image's height");
    NT_REQUIRE(!L.num_ref || !sharded, "reference textures need an unsharded call");
    // latent representation: UNCONSTRAINED trains fp16 grids, BLOCK_FEATURES trains BC6 block
    // features (train.cu:902-913), FINALIZE samples either and trains the network only
    NT_REQUIRE(type != NT_TRAIN_UNCONSTRAINED || p->latent_format == NT_LATENT_GRID_F16,
               "UNCONSTRAINED training needs latent_format NT_LATENT_GRID_F16");
    NT_REQUIRE(type != NT_TRAIN_BLOCK_FEATURES || p->latent_format == NT_LATENT_BC6_BLOCKS,
               "BLOCK_FEATURES training needs latent_format NT_LATENT_BC6_BLOCKS");
    L.blocks = p->latent_format == NT_LATENT_BC6_BLOCKS;
    NT_REQUIRE(!L.blocks || !sharded, "BC6 block features need an unsharded call");
    if (type == NT_TRAIN_BLOCK_FEATURES) L.finalize = 0;
    L.tiles_x = (p->lattice_width + kTileSide - 1) / kTileSide;
    L.tiles_y = (p->lattice_height + kTileSide - 1) / kTileSide;
    return check_cuda(launch_train_tc(L, p->latent_channels, (cudaStream_t)stream), "training kernel");
}

nt_status nt_invoke_optimize_network(const NtKernelParams *p, nt_stream_t stream)
{
    NT_REQUIRE(p, "params is null");
    nt_status st = validate_network(p);
    if (st != NT_OK) return st;
    AdamLaunch a;
    memset(&a, 0, sizeof a);
    if ((st = add_network_segments(p, a)) != NT_OK) return st;
    finalize_adam(a);
    return check_cuda(launch_adam(a, (cudaStream_t)stream), "Adam (network)");
}

nt_status nt_invoke_optimize_features(const NtKernelParams *p, NtTrainingKernelType type, nt_stream_t stream)
{
    NT_REQUIRE(p, "params is null");
    if (type == NT_TRAIN_FINALIZE) return NT_OK;  // main.cpp:1074: features are frozen
    // OptimizeFeatures<UNCONSTRAINED> / <BLOCK_FEATURES> (train.cu:990-1026): the type names the representation
    NT_REQUIRE(type == (p->latent_format == NT_LATENT_BC6_BLOCKS ? NT_TRAIN_BLOCK_FEATURES : NT_TRAIN_UNCONSTRAINED),
               "optimiser type %d does not match latent_format %d", (int)type, p->latent_format);
    nt_status st = validate_network(p);
    if (st != NT_OK) return st;
    AdamLaunch a;
    memset(&a, 0, sizeof a);
    if ((st = add_feature_segments(p, a)) != NT_OK) return st;
    finalize_adam(a);
    return check_cuda(launch_adam(a, (cudaStream_t)stream), "Adam (features)");
}

nt_status nt_invoke_optimize_all(const NtKernelParams *p, nt_stream_t stream)
{
    NT_REQUIRE(p, "params is null");
    nt_status st = validate_network(p);
    if (st != NT_OK) return st;
    AdamLaunch a;
    memset(&a, 0, sizeof a);
    if ((st = add_network_segments(p, a)) != NT_OK) return st;
    if ((st = add_feature_segments(p, a)) != NT_OK) return st;
    finalize_adam(a);
    return check_cuda(launch_adam(a, (cudaStream_t)stream), "Adam (fused)");
}

nt_status nt_invoke_inference(const NtKernelParams *p, nt_stream_t stream)
{
    NT_REQUIRE(p, "params is null");
    nt_status st = validate_network(p);
    if (st != NT_OK) return st;
    NT_REQUIRE(p->image_width >= 1 && p->image_height >= 1, "image size must be positive");
    NT_REQUIRE(p->inference_output, "inference_output is null");
    NT_REQUIRE(p->latent_format == NT_LATENT_GRID_F16,
               "inference samples fp16 latent grids (train.cu:935, SampleUnconstrainedFeaturesTrilinear)");
    NT_REQUIRE(p->inference_output_dtype == NT_DTYPE_F16 || p->inference_output_dtype == NT_DTYPE_F32,
               "inference_output_dtype must be NT_DTYPE_F16 or NT_DTYPE_F32");
    NT_REQUIRE(p->inference_output_stride == 0 ||
                   (p->inference_output_stride >= p->output_channels && p->inference_output_stride <= NT_MAX_OUTPUT),
               "inference_output_stride (%d) must be 0 or in [output_channels, %d]", p->inference_output_stride,
               NT_MAX_OUTPUT);
    const int out_stride = p->inference_output_stride ? p->inference_output_stride : p->output_channels;
    NT_REQUIRE(!(p->inference_output_dtype == NT_DTYPE_F16 && out_stride == 8) || aligned16(p->inference_output),
               "inference_output must be 16-byte aligned");
    NT_REQUIRE(!p->inference_mse_accum || p->target || p->num_reference_textures > 0,
               "inference_mse_accum requires a target or reference textures");
    DecodeLaunch L;
    memset(&L, 0, sizeof L);
    for (int f = 0; f < 2; ++f) {
        const LevelView v = feature_levels(p, f);
        L.grid[f] = reinterpret_cast<const __half *>(v.grid);
        L.gw[f] = v.w;
        L.gh[f] = v.h;
        if (v.t > 0.f) {
            L.grid_b[f] = reinterpret_cast<const __half *>(v.grid_b);
            L.gw_b[f] = v.w_b;
            L.gh_b[f] = v.h_b;
            L.mip_t[f] = v.t;
        }
    }
    L.net = net_view(p);
    L.out = p->inference_output;
    L.out_f32 = p->inference_output_dtype == NT_DTYPE_F32;
    L.out_stride = out_stride;
    // the target is read only for the squared error
    L.target = p->inference_mse_accum ? reinterpret_cast<const __half *>(p->target) : nullptr;
    if ((st = reference_views(p, L.ref, L.num_ref)) != NT_OK) return st;
    L.ref_lod = p->lod;
    if (L.num_ref > 0) {
        L.target = nullptr;  // the MSE compares with the textures
    } else if (p->inference_mse_accum) {  // the target level of this lod, texel for texel
        const int tw = p->target_width ? p->target_width : p->image_width;
        const int th = p->target_height ? p->target_height : p->image_height;
        const MipSel ts = mip_select(p->target_num_mips, p->lod);
        NT_REQUIRE(ts.t == 0.f && mip_dim(tw, ts.m0) == p->image_width && mip_dim(th, ts.m0) == p->image_height,
                   "inference_mse_accum needs an integer lod whose target level has the image's size");
        L.target += mip_offset(tw, th, ts.m0, false) * p->output_channels;
    }
    L.mse_accum = p->inference_mse_accum;
    L.image_w = p->image_width;
    L.image_h = p->image_height;
    L.tiles_x = (p->image_width + kTileSide - 1) / kTileSide;
    L.tiles_y = (p->image_height + kTileSide - 1) / kTileSide;
    return check_cuda(launch_decode_tc(L, p->latent_channels, (cudaStream_t)stream), "decode kernel");
}

nt_status nt_train_step(const NtKernelParams *p, nt_stream_t stream)
{
    NT_REQUIRE(p, "params is null");
    const NtTrainingKernelType type =
        p->latent_format == NT_LATENT_BC6_BLOCKS ? NT_TRAIN_BLOCK_FEATURES : NT_TRAIN_UNCONSTRAINED;
    nt_status st = nt_invoke_training(p, type, stream);
    if (st != NT_OK) return st;
    return nt_invoke_optimize_all(p, stream);
}

size_t nt_bc6h_blocks_bytes(int32_t width, int32_t height, int32_t channels)
{
    if (width < 1 || height < 1 || channels < 1) return 0;
    return (size_t)((channels + 2) / 3) * (size_t)((height + 3) / 4) * (size_t)((width + 3) / 4) * 16u;
}

static nt_status validate_surface(const NtBc6hSurface *s, const void *blocks)
{
    NT_REQUIRE(s, "surface is null");
    NT_REQUIRE(s->data && (reinterpret_cast<uintptr_t>(s->data) & 1u) == 0, "surface data must be a 2-byte aligned pointer");
    NT_REQUIRE(blocks && aligned16(blocks), "blocks must be a 16-byte aligned device pointer");
    NT_REQUIRE(s->width >= 1 && s->height >= 1 && s->channels >= 1, "surface size must be positive");
    NT_REQUIRE(s->channel_stride >= 0 && s->row_stride >= 0 && s->texel_stride >= 0, "strides must be non-negative");
    return NT_OK;
}

nt_status nt_bc6h_encode(const NtBc6hSurface *src, void *blocks, float bias, nt_stream_t stream)
{
    nt_status st = validate_surface(src, blocks);
    if (st != NT_OK) return st;
    return check_cuda(launch_bc6h(src, blocks, bias, true, (cudaStream_t)stream), "BC6H encode");
}

nt_status nt_bc6h_decode(const void *blocks, const NtBc6hSurface *dst, float bias, nt_stream_t stream)
{
    nt_status st = validate_surface(dst, blocks);
    if (st != NT_OK) return st;
    return check_cuda(launch_bc6h(dst, blocks, bias, false, (cudaStream_t)stream), "BC6H decode");
}

nt_status nt_bc6h_decode_raw(const void *blocks, int64_t num_blocks, int32_t is_signed, void *texels,
                             nt_stream_t stream)
{
    NT_REQUIRE(blocks && aligned16(blocks), "blocks must be a 16-byte aligned device pointer");
    NT_REQUIRE(texels, "texels is null");
    NT_REQUIRE(num_blocks >= 0, "num_blocks must be non-negative");
    if (num_blocks == 0) return NT_OK;
    return check_cuda(launch_bc6h_raw(blocks, num_blocks, is_signed, texels, (cudaStream_t)stream), "BC6H raw decode");
}

size_t nt_bc6f_records_floats(int32_t width, int32_t height, int32_t channels)
{
    if (width < 4 || height < 4 || width % 4 || height % 4 || channels < 1) return 0;
    return (size_t)(width / 4) * (size_t)(height / 4) * (size_t)((channels + 2) / 3) * NT_BC6F_RECORD_FLOATS;
}

static nt_status validate_records(const void *blocks, const float *records, int32_t w, int32_t h, int32_t channels)
{
    NT_REQUIRE(blocks && aligned16(blocks), "blocks must be a 16-byte aligned device pointer");
    NT_REQUIRE(records && aligned16(records), "records must be a 16-byte aligned device pointer");
    NT_REQUIRE(w >= 4 && h >= 4 && w % 4 == 0 && h % 4 == 0,
               "block records need a width and height that are positive multiples of 4 (got %d x %d)", w, h);
    NT_REQUIRE(channels >= 1, "channels must be positive");
    return NT_OK;
}

nt_status nt_bc6f_from_bc6h(const void *blocks, int32_t width, int32_t height, int32_t channels, float *records,
                            nt_stream_t stream)
{
    nt_status st = validate_records(blocks, records, width, height, channels);
    if (st != NT_OK) return st;
    return check_cuda(launch_bc6f_convert(blocks, records, width, height, channels, true, (cudaStream_t)stream),
                      "BC6H blocks to block records");
}

nt_status nt_bc6f_to_bc6h(const float *records, int32_t width, int32_t height, int32_t channels, void *blocks,
                          nt_stream_t stream)
{
    nt_status st = validate_records(blocks, records, width, height, channels);
    if (st != NT_OK) return st;
    return check_cuda(launch_bc6f_convert(blocks, const_cast<float *>(records), width, height, channels, false,
                                          (cudaStream_t)stream),
                      "block records to BC6H blocks");
}

nt_status nt_bc6h_decode_hardware(const void *blocks, int32_t blocks_w, int32_t blocks_h, int32_t is_signed,
                                  float *rgba)
{
    NT_REQUIRE(blocks && rgba, "blocks and rgba are required");
    NT_REQUIRE(blocks_w >= 1 && blocks_h >= 1, "block counts must be positive");
    return check_cuda(hardware_decode(blocks, blocks_w, blocks_h, is_signed, rgba), "BC6H hardware decode");
}

nt_status nt_generate_target(void *target, int32_t width, int32_t height, int32_t channels, uint32_t seed,
                             int32_t pbr_normals, nt_stream_t stream)
{
    NT_REQUIRE(target, "target is null");
    NT_REQUIRE(width >= 1 && height >= 1, "target size must be positive");
    NT_REQUIRE(channels >= 1 && channels <= 16, "target channels must be in [1, 16]");
    return check_cuda(launch_target(target, width, height, channels, seed, pbr_normals, (cudaStream_t)stream),
                      "target generator");
}

nt_status nt_init_latents(void *grid, int64_t count, uint32_t seed, nt_stream_t stream)
{
    NT_REQUIRE(grid, "grid is null");
    NT_REQUIRE(count >= 0, "count must be non-negative");
    if (count == 0) return NT_OK;
    return check_cuda(launch_init_latents(grid, count, seed, (cudaStream_t)stream), "latent init");
}

nt_status nt_reference_texture_create(const float *chain, int32_t width, int32_t height, int32_t num_channels,
                                      int32_t num_mips, float loss_weight, NtReferenceTexture *out)
{
    NT_REQUIRE(chain && out, "chain and out are required");
    NT_REQUIRE(width >= 1 && height >= 1 && width <= 65536 && height <= 65536, "texture size must be in [1, 65536]");
    NT_REQUIRE(num_channels >= 1 && num_channels <= 4, "num_channels must be 1 .. 4");
    NT_REQUIRE(num_mips >= 0 && num_mips <= 16, "num_mips must be in [0, 16]");
    memset(out, 0, sizeof *out);
    out->loss_weight = loss_weight;
    return check_cuda(ref_texture_create(chain, width, height, num_channels, num_mips, out), "reference texture");
}

nt_status nt_reference_texture_destroy(NtReferenceTexture *texture)
{
    NT_REQUIRE(texture, "texture is null");
    return check_cuda(ref_texture_destroy(texture), "reference texture release");
}

nt_status nt_reference_texture_sample(const NtReferenceTexture *texture, const float *uv, int64_t n, float lod,
                                      float *out, nt_stream_t stream)
{
    NT_REQUIRE(texture && texture->texture, "texture is null");
    NT_REQUIRE(n >= 0, "n must be non-negative");
    if (n == 0) return NT_OK;
    NT_REQUIRE(uv && out && aligned16(out) && (reinterpret_cast<uintptr_t>(uv) & 7u) == 0,
               "uv (8-byte aligned) and out (16-byte aligned) device pointers are required");
    return check_cuda(launch_ref_sample(*texture, uv, n, lod, out, (cudaStream_t)stream), "reference texture sample");
}

int64_t nt_mip_chain_texels(int32_t width, int32_t height, int32_t num_mips)
{
    if (width < 1 || height < 1 || num_mips < 0 || num_mips > 16) return 0;
    return mip_offset(width, height, num_mips > 1 ? num_mips : 1, false);
}

nt_status nt_build_mips(void *chain, int32_t width, int32_t height, int32_t channels, int32_t num_mips,
                        nt_stream_t stream)
{
    NT_REQUIRE(chain && (reinterpret_cast<uintptr_t>(chain) & 1u) == 0, "chain must be a 2-byte aligned device pointer");
    NT_REQUIRE(width >= 1 && height >= 1 && channels >= 1, "chain size must be positive");
    NT_REQUIRE(num_mips >= 0 && num_mips <= 16, "num_mips must be in [0, 16]");
    if (num_mips <= 1) return NT_OK;
    return check_cuda(launch_build_mips(reinterpret_cast<__half *>(chain), width, height, channels, num_mips,
                                        (cudaStream_t)stream),
                      "mip chain build");
}

nt_status nt_flush_l2(void *scratch, size_t bytes, nt_stream_t stream)
{
    NT_REQUIRE(scratch && aligned16(scratch), "scratch must be a 16-byte aligned device pointer");
    if (bytes < 16) return NT_OK;
    return check_cuda(launch_flush(scratch, bytes, (cudaStream_t)stream), "L2 flush");
}

}  // extern "C"

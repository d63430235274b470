// nt_dist.cu -- one training step of a row-sharded material (config 4b) driven from one host
// thread, with the exchanges done by kernels that read the neighbouring shards' memory.
//
// The reference trains one material on one device (main.cpp:1071-1077); its per-step work is
// InvokeTraining, InvokeOptimizeNetwork and InvokeOptimizeFeatures (train.cu:985-1026).  For
// a material split into bands of lattice rows (one per shard), the step here is:
//   phase 1  every shard: the training pass over its band (nt_invoke_training);
//   phase 2  every shard, after every phase 1: dist_reduce_kernel -- the gradients that the
//            neighbours' samples left in their halo rows are added to this shard's band edges
//            (read from the neighbours' memory), and Adam (train.cu:521-543, zero-skip of
//            :580-583) updates this shard's copy of the network with the sum of every shard's
//            network gradients, read from their memory and summed in shard order; then Adam
//            over the owned band (the fused Adam launch, own memory);
//   phase 3  every shard, after every phase 2: dist_refresh_kernel -- the neighbours' updated
//            band edges are copied into this shard's halo rows, and this shard's halo and
//            network gradients are zeroed (every reader of them has finished).
// Each kernel writes only its own shard's memory, and reads of another shard's memory happen
// only after that shard's writes are complete: the phases are ordered by events recorded on
// the shards' streams and waited on by the other streams (cudaStreamWaitEvent), never by a
// kernel waiting on a flag.  The result equals the single-device step up to the order of
// float additions (the same as the NCCL path of neural_textures_b200/sharded.py).
#include <cstring>
#include <mutex>
#include <vector>

#include "nt_adam_math.cuh"
#include "nt_kernels.cuh"

namespace nt {

nt_status set_error(nt_status st, const char *fmt, ...);

constexpr int kDistThreads = 256;
constexpr int kDistPerThread = 4;  // floats (or fp16 pairs) per thread and block pass

struct DistAddSeg {  // dst[i] += src[i], n floats
    float *dst;
    const float *src;
    int64_t n;
};

struct DistNetSeg {  // Adam on w / m / v with g = sum over shards of g[k][i]
    __half *w;
    float *m, *v;
    const float *g[NT_DIST_MAX_SHARDS];
    int64_t n;
};

struct DistReduceLaunch {
    DistAddSeg add[2 * NT_NUM_FEATURES];
    DistNetSeg net[2 * NT_NUM_NETWORK_LAYERS];
    int32_t nadd, nnet, nshards;
    float lr, beta1, beta2, eps, bc1, bc2;
};

struct DistCopySeg {  // dst[i] = src[i], n fp16 values
    __half *dst;
    const __half *src;
    int64_t n;
};

struct DistZeroSeg {
    float *dst;
    int64_t n;
};

struct DistRefreshLaunch {
    DistCopySeg copy[2 * NT_NUM_FEATURES];
    DistZeroSeg zero[2 * NT_NUM_FEATURES + 2 * NT_NUM_NETWORK_LAYERS];
    int32_t ncopy, nzero;
};

__device__ __forceinline__ bool aligned_to(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// blockIdx.y picks the segment (band-edge additions first, then the network segments);
// blockIdx.x strides over its entries.
__global__ void __launch_bounds__(kDistThreads) dist_reduce_kernel(const DistReduceLaunch p)
{
    const int seg = blockIdx.y;
    const int64_t stride = (int64_t)gridDim.x * kDistThreads;
    const int64_t t0 = (int64_t)blockIdx.x * kDistThreads + threadIdx.x;
    if (seg < p.nadd) {
        const DistAddSeg s = p.add[seg];
        if (aligned_to(s.dst, 16) && aligned_to(s.src, 16)) {
            const int64_t n4 = s.n / 4;
            for (int64_t i = t0; i < n4; i += stride) {
                float4 a = reinterpret_cast<float4 *>(s.dst)[i];
                const float4 b = reinterpret_cast<const float4 *>(s.src)[i];
                a.x = __fadd_rn(a.x, b.x);
                a.y = __fadd_rn(a.y, b.y);
                a.z = __fadd_rn(a.z, b.z);
                a.w = __fadd_rn(a.w, b.w);
                reinterpret_cast<float4 *>(s.dst)[i] = a;
            }
            for (int64_t i = 4 * n4 + t0; i < s.n; i += stride) s.dst[i] = __fadd_rn(s.dst[i], s.src[i]);
        } else {
            for (int64_t i = t0; i < s.n; i += stride) s.dst[i] = __fadd_rn(s.dst[i], s.src[i]);
        }
        return;
    }
    const int k = seg - p.nadd;
    if (k >= p.nnet) return;
    const DistNetSeg &s = p.net[k];
    for (int64_t i = t0; i < s.n; i += stride) {
        float g = 0.f;
        for (int r = 0; r < p.nshards; ++r) g = __fadd_rn(g, s.g[r][i]);  // shard order: same sum everywhere
        if (g == 0.f) continue;  // OptimizeParameterBuffer skips zero gradients (train.cu:580-583)
        float m = s.m[i], v = s.v[i];
        s.w[i] = __float2half_rn(
            adam_update(__half2float(s.w[i]), g, m, v, p.lr, p.beta1, p.beta2, p.eps, p.bc1, p.bc2));
        s.m[i] = m;
        s.v[i] = v;
    }
}

__global__ void __launch_bounds__(kDistThreads) dist_refresh_kernel(const DistRefreshLaunch p)
{
    const int seg = blockIdx.y;
    const int64_t stride = (int64_t)gridDim.x * kDistThreads;
    const int64_t t0 = (int64_t)blockIdx.x * kDistThreads + threadIdx.x;
    if (seg < p.ncopy) {
        const DistCopySeg s = p.copy[seg];
        if (aligned_to(s.dst, 16) && aligned_to(s.src, 16)) {
            const int64_t n8 = s.n / 8;
            for (int64_t i = t0; i < n8; i += stride)
                reinterpret_cast<uint4 *>(s.dst)[i] = reinterpret_cast<const uint4 *>(s.src)[i];
            for (int64_t i = 8 * n8 + t0; i < s.n; i += stride) s.dst[i] = s.src[i];
        } else {
            for (int64_t i = t0; i < s.n; i += stride) s.dst[i] = s.src[i];
        }
        return;
    }
    const int k = seg - p.ncopy;
    if (k >= p.nzero) return;
    const DistZeroSeg s = p.zero[k];
    if (aligned_to(s.dst, 16)) {
        const int64_t n4 = s.n / 4;
        for (int64_t i = t0; i < n4; i += stride) reinterpret_cast<float4 *>(s.dst)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int64_t i = 4 * n4 + t0; i < s.n; i += stride) s.dst[i] = 0.f;
    } else {
        for (int64_t i = t0; i < s.n; i += stride) s.dst[i] = 0.f;
    }
}

static int dist_blocks(int64_t max_n)
{
    const int64_t per_block = (int64_t)kDistThreads * kDistPerThread;
    const int64_t b = (max_n + per_block - 1) / per_block;
    return (int)(b < 1 ? 1 : (b > 1184 ? 1184 : b));
}

// ---- host side -----------------------------------------------------------------------------

namespace {

// Events reused from step to step: a wait enqueued by cudaStreamWaitEvent refers to the
// record made before it, so recording the same event again in the next step is safe.  One
// pool per host thread: two threads stepping two materials never share an event.
struct EventPool {
    std::vector<std::pair<int, cudaEvent_t>> events;  // (device, event), indexed by slot

    ~EventPool()
    {
        for (auto &e : events)
            if (e.second) cudaEventDestroy(e.second);
    }

    cudaError_t get(int slot, int device, cudaEvent_t *out)
    {
        if ((int)events.size() <= slot) events.resize(slot + 1, {-1, nullptr});
        auto &e = events[slot];
        if (e.second && e.first != device) {
            cudaEventDestroy(e.second);  // the slot moved to another device: recreate it there
            e.second = nullptr;
        }
        if (!e.second) {
            cudaError_t err = cudaEventCreateWithFlags(&e.second, cudaEventDisableTiming);
            if (err != cudaSuccess) {
                e.second = nullptr;
                return err;
            }
            e.first = device;
        }
        *out = e.second;
        return cudaSuccess;
    }
};

thread_local EventPool g_events;

std::mutex g_peer_mu;
std::vector<std::pair<int, int>> g_peer_enabled;

// Peer access from `dev` to `peer` (enabled once per pair and process).
nt_status ensure_peer(int dev, int peer)
{
    if (dev == peer) return NT_OK;
    std::lock_guard<std::mutex> lock(g_peer_mu);
    for (auto &pr : g_peer_enabled)
        if (pr.first == dev && pr.second == peer) return NT_OK;
    int can = 0;
    cudaError_t e = cudaDeviceCanAccessPeer(&can, dev, peer);
    if (e != cudaSuccess) return set_error(NT_ERR_CUDA, "cudaDeviceCanAccessPeer(%d, %d): %s", dev, peer, cudaGetErrorString(e));
    if (!can) return set_error(NT_ERR_CUDA, "device %d cannot access device %d's memory (no peer path)", dev, peer);
    if ((e = cudaSetDevice(dev)) != cudaSuccess)
        return set_error(NT_ERR_CUDA, "cudaSetDevice(%d): %s", dev, cudaGetErrorString(e));
    e = cudaDeviceEnablePeerAccess(peer, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        e = cudaSuccess;
    }
    if (e != cudaSuccess)
        return set_error(NT_ERR_CUDA, "cudaDeviceEnablePeerAccess(%d -> %d): %s", dev, peer, cudaGetErrorString(e));
    g_peer_enabled.push_back({dev, peer});
    return NT_OK;
}

// The buffer must be device memory of `device` (a kernel on another device reaches it only
// through a peer mapping, so a host or foreign pointer is refused before any launch).
nt_status check_on_device(const void *ptr, int device, const char *what, int shard)
{
    if (!ptr) return set_error(NT_ERR_INVALID_ARG, "shard %d: %s is null", shard, what);
    cudaPointerAttributes a;
    cudaError_t e = cudaPointerGetAttributes(&a, ptr);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(NT_ERR_INVALID_ARG, "shard %d: %s is not a CUDA pointer (%s)", shard, what, cudaGetErrorString(e));
    }
    if (a.type != cudaMemoryTypeDevice || a.device != device)
        return set_error(NT_ERR_INVALID_ARG, "shard %d: %s is not device memory of device %d", shard, what, device);
    return NT_OK;
}

struct DeviceRestore {
    int dev = -1;
    DeviceRestore() { cudaGetDevice(&dev); }
    ~DeviceRestore()
    {
        if (dev >= 0) cudaSetDevice(dev);
    }
};

constexpr int64_t kNetWeights[NT_NUM_NETWORK_LAYERS] = {64 * 32, 64 * 64, 16 * 64};

int64_t net_biases(const NtKernelParams &p, int l) { return l < 2 ? 64 : p.output_channels; }

#define DIST_REQUIRE(cond, ...)                                   \
    do {                                                          \
        if (!(cond)) return set_error(NT_ERR_INVALID_ARG, __VA_ARGS__); \
    } while (0)

// Host-only checks: sizes, band layout and agreement between the shards.
nt_status validate_shards(const NtShard *sh, int n)
{
    const NtKernelParams &p0 = sh[0].params;
    for (int r = 0; r < n; ++r) {
        const NtKernelParams &p = sh[r].params;
        DIST_REQUIRE(p.latent_format == NT_LATENT_GRID_F16, "shard %d: sharded training needs fp16 latent grids", r);
        DIST_REQUIRE(p.latent_channels == p0.latent_channels && p.output_channels == p0.output_channels,
                     "shard %d: network shape differs from shard 0", r);
        DIST_REQUIRE(p.step == p0.step, "shard %d: step %d differs from shard 0's %d", r, p.step, p0.step);
        DIST_REQUIRE(p.num_samples == p0.num_samples && p.lattice_width == p0.lattice_width &&
                         p.lattice_height == p0.lattice_height && p.image_width == p0.image_width &&
                         p.image_height == p0.image_height,
                     "shard %d: image, lattice or num_samples differs from shard 0 (every band scales its "
                     "gradients by the whole material's sample count)", r);
        DIST_REQUIRE(!memcmp(&p.network_adam, &p0.network_adam, sizeof p.network_adam),
                     "shard %d: network Adam constants differ from shard 0", r);
        DIST_REQUIRE(sh[r].device >= 0, "shard %d: device %d", r, sh[r].device);
        for (int g = 0; g < NT_NUM_FEATURES; ++g) {
            const NtFeature &f = p.features[g], &f0 = p0.features[g];
            DIST_REQUIRE(f.width == f0.width && f.height == f0.height, "shard %d: grid %d size differs from shard 0", r, g);
            DIST_REQUIRE(f.num_mips <= 1, "shard %d: grid %d: sharded grids hold one level", r, g);
            const int halo = sh[r].halo_rows[g], stored = p.stored_rows[g];
            DIST_REQUIRE(halo == sh[0].halo_rows[g], "shard %d: grid %d: halo_rows differs from shard 0", r, g);
            DIST_REQUIRE(halo >= 1 && stored > 2 * halo && stored <= f.height,
                         "shard %d: grid %d: %d stored rows cannot hold a band between two %d-row halos", r, g, stored, halo);
            // the first and the last halo_rows of the band take the neighbours' halo gradients in
            // one launch: they must not overlap
            DIST_REQUIRE(stored - 2 * halo >= 2 * halo, "shard %d: grid %d: band of %d rows is thinner than two %d-row halos",
                         r, g, stored - 2 * halo, halo);
        }
    }
    // every shard owns its buffers: two shards updating one buffer in place would race (their
    // Adam kernels run on different streams) and apply the update once per shard
    for (int r = 0; r < n; ++r) {
        const NtKernelParams &p = sh[r].params;
        for (int q = 0; q < r; ++q) {
            const NtKernelParams &o = sh[q].params;
            for (int l = 0; l < NT_NUM_NETWORK_LAYERS; ++l) {
                const void *a[8] = {p.network_weights[l], p.network_weight_gradients[l], p.network_weight_moment1[l],
                                    p.network_weight_moment2[l], p.network_biases[l], p.network_bias_gradients[l],
                                    p.network_bias_moment1[l], p.network_bias_moment2[l]};
                const void *b[8] = {o.network_weights[l], o.network_weight_gradients[l], o.network_weight_moment1[l],
                                    o.network_weight_moment2[l], o.network_biases[l], o.network_bias_gradients[l],
                                    o.network_bias_moment1[l], o.network_bias_moment2[l]};
                for (int i = 0; i < 8; ++i)
                    DIST_REQUIRE(!a[i] || a[i] != b[i], "shards %d and %d share a network buffer of layer %d", q, r, l);
            }
            for (int g = 0; g < NT_NUM_FEATURES; ++g) {
                const NtFeature &f = p.features[g], &e = o.features[g];
                const void *a[4] = {f.grid, f.gradients, f.moment1, f.moment2};
                const void *b[4] = {e.grid, e.gradients, e.moment1, e.moment2};
                for (int i = 0; i < 4; ++i)
                    DIST_REQUIRE(!a[i] || a[i] != b[i], "shards %d and %d share a buffer of latent grid %d", q, r, g);
            }
        }
    }
    for (int g = 0; g < NT_NUM_FEATURES; ++g) {  // bands tile the grid in a ring
        const int h = p0.features[g].height, halo = sh[0].halo_rows[g];
        int64_t total = 0;
        for (int r = 0; r < n; ++r) {
            const NtKernelParams &p = sh[r].params, &q = sh[(r + 1) % n].params;
            const int owned = p.stored_rows[g] - 2 * halo;
            total += owned;
            const int next_lo = (p.row_origin[g] + halo + owned) % h, q_lo = (q.row_origin[g] + halo) % h;
            DIST_REQUIRE(next_lo == q_lo, "grid %d: shard %d's band does not start where shard %d's ends", g, (r + 1) % n, r);
        }
        DIST_REQUIRE(total == h, "grid %d: the bands cover %lld of its %d rows", g, (long long)total, h);
    }
    return NT_OK;
}

// Device-side checks: every buffer that another shard's kernels read or that this shard's
// kernels write is memory of the shard's device.
nt_status check_buffers(const NtShard &s, int r)
{
    nt_status st;
    const NtKernelParams &p = s.params;
    for (int g = 0; g < NT_NUM_FEATURES; ++g) {
        if ((st = check_on_device(p.features[g].grid, s.device, "latent grid", r)) != NT_OK) return st;
        if ((st = check_on_device(p.features[g].gradients, s.device, "latent gradients", r)) != NT_OK) return st;
        if ((st = check_on_device(p.features[g].moment1, s.device, "latent moment1", r)) != NT_OK) return st;
        if ((st = check_on_device(p.features[g].moment2, s.device, "latent moment2", r)) != NT_OK) return st;
    }
    for (int l = 0; l < NT_NUM_NETWORK_LAYERS; ++l) {
        if ((st = check_on_device(p.network_weights[l], s.device, "network weights", r)) != NT_OK) return st;
        if ((st = check_on_device(p.network_weight_gradients[l], s.device, "network weight gradients", r)) != NT_OK)
            return st;
        if ((st = check_on_device(p.network_weight_moment1[l], s.device, "network weight moment1", r)) != NT_OK) return st;
        if ((st = check_on_device(p.network_weight_moment2[l], s.device, "network weight moment2", r)) != NT_OK) return st;
        if ((st = check_on_device(p.network_biases[l], s.device, "network biases", r)) != NT_OK) return st;
        if ((st = check_on_device(p.network_bias_gradients[l], s.device, "network bias gradients", r)) != NT_OK)
            return st;
        if ((st = check_on_device(p.network_bias_moment1[l], s.device, "network bias moment1", r)) != NT_OK) return st;
        if ((st = check_on_device(p.network_bias_moment2[l], s.device, "network bias moment2", r)) != NT_OK) return st;
    }
    return NT_OK;
}

// Row `row` (stored index) of grid g of a shard, for latents (fp16) or gradients (fp32).
template <typename T>
T *row_ptr(void *base, const NtKernelParams &p, int g, int64_t row)
{
    return reinterpret_cast<T *>(base) + row * (int64_t)p.features[g].width * p.latent_channels;
}

nt_status cuda_fail(cudaError_t e, const char *what, int r)
{
    return set_error(NT_ERR_CUDA, "shard %d: %s: %s", r, what, cudaGetErrorString(e));
}

}  // namespace
}  // namespace nt

using namespace nt;

extern "C" {

nt_status nt_dist_band(int32_t rank, int32_t world, int32_t lattice_height, int32_t height, int32_t halo, int32_t *lo,
                       int32_t *hi)
{
    DIST_REQUIRE(lo && hi, "lo / hi are null");
    DIST_REQUIRE(world >= 1 && rank >= 0 && rank < world, "rank %d of %d", rank, world);
    DIST_REQUIRE(lattice_height >= world && height >= 1 && halo >= 0, "lattice height %d, height %d, halo %d",
                 lattice_height, height, halo);
    const int64_t a = (int64_t)rank * lattice_height / world, b = (int64_t)(rank + 1) * lattice_height / world;
    const auto rnd = [&](int64_t x) { return (2 * x * height + lattice_height) / (2 * (int64_t)lattice_height); };
    int64_t l = rnd(a), h = rnd(b);
    if (world == 1) {
        l = 0;
        h = height;
    } else {
        // nt_dist_train_step adds the neighbours' halo gradients to the first and the last
        // `halo` rows of a band in one launch, so a band holds at least two halos
        DIST_REQUIRE(h - l >= 2 * halo && h - l + 2 * halo <= height,
                     "rank %d: a band of %lld rows of a %d-row source cannot be sharded %d ways with a %d-row halo "
                     "(a band needs at least %d rows)", rank, (long long)(h - l), height, world, halo, 2 * halo);
    }
    *lo = (int32_t)l;
    *hi = (int32_t)h;
    return NT_OK;
}

nt_status nt_dist_train_step(const NtShard *shards, int32_t count)
{
    DIST_REQUIRE(shards, "shards is null");
    DIST_REQUIRE(count >= 1 && count <= NT_DIST_MAX_SHARDS, "count must be in [1, %d] (got %d)", NT_DIST_MAX_SHARDS,
                 count);
    DeviceRestore restore;
    if (count == 1) {
        cudaError_t e = cudaSetDevice(shards[0].device);
        if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice", 0);
        return nt_train_step(&shards[0].params, shards[0].stream);
    }
    nt_status st = validate_shards(shards, count);
    if (st != NT_OK) return st;
    for (int r = 0; r < count; ++r) {
        cudaError_t e = cudaSetDevice(shards[r].device);
        if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice", r);
        if ((st = check_buffers(shards[r], r)) != NT_OK) return st;
    }
    for (int r = 0; r < count; ++r)  // every shard reads every other shard's network gradients
        for (int q = 0; q < count; ++q)
            if ((st = ensure_peer(shards[r].device, shards[q].device)) != NT_OK) return st;

    std::vector<cudaEvent_t> trained(count), updated(count);
    for (int r = 0; r < count; ++r) {  // events are created on the current device
        cudaError_t e = cudaSetDevice(shards[r].device);
        if (e == cudaSuccess) e = g_events.get(2 * r, shards[r].device, &trained[r]);
        if (e == cudaSuccess) e = g_events.get(2 * r + 1, shards[r].device, &updated[r]);
        if (e != cudaSuccess) return cuda_fail(e, "event", r);
    }
    const auto stream_of = [&](int r) { return (cudaStream_t)shards[r].stream; };
    const auto wait_all = [&](int r, const std::vector<cudaEvent_t> &ev) -> cudaError_t {
        for (int q = 0; q < count; ++q) {
            if (q == r) continue;
            cudaError_t e = cudaStreamWaitEvent(stream_of(r), ev[q], 0);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    };

    // phase 1: training passes
    for (int r = 0; r < count; ++r) {
        cudaSetDevice(shards[r].device);
        if ((st = nt_invoke_training(&shards[r].params, NT_TRAIN_UNCONSTRAINED, shards[r].stream)) != NT_OK) return st;
        cudaError_t e = cudaEventRecord(trained[r], stream_of(r));
        if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord", r);
    }

    // phase 2: band edges += neighbours' halo gradients; network Adam on the shard-order sum; band Adam
    const NtKernelParams &p0 = shards[0].params;
    for (int r = 0; r < count; ++r) {
        const NtKernelParams &p = shards[r].params;
        const NtKernelParams &above = shards[(r + count - 1) % count].params, &below = shards[(r + 1) % count].params;
        DistReduceLaunch L;
        memset(&L, 0, sizeof L);
        int64_t max_n = 0;
        for (int g = 0; g < NT_NUM_FEATURES; ++g) {
            const int halo = shards[r].halo_rows[g], owned = p.stored_rows[g] - 2 * halo;
            const int64_t n = (int64_t)halo * p.features[g].width * p.latent_channels;
            // my last rows <- the halo above the band below; my first rows <- the halo below the band above
            L.add[L.nadd++] = {row_ptr<float>(p.features[g].gradients, p, g, owned),
                               row_ptr<float>(below.features[g].gradients, below, g, 0), n};
            L.add[L.nadd++] = {row_ptr<float>(p.features[g].gradients, p, g, halo),
                               row_ptr<float>(above.features[g].gradients, above, g, halo + (above.stored_rows[g] - 2 * halo)),
                               n};
            max_n = n > max_n ? n : max_n;
        }
        for (int l = 0; l < NT_NUM_NETWORK_LAYERS; ++l) {
            DistNetSeg &w = L.net[L.nnet++];
            w.w = reinterpret_cast<__half *>(p.network_weights[l]);
            w.m = p.network_weight_moment1[l];
            w.v = p.network_weight_moment2[l];
            w.n = kNetWeights[l];
            DistNetSeg &b = L.net[L.nnet++];
            b.w = reinterpret_cast<__half *>(p.network_biases[l]);
            b.m = p.network_bias_moment1[l];
            b.v = p.network_bias_moment2[l];
            b.n = net_biases(p, l);
            for (int q = 0; q < count; ++q) {
                w.g[q] = shards[q].params.network_weight_gradients[l];
                b.g[q] = shards[q].params.network_bias_gradients[l];
            }
            max_n = w.n > max_n ? w.n : max_n;
        }
        L.nshards = count;
        L.lr = p0.network_adam.learning_rate;
        L.beta1 = p0.network_adam.beta1;
        L.beta2 = p0.network_adam.beta2;
        L.eps = p0.network_adam.epsilon;
        const int t = p0.step > 0 ? p0.step : 1;  // train.cu:528
        L.bc1 = 1.0f - powf(L.beta1, (float)t);
        L.bc2 = 1.0f - powf(L.beta2, (float)t);

        cudaSetDevice(shards[r].device);
        cudaError_t e = wait_all(r, trained);
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent", r);
        dist_reduce_kernel<<<dim3(dist_blocks(max_n), L.nadd + L.nnet), kDistThreads, 0, stream_of(r)>>>(L);
        count_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "shard reduce kernel", r);

        NtKernelParams band = p;  // Adam over the owned rows only (the halo rows belong to the neighbours)
        for (int g = 0; g < NT_NUM_FEATURES; ++g) {
            NtFeature &f = band.features[g];
            const int halo = shards[r].halo_rows[g];
            f.grid = row_ptr<__half>(f.grid, p, g, halo);
            f.gradients = row_ptr<float>(f.gradients, p, g, halo);
            f.moment1 = row_ptr<float>(f.moment1, p, g, halo);
            f.moment2 = row_ptr<float>(f.moment2, p, g, halo);
            f.height = p.stored_rows[g] - 2 * halo;
            f.num_mips = 1;
        }
        if ((st = nt_invoke_optimize_features(&band, NT_TRAIN_UNCONSTRAINED, shards[r].stream)) != NT_OK) return st;
        if ((e = cudaEventRecord(updated[r], stream_of(r))) != cudaSuccess) return cuda_fail(e, "cudaEventRecord", r);
    }

    // phase 3: halo rows <- neighbours' updated band edges; halo and network gradients cleared
    for (int r = 0; r < count; ++r) {
        const NtKernelParams &p = shards[r].params;
        const NtKernelParams &above = shards[(r + count - 1) % count].params, &below = shards[(r + 1) % count].params;
        DistRefreshLaunch L;
        memset(&L, 0, sizeof L);
        int64_t max_n = 0;
        for (int g = 0; g < NT_NUM_FEATURES; ++g) {
            const int halo = shards[r].halo_rows[g], owned = p.stored_rows[g] - 2 * halo;
            const int above_owned = above.stored_rows[g] - 2 * halo;
            const int64_t n = (int64_t)halo * p.features[g].width * p.latent_channels;
            // my halo above <- the last rows of the band above; my halo below <- the first rows of the band below
            L.copy[L.ncopy++] = {row_ptr<__half>(p.features[g].grid, p, g, 0),
                                 row_ptr<__half>(above.features[g].grid, above, g, above_owned), n};
            L.copy[L.ncopy++] = {row_ptr<__half>(p.features[g].grid, p, g, halo + owned),
                                 row_ptr<__half>(below.features[g].grid, below, g, halo), n};
            L.zero[L.nzero++] = {row_ptr<float>(p.features[g].gradients, p, g, 0), n};
            L.zero[L.nzero++] = {row_ptr<float>(p.features[g].gradients, p, g, halo + owned), n};
            max_n = n > max_n ? n : max_n;
        }
        for (int l = 0; l < NT_NUM_NETWORK_LAYERS; ++l) {
            L.zero[L.nzero++] = {p.network_weight_gradients[l], kNetWeights[l]};
            L.zero[L.nzero++] = {p.network_bias_gradients[l], net_biases(p, l)};
        }
        cudaSetDevice(shards[r].device);
        cudaError_t e = wait_all(r, updated);
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent", r);
        dist_refresh_kernel<<<dim3(dist_blocks(max_n), L.ncopy + L.nzero), kDistThreads, 0, stream_of(r)>>>(L);
        count_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "shard refresh kernel", r);
    }
    return NT_OK;
}

}  // extern "C"

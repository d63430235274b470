// nt_nccl.cu -- row-sharded training with one process (or host thread) per GPU, the exchanges
// over NCCL (include/nt_capi.h: nt_nccl_*).
//
// Same band plan and the same result as nt_dist_train_step (nt_dist.cu), where one host thread
// drives every shard and the exchanges are kernels reading the neighbours' memory; and as the
// torch.distributed path of neural_textures_b200/sharded.py (train_step), which this restates
// without Python: halo gradients to their owners and a sum of the network gradients over the
// ranks, Adam on the band and the network, the band edges back into the neighbours' halo rows.
// The reference has no multi-device code (it trains one material on one device,
// main.cpp:1071-1077); the per-rank training pass and Adam are its InvokeTraining and
// InvokeOptimizeNetwork / InvokeOptimizeFeatures (train.h:158-160) on the band.
//
// NCCL is loaded at the first call (dlopen of libnccl.so.2; a process that already loaded it,
// e.g. through torch, gets that copy), so the library itself does not depend on it.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdio>
#include <type_traits>
#include <cstring>
#include <mutex>
#include <thread>

#include "nt_capi.h"
#include "nt_kernels.cuh"

namespace nt {

nt_status set_error(nt_status st, const char *fmt, ...);

namespace {

// ---- NCCL entry points ---------------------------------------------------------------------

struct NcclApi {
    bool ok = false;
    char why[256] = {0};
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    const char *(*GetErrorString)(ncclResult_t);
};

const NcclApi &nccl()
{
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            snprintf(api.why, sizeof api.why, "libnccl.so.2 could not be loaded (%s)", dlerror());
            return;
        }
        bool all = true;
        auto sym = [&](auto &fn, const char *name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            if (!fn) {
                all = false;
                snprintf(api.why, sizeof api.why, "libnccl.so.2 has no %s", name);
            }
        };
        sym(api.GetUniqueId, "ncclGetUniqueId");
        sym(api.CommInitRank, "ncclCommInitRank");
        sym(api.CommDestroy, "ncclCommDestroy");
        sym(api.CommAbort, "ncclCommAbort");
        sym(api.CommGetAsyncError, "ncclCommGetAsyncError");
        sym(api.GroupStart, "ncclGroupStart");
        sym(api.GroupEnd, "ncclGroupEnd");
        sym(api.Send, "ncclSend");
        sym(api.Recv, "ncclRecv");
        sym(api.AllReduce, "ncclAllReduce");
        sym(api.GetErrorString, "ncclGetErrorString");
        api.ok = all;
    });
    return api;
}

nt_status nccl_fail(ncclResult_t r, const char *what)
{
    return set_error(NT_ERR_NCCL, "%s: %s", what, nccl().GetErrorString ? nccl().GetErrorString(r) : "NCCL error");
}

#define NCCL_TRY(call, what)                          \
    do {                                              \
        const ncclResult_t r_ = (call);               \
        if (r_ != ncclSuccess) return nccl_fail(r_, what); \
    } while (0)

#define NCCL_REQUIRE(cond, ...)                                          \
    do {                                                                 \
        if (!(cond)) return set_error(NT_ERR_INVALID_ARG, __VA_ARGS__); \
    } while (0)

// ---- band geometry -------------------------------------------------------------------------

struct GridBand {
    int64_t row_elems;  // elements (width x channels) of one row
    int halo, owned, stored;
};

GridBand band_of(const NtShard &sh, int g)
{
    const NtKernelParams &p = sh.params;
    GridBand b;
    b.row_elems = (int64_t)p.features[g].width * p.latent_channels;
    b.halo = sh.halo_rows[g];
    b.stored = p.stored_rows[g] ? p.stored_rows[g] : p.features[g].height;
    b.owned = b.stored - 2 * b.halo;
    return b;
}

size_t workspace_bytes(const NtShard &sh)
{
    size_t n = 0;
    for (int g = 0; g < NT_NUM_FEATURES; ++g) {
        const GridBand b = band_of(sh, g);
        n += 2 * (size_t)b.halo * (size_t)b.row_elems * sizeof(float);  // received halo gradients, both edges
    }
    return (n + 15) / 16 * 16;
}

nt_status validate(const NtShard &sh, int world)
{
    const NtKernelParams &p = sh.params;
    NCCL_REQUIRE(p.latent_format == NT_LATENT_GRID_F16, "sharded training needs fp16 latent grids");
    NCCL_REQUIRE(p.latent_channels == 8 || p.latent_channels == 12, "latent_channels must be 8 or 12");
    for (int g = 0; g < NT_NUM_FEATURES; ++g) {
        const NtFeature &f = p.features[g];
        NCCL_REQUIRE(f.grid && f.gradients && f.moment1 && f.moment2, "grid %d: buffers are required", g);
        NCCL_REQUIRE(f.num_mips <= 1, "grid %d: sharded grids hold one level", g);
        const GridBand b = band_of(sh, g);
        if (world == 1) {
            NCCL_REQUIRE(b.halo == 0, "grid %d: one rank has no halo rows", g);
            continue;
        }
        NCCL_REQUIRE(b.halo >= 1 && p.stored_rows[g] > 0 && b.stored <= f.height,
                     "grid %d: %d stored rows with %d-row halos do not fit a %d-row grid", g, b.stored, b.halo,
                     f.height);
        NCCL_REQUIRE(b.owned >= 2 * b.halo,
                     "grid %d: band of %d rows is thinner than two %d-row halos (the edge additions would overlap)",
                     g, b.owned, b.halo);
    }
    return NT_OK;
}

// ---- kernels: halo gradients into the band edges ---------------------------------------------

struct AddSeg {
    float *dst;
    const float *src;
    int64_t n;  // floats, multiple of 4
};

struct AddLaunch {
    AddSeg seg[2 * NT_NUM_FEATURES];
    int32_t nseg;
};

__global__ void halo_add_kernel(const AddLaunch L)
{
    for (int s = 0; s < L.nseg; ++s) {
        const AddSeg a = L.seg[s];
        float4 *d = reinterpret_cast<float4 *>(a.dst);
        const float4 *x = reinterpret_cast<const float4 *>(a.src);
        const int64_t n4 = a.n / 4;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
            float4 v = d[i];
            const float4 w = x[i];
            v.x += w.x;
            v.y += w.y;
            v.z += w.z;
            v.w += w.w;
            d[i] = v;
        }
    }
}

}  // namespace
}  // namespace nt

using namespace nt;

struct NtNcclComm {
    ncclComm_t comm = nullptr;
    int world = 0, rank = 0, device = -1;
    cudaEvent_t done = nullptr;
    bool queued = false;
};

extern "C" {

nt_status nt_nccl_unique_id(void *id)
{
    NCCL_REQUIRE(id, "id is null");
    const NcclApi &api = nccl();
    if (!api.ok) return set_error(NT_ERR_NCCL, "%s", api.why);
    ncclUniqueId u;
    NCCL_TRY(api.GetUniqueId(&u), "ncclGetUniqueId");
    static_assert(sizeof(ncclUniqueId) == NT_NCCL_UNIQUE_ID_BYTES, "ncclUniqueId size");
    memcpy(id, &u, sizeof u);
    return NT_OK;
}

nt_status nt_nccl_comm_create(const void *id, int32_t world, int32_t rank, int32_t device, NtNcclComm **comm)
{
    NCCL_REQUIRE(comm, "comm is null");
    *comm = nullptr;
    NCCL_REQUIRE(id, "id is null");
    NCCL_REQUIRE(world >= 1 && rank >= 0 && rank < world, "rank %d of %d", rank, world);
    NCCL_REQUIRE(device >= 0, "device %d", device);
    const NcclApi &api = nccl();
    if (!api.ok) return set_error(NT_ERR_NCCL, "%s", api.why);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return set_error(NT_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
    NtNcclComm *c = new NtNcclComm;
    c->world = world;
    c->rank = rank;
    c->device = device;
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    const ncclResult_t r = api.CommInitRank(&c->comm, world, u, rank);
    if (r == ncclSuccess) e = cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming);
    cudaSetDevice(prev);
    if (r != ncclSuccess) {
        delete c;
        return nccl_fail(r, "ncclCommInitRank");
    }
    if (e != cudaSuccess) {
        api.CommDestroy(c->comm);
        delete c;
        return set_error(NT_ERR_CUDA, "cudaEventCreate: %s", cudaGetErrorString(e));
    }
    *comm = c;
    return NT_OK;
}

nt_status nt_nccl_comm_destroy(NtNcclComm *comm)
{
    if (!comm) return NT_OK;
    const NcclApi &api = nccl();
    nt_status st = NT_OK;
    if (comm->comm && api.ok) {
        const ncclResult_t r = api.CommDestroy(comm->comm);
        if (r != ncclSuccess) st = nccl_fail(r, "ncclCommDestroy");
    }
    if (comm->done) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(comm->device);
        cudaEventDestroy(comm->done);
        cudaSetDevice(prev);
    }
    delete comm;
    return st;
}

size_t nt_nccl_workspace_bytes(const NtShard *shard)
{
    return shard ? workspace_bytes(*shard) : 0;
}

nt_status nt_nccl_train_step(NtNcclComm *comm, const NtShard *shard, void *workspace, size_t workspace_bytes_)
{
    NCCL_REQUIRE(comm && comm->comm, "comm is null");
    NCCL_REQUIRE(shard, "shard is null");
    NCCL_REQUIRE(shard->device == comm->device, "the shard's device %d is not the communicator's device %d",
                 shard->device, comm->device);
    nt_status st = validate(*shard, comm->world);
    if (st != NT_OK) return st;
    const size_t need = workspace_bytes(*shard);
    NCCL_REQUIRE(comm->world == 1 || (workspace && workspace_bytes_ >= need && ((uintptr_t)workspace & 15) == 0),
                 "the workspace must hold %zu bytes, 16-byte aligned (got %zu)", need, workspace_bytes_);
    const NcclApi &api = nccl();
    const NtKernelParams &p = shard->params;
    cudaStream_t s = (cudaStream_t)shard->stream;
    int prev = 0;
    cudaGetDevice(&prev);
    struct Restore {
        int dev;
        ~Restore() { cudaSetDevice(dev); }
    } restore{prev};
    cudaError_t e = cudaSetDevice(comm->device);
    if (e != cudaSuccess) return set_error(NT_ERR_CUDA, "cudaSetDevice(%d): %s", comm->device, cudaGetErrorString(e));

    // 1. the training pass of the band (InvokeTraining, train.h:160)
    if ((st = nt_invoke_training(&p, NT_TRAIN_UNCONSTRAINED, shard->stream)) != NT_OK) return st;
    if (comm->world == 1) {
        if ((st = nt_invoke_optimize_all(&p, shard->stream)) != NT_OK) return st;
        if ((e = cudaEventRecord(comm->done, s)) != cudaSuccess)
            return set_error(NT_ERR_CUDA, "cudaEventRecord: %s", cudaGetErrorString(e));
        comm->queued = true;
        return NT_OK;
    }
    const int up = (comm->rank - 1 + comm->world) % comm->world, dn = (comm->rank + 1) % comm->world;
    GridBand b[NT_NUM_FEATURES];
    float *ws_last[NT_NUM_FEATURES], *ws_first[NT_NUM_FEATURES];
    {
        float *w = static_cast<float *>(workspace);
        for (int g = 0; g < NT_NUM_FEATURES; ++g) {
            b[g] = band_of(*shard, g);
            const int64_t n = (int64_t)b[g].halo * b[g].row_elems;
            ws_last[g] = w;
            ws_first[g] = w + n;
            w += 2 * n;
        }
    }
    // 2. halo gradients to their owners; network gradients summed over the ranks.  Every rank
    // posts its operations in the same order, so that with two ranks (both neighbours are the
    // same peer) the k-th send to the peer meets the peer's k-th receive from this rank.
    NCCL_TRY(api.GroupStart(), "ncclGroupStart");
    for (int g = 0; g < NT_NUM_FEATURES; ++g) {
        float *grad = p.features[g].gradients;
        const size_t n = (size_t)b[g].halo * (size_t)b[g].row_elems;
        float *halo_above = grad, *halo_below = grad + (int64_t)(b[g].halo + b[g].owned) * b[g].row_elems;
        NCCL_TRY(api.Send(halo_above, n, ncclFloat32, up, comm->comm, s), "ncclSend");
        NCCL_TRY(api.Send(halo_below, n, ncclFloat32, dn, comm->comm, s), "ncclSend");
        NCCL_TRY(api.Recv(ws_last[g], n, ncclFloat32, dn, comm->comm, s), "ncclRecv");
        NCCL_TRY(api.Recv(ws_first[g], n, ncclFloat32, up, comm->comm, s), "ncclRecv");
    }
    NCCL_TRY(api.GroupEnd(), "ncclGroupEnd");
    static const int64_t kWeights[NT_NUM_NETWORK_LAYERS] = {64 * 32, 64 * 64, 16 * 64};
    NCCL_TRY(api.GroupStart(), "ncclGroupStart");
    for (int l = 0; l < NT_NUM_NETWORK_LAYERS; ++l) {
        const size_t nb = l < 2 ? 64 : (size_t)p.output_channels;
        NCCL_TRY(api.AllReduce(p.network_weight_gradients[l], p.network_weight_gradients[l], (size_t)kWeights[l],
                               ncclFloat32, ncclSum, comm->comm, s),
                 "ncclAllReduce");
        NCCL_TRY(api.AllReduce(p.network_bias_gradients[l], p.network_bias_gradients[l], nb, ncclFloat32, ncclSum,
                               comm->comm, s),
                 "ncclAllReduce");
    }
    NCCL_TRY(api.GroupEnd(), "ncclGroupEnd");

    // 3. received halo gradients into the band edges, halo gradients cleared, then Adam on the
    // network and the owned band (InvokeOptimizeNetwork / InvokeOptimizeFeatures, train.h:158-159)
    AddLaunch L;
    memset(&L, 0, sizeof L);
    for (int g = 0; g < NT_NUM_FEATURES; ++g) {
        float *grad = p.features[g].gradients;
        const int64_t n = (int64_t)b[g].halo * b[g].row_elems;
        L.seg[L.nseg++] = AddSeg{grad + (int64_t)b[g].owned * b[g].row_elems, ws_last[g], n};  // band's last rows
        L.seg[L.nseg++] = AddSeg{grad + (int64_t)b[g].halo * b[g].row_elems, ws_first[g], n};  // band's first rows
    }
    halo_add_kernel<<<2 * sm_count(), 256, 0, s>>>(L);
    count_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return set_error(NT_ERR_CUDA, "halo add: %s", cudaGetErrorString(e));
    for (int g = 0; g < NT_NUM_FEATURES; ++g) {
        float *grad = p.features[g].gradients;
        const size_t bytes = (size_t)b[g].halo * (size_t)b[g].row_elems * sizeof(float);
        e = cudaMemsetAsync(grad, 0, bytes, s);
        if (e == cudaSuccess)
            e = cudaMemsetAsync(grad + (int64_t)(b[g].halo + b[g].owned) * b[g].row_elems, 0, bytes, s);
        if (e != cudaSuccess) return set_error(NT_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    }
    NtKernelParams a = p;
    for (int g = 0; g < NT_NUM_FEATURES; ++g) {
        NtFeature &f = a.features[g];
        const int64_t off = (int64_t)b[g].halo * b[g].row_elems;
        f.grid = static_cast<__half *>(f.grid) + off;
        f.gradients += off;
        f.moment1 += off;
        f.moment2 += off;
        f.height = b[g].owned;
        a.row_origin[g] = 0;
        a.stored_rows[g] = 0;
    }
    if ((st = nt_invoke_optimize_all(&a, shard->stream)) != NT_OK) return st;

    // 4. the band's updated first / last rows into the neighbours' halo rows
    NCCL_TRY(api.GroupStart(), "ncclGroupStart");
    for (int g = 0; g < NT_NUM_FEATURES; ++g) {
        __half *lat = static_cast<__half *>(p.features[g].grid);
        const size_t n = (size_t)b[g].halo * (size_t)b[g].row_elems;
        __half *first = lat + (int64_t)b[g].halo * b[g].row_elems, *last = lat + (int64_t)b[g].owned * b[g].row_elems;
        __half *halo_above = lat, *halo_below = lat + (int64_t)(b[g].halo + b[g].owned) * b[g].row_elems;
        NCCL_TRY(api.Send(first, n, ncclFloat16, up, comm->comm, s), "ncclSend");
        NCCL_TRY(api.Send(last, n, ncclFloat16, dn, comm->comm, s), "ncclSend");
        NCCL_TRY(api.Recv(halo_below, n, ncclFloat16, dn, comm->comm, s), "ncclRecv");
        NCCL_TRY(api.Recv(halo_above, n, ncclFloat16, up, comm->comm, s), "ncclRecv");
    }
    NCCL_TRY(api.GroupEnd(), "ncclGroupEnd");
    if ((e = cudaEventRecord(comm->done, s)) != cudaSuccess)
        return set_error(NT_ERR_CUDA, "cudaEventRecord: %s", cudaGetErrorString(e));
    comm->queued = true;
    return NT_OK;
}

nt_status nt_nccl_comm_wait(NtNcclComm *comm, int32_t timeout_ms)
{
    NCCL_REQUIRE(comm && comm->comm, "comm is null");
    NCCL_REQUIRE(timeout_ms >= 0, "timeout_ms must not be negative");
    if (!comm->queued) return NT_OK;
    const NcclApi &api = nccl();
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaEventQuery(comm->done);
        if (q == cudaSuccess) {
            comm->queued = false;
            return NT_OK;
        }
        if (q != cudaErrorNotReady) return set_error(NT_ERR_CUDA, "cudaEventQuery: %s", cudaGetErrorString(q));
        ncclResult_t ar = ncclSuccess;
        const ncclResult_t r = api.CommGetAsyncError(comm->comm, &ar);
        if (r != ncclSuccess || (ar != ncclSuccess && ar != ncclInProgress)) {
            api.CommAbort(comm->comm);
            comm->comm = nullptr;
            return nccl_fail(r != ncclSuccess ? r : ar, "NCCL asynchronous error (communicator aborted)");
        }
        const double ms =
            std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        if (ms > timeout_ms) {
            api.CommAbort(comm->comm);
            comm->comm = nullptr;
            return set_error(NT_ERR_TIMEOUT, "the step did not complete within %d ms (communicator aborted)",
                             timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

}  // extern "C"

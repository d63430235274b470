// nt_static_scratch.cu -- nt_invoke_training_static_scratch: the training pass with its tile
// counters in a fixed array of device memory that belongs to the library, for callers that
// cannot allocate device memory when they train.
//
// nt_invoke_training hands out tiles through counters in NtKernelParams.workspace, which the
// caller allocates.  Some callers cannot: a renderer or engine that reserves all of its device
// memory at start-up and may not allocate or free afterwards (cudaMalloc / cudaFree can stall
// the whole device and break its memory budget), or a host that reaches the library through a
// binding that passes parameter blocks only and has no device allocator of its own.  For them
// this entry point takes the counters from g_static_scratch below, a file-scope device array of
// kStaticScratchBytes; it calls no cudaMalloc, cudaFree or other allocating routine.
//
// Set-up: the first call on a device, with that device current, looks up the array's address
// once (cudaGetSymbolAddress) and keeps it; that first call should come before any stream
// capture starts.  Every call on a device shares the one array, which keeps what the last call
// left there, so each call first zeroes the counters on its own stream.  Calls whose work
// overlaps on the GPU (two streams, or two host threads) race on the counters: order them on
// one stream, or give each its own workspace through nt_invoke_training.
#include <atomic>
#include <cstring>

#include "nt_kernels.cuh"

namespace nt {

nt_status set_error(nt_status st, const char *fmt, ...);

// Largest scratch a call may need: one pair of 32-bit tile counters, padded to 256 bytes.
constexpr size_t kStaticScratchBytes = 256;
static_assert(kWorkspaceBytes <= kStaticScratchBytes, "the tile counters must fit the static scratch");

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;

// The array's device address per device (looked up once; a race between host threads only
// repeats the same lookup).
static void *scratch_of(int dev, cudaError_t *err)
{
    static std::atomic<void *> ptrs[kMaxDevices];
    void *ptr = ptrs[dev].load(std::memory_order_acquire);
    if (!ptr) {
        *err = cudaGetSymbolAddress(&ptr, g_static_scratch);
        if (*err != cudaSuccess) return nullptr;
        ptrs[dev].store(ptr, std::memory_order_release);
    }
    return ptr;
}

}  // namespace nt

using namespace nt;

nt_status nt_invoke_training_static_scratch(const NtKernelParams *params, NtTrainingKernelType type,
                                            nt_stream_t stream)
{
    if (!params) return set_error(NT_ERR_INVALID_ARG, "params must not be null");
    if (params->workspace)
        return set_error(NT_ERR_INVALID_ARG,
                         "workspace must be NULL: nt_invoke_training_static_scratch uses the library's "
                         "static scratch (pass a workspace to nt_invoke_training instead)");
    const size_t need = nt_workspace_bytes();
    if (need > kStaticScratchBytes)
        return set_error(NT_ERR_INVALID_ARG,
                         "the training pass needs %zu bytes of scratch, beyond the static scratch's %zu bytes",
                         need, kStaticScratchBytes);
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(NT_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices)
        return set_error(NT_ERR_INVALID_ARG, "device %d is beyond the %d devices the static scratch serves", dev,
                         kMaxDevices);
    e = cudaSuccess;
    void *scratch = scratch_of(dev, &e);
    if (!scratch)
        return set_error(NT_ERR_CUDA, "cudaGetSymbolAddress(static scratch) on device %d: %s", dev,
                         cudaGetErrorString(e));
    // the counters must start at zero; the previous call (on this or another stream) may have
    // left them otherwise if it failed part-way
    e = cudaMemsetAsync(scratch, 0, need, (cudaStream_t)stream);
    if (e != cudaSuccess) return set_error(NT_ERR_CUDA, "clearing the static scratch: %s", cudaGetErrorString(e));
    NtKernelParams p;
    std::memcpy(&p, params, sizeof p);
    p.workspace = scratch;
    p.workspace_bytes = (int64_t)kStaticScratchBytes;
    return nt_invoke_training(&p, type, stream);
}

// nt_reftex.cu -- reference textures: upload of an fp32 mip chain into a mipmapped CUDA array
// with the reference's texture descriptor (mavenkim2/neural_textures main.cpp:558-637), and a
// sampling kernel over arbitrary coordinates.
#include <algorithm>

#include "nt_capi.h"
#include "nt_kernels.cuh"
#include "nt_reftex.cuh"

namespace nt {

cudaError_t ref_texture_create(const float *chain, int w, int h, int ch, int mips, NtReferenceTexture *out)
{
    const int cc = ch == 3 ? 4 : ch;  // main.cpp:216-224: RGB is stored as RGBA
    const int n = mips > 1 ? mips : 1;
    const cudaChannelFormatDesc desc =
        cudaCreateChannelDesc(32, cc >= 2 ? 32 : 0, cc >= 3 ? 32 : 0, cc >= 4 ? 32 : 0, cudaChannelFormatKindFloat);
    cudaMipmappedArray_t arr = nullptr;
    cudaError_t e = cudaMallocMipmappedArray(&arr, &desc, make_cudaExtent((size_t)w, (size_t)h, 0), (unsigned)n);
    if (e != cudaSuccess) return e;
    size_t off = 0;
    for (int m = 0; m < n && e == cudaSuccess; ++m) {  // one 2D copy per level
        cudaArray_t level = nullptr;
        e = cudaGetMipmappedArrayLevel(&level, arr, (unsigned)m);
        if (e != cudaSuccess) break;
        const int lw = std::max(w >> m, 1), lh = std::max(h >> m, 1);
        const size_t pitch = (size_t)lw * cc * sizeof(float);
        e = cudaMemcpy2DToArray(level, 0, 0, chain + off, pitch, pitch, (size_t)lh, cudaMemcpyDefault);
        off += (size_t)lw * lh * cc;
    }
    cudaTextureObject_t tex = 0;
    if (e == cudaSuccess) {
        cudaResourceDesc rd = {};
        rd.resType = cudaResourceTypeMipmappedArray;
        rd.res.mipmap.mipmap = arr;
        cudaTextureDesc td = {};  // main.cpp:609-619
        td.addressMode[0] = td.addressMode[1] = cudaAddressModeWrap;
        td.filterMode = cudaFilterModeLinear;
        td.mipmapFilterMode = cudaFilterModeLinear;
        td.readMode = cudaReadModeElementType;
        td.normalizedCoords = 1;
        td.minMipmapLevelClamp = 0.f;
        td.maxMipmapLevelClamp = (float)(n - 1);
        e = cudaCreateTextureObject(&tex, &rd, &td, nullptr);
    }
    if (e != cudaSuccess) {
        cudaFreeMipmappedArray(arr);
        return e;
    }
    out->texture = (uint64_t)tex;
    out->storage = reinterpret_cast<uint64_t>(arr);
    out->width = w;
    out->height = h;
    out->num_channels = ch;
    out->num_mips = n;
    return cudaSuccess;
}

cudaError_t ref_texture_destroy(NtReferenceTexture *t)
{
    cudaError_t e = cudaSuccess;
    if (t->texture) e = cudaDestroyTextureObject((cudaTextureObject_t)t->texture);
    if (t->storage) {
        const cudaError_t e2 = cudaFreeMipmappedArray(reinterpret_cast<cudaMipmappedArray_t>(t->storage));
        if (e == cudaSuccess) e = e2;
    }
    t->texture = 0;
    t->storage = 0;
    return e;
}

RefTexView ref_view(const NtReferenceTexture &t)
{
    RefTexView v;
    v.tex = (cudaTextureObject_t)t.texture;
    v.w = t.width;
    v.h = t.height;
    v.ch = t.num_channels;
    v.mips = t.num_mips > 1 ? t.num_mips : 1;
    return v;
}

__global__ void ref_sample_kernel(const RefTexView r, const float2 *__restrict__ uv, int64_t n, float lod,
                                  float4 *__restrict__ out)
{
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float2 c = uv[i];
        out[i] = ref_trilinear(r, c.x, c.y, lod);
    }
}

cudaError_t launch_ref_sample(const NtReferenceTexture &t, const float *uv, int64_t n, float lod, float *out,
                              cudaStream_t st)
{
    const int blocks = (int)std::min<int64_t>((n + 255) / 256, 8 * sm_count());
    ref_sample_kernel<<<blocks, 256, 0, st>>>(ref_view(t), reinterpret_cast<const float2 *>(uv), n, lod,
                                              reinterpret_cast<float4 *>(out));
    count_launch();
    return cudaGetLastError();
}

}  // namespace nt

// fp16 <-> fp32 conversion passes of ptqkit's compressed format.
//
// ptqkit stores scales, zeros and the AWQ channel scale of every quantized
// layer in fp16 on disk (src/ptqkit/convert.py:296-336, `.to(torch.float16)`)
// while its kernels read fp32 [rows, groups] arrays. The loader uploads the
// fp16 payload of all layers as one contiguous block and widens it in one
// launch into the fp32 arrays the dequant-GEMM reads; the save path narrows
// each fp32 array on the device before it leaves the GPU.
//
// Both passes are HBM streams (6 bytes per value). Widening is exact. Narrowing
// rounds to nearest even with overflow to infinity and keeps signed zeros and
// fp16 subnormals, the IEEE conversion torch applies on the CPU.

#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"

namespace wq {
namespace {

constexpr int kConvThreads = 256;

// Eight values per thread per step: one 16-byte fp16 load and two 16-byte
// fp32 stores (or the reverse), in a grid-stride loop over the vector body.
__global__ void __launch_bounds__(kConvThreads) widen_kernel(const __half* __restrict__ src,
                                                             float* __restrict__ dst, int64_t n) {
    const int64_t nvec = n / 8;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (int64_t v = tid; v < nvec; v += stride) {
        const uint4 raw = __ldcs(reinterpret_cast<const uint4*>(src) + v);
        const __half2* h = reinterpret_cast<const __half2*>(&raw);
        const float2 a = __half22float2(h[0]);
        const float2 b = __half22float2(h[1]);
        const float2 c = __half22float2(h[2]);
        const float2 d = __half22float2(h[3]);
        float4* out = reinterpret_cast<float4*>(dst) + 2 * v;
        __stcs(out, make_float4(a.x, a.y, b.x, b.y));
        __stcs(out + 1, make_float4(c.x, c.y, d.x, d.y));
    }
    for (int64_t i = nvec * 8 + tid; i < n; i += stride) dst[i] = __half2float(src[i]);
}

__global__ void __launch_bounds__(kConvThreads) narrow_kernel(const float* __restrict__ src,
                                                              __half* __restrict__ dst, int64_t n) {
    const int64_t nvec = n / 8;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (int64_t v = tid; v < nvec; v += stride) {
        const float4* in = reinterpret_cast<const float4*>(src) + 2 * v;
        const float4 a = __ldcs(in);
        const float4 b = __ldcs(in + 1);
        uint4 raw;
        __half2* h = reinterpret_cast<__half2*>(&raw);
        h[0] = __floats2half2_rn(a.x, a.y);
        h[1] = __floats2half2_rn(a.z, a.w);
        h[2] = __floats2half2_rn(b.x, b.y);
        h[3] = __floats2half2_rn(b.z, b.w);
        __stcs(reinterpret_cast<uint4*>(dst) + v, raw);
    }
    for (int64_t i = nvec * 8 + tid; i < n; i += stride) dst[i] = __float2half_rn(src[i]);
}

// Element-wise fallbacks for pointers that are not 16-byte aligned.
__global__ void __launch_bounds__(kConvThreads) widen_scalar_kernel(const __half* __restrict__ src,
                                                                    float* __restrict__ dst, int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = __half2float(src[i]);
}

__global__ void __launch_bounds__(kConvThreads) narrow_scalar_kernel(const float* __restrict__ src,
                                                                     __half* __restrict__ dst, int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = __float2half_rn(src[i]);
}

// Enough CTAs to cover every SM several times over, never more than the work.
int conv_grid(int64_t units) {
    const int64_t per_cta = kConvThreads;
    const int64_t want = (units + per_cta - 1) / per_cta;
    const int64_t cap = (int64_t)sm_count() * 8;
    return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

cudaError_t launch_widen_f16_f32(const uint16_t* src, float* dst, int64_t n, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    const __half* h = reinterpret_cast<const __half*>(src);
    if (aligned16(src) && aligned16(dst))
        widen_kernel<<<conv_grid(n / 8 > 0 ? n / 8 : n), kConvThreads, 0, s>>>(h, dst, n);
    else
        widen_scalar_kernel<<<conv_grid(n), kConvThreads, 0, s>>>(h, dst, n);
    return cudaGetLastError();
}

cudaError_t launch_narrow_f32_f16(const float* src, uint16_t* dst, int64_t n, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    __half* h = reinterpret_cast<__half*>(dst);
    if (aligned16(src) && aligned16(dst))
        narrow_kernel<<<conv_grid(n / 8 > 0 ? n / 8 : n), kConvThreads, 0, s>>>(src, h, n);
    else
        narrow_scalar_kernel<<<conv_grid(n), kConvThreads, 0, s>>>(src, h, n);
    return cudaGetLastError();
}

}  // namespace wq

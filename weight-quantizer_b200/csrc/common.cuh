// Shared device helpers for the wq_b200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "wq_b200 kernels are written for sm_100a (B200) only"
#endif

namespace wq {

constexpr int kWarp = 32;

// 16-byte streaming load that bypasses L1 allocation: the packed weight stream
// is read exactly once per launch, so it should not evict the staged
// activations from L1/shared memory.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float ld_ro(const float* p) { return __ldg(p); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Exact power of two 2^e for e in [-126, 127] built from its bit pattern.
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

}  // namespace wq

// wq_dequant_gemm_f32_noalloc: the dequant-GEMM for callers that cannot
// allocate device memory.
//
// Who needs it: code that must not call cudaMalloc (or a caching allocator
// such as torch's) at the point where it runs the layer, for example an
// inference server that reserves every device byte at start-up and forbids
// allocation on its request path, or a host runtime whose only device memory
// is what its caller hands it. The regular entry point asks such callers for a
// workspace whenever the batch takes the tensor-core path (it holds x split
// into fp16 hi/lo planes); this one uses a fixed scratch array that lives in
// the library instead, so the caller passes only inputs and outputs.
//
// Costs and limits:
//   - The scratch is a static device array of kNoAllocScratchBytes (32 MiB).
//     Every GPU that loads this library holds it until the process exits.
//   - A problem whose workspace query exceeds it is rejected with
//     WQ_E_NOALLOC_LIMIT (the tensor-core path needs about 4 * B * K bytes, so
//     for K = 8192 up to 896 batch rows fit).
//   - All calls on a device share the one array. The tensor-core path writes
//     every scratch byte it reads before reading it, so nothing has to be
//     cleared between calls, but two calls whose work overlaps on the GPU
//     (different streams, no ordering between them) race on it.
//   - The first call on each device looks up the array's device address with
//     cudaGetSymbolAddress while that device is current; make that first call
//     before capturing a stream. The address is kept per device together with
//     the CUDA context it belongs to: after a cudaDeviceReset the device has a
//     new context, and the next call looks the address up again instead of
//     handing the kernels a pointer into the destroyed one.
#include <cuda.h>

#include <mutex>

#include "../../include/wq_b200.h"
#include "common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;

// Device-resident scratch for the calls of wq_dequant_gemm_f32_noalloc. In
// host code this name stands for the symbol, not a device address: only the
// address returned by cudaGetSymbolAddress may be handed to a kernel.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// The driver's cuCtxGetCurrent, reached through the runtime (no link-time
// dependency on libcuda); nullptr if unavailable.
CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
    });
    return fn;
}

// Device address of g_noalloc_scratch on the current device, looked up once
// per device and context (nullptr if the lookup failed).
void* scratch_address(cudaError_t* err) {
    static void* cached[64] = {nullptr};
    static CUcontext cached_ctx[64] = {nullptr};
    static std::mutex mu;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) {
        *err = e != cudaSuccess ? e : cudaErrorInvalidDevice;
        return nullptr;
    }
    CtxGetCurrentFn get = ctx_get_current();
    CUcontext ctx = nullptr;
    if (get != nullptr && get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (cached[dev] == nullptr || ctx == nullptr || cached_ctx[dev] != ctx) {
        // (the lookup makes the device's primary context current if none is;
        // the context is read again after it)
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess) {
            *err = e;
            return nullptr;
        }
        if (get != nullptr && get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
        cached[dev] = ptr;
        cached_ctx[dev] = ctx;
    }
    *err = cudaSuccess;
    return cached[dev];
}

}  // namespace

extern "C" {

int wq_dequant_gemm_f32_noalloc(const float* x, int64_t B, int64_t K,
                                const uint8_t* q, int64_t M, int64_t q_cols,
                                const float* scales, int64_t scale_rows, int64_t groups,
                                const float* zeros, int64_t zero_rows, int64_t zero_groups,
                                const float* channel_scale, int64_t channel_len,
                                int group_size, int bits,
                                float* y, int64_t ldy,
                                void* stream) {
    const size_t need = wq_dequant_gemm_workspace_bytes(B, M, K, group_size, bits);
    if (need > kNoAllocScratchBytes) return WQ_E_NOALLOC_LIMIT;
    cudaError_t err = cudaSuccess;
    void* scratch = scratch_address(&err);
    if (scratch == nullptr) {
        // the address lookup failed; clear the sticky-free error state so the
        // caller's next CUDA call is not blamed for it
        cudaGetLastError();
        return WQ_E_CUDA;
    }
    return wq_dequant_gemm_f32(x, B, K, q, M, q_cols, scales, scale_rows, groups, zeros, zero_rows, zero_groups,
                               channel_scale, channel_len, group_size, bits, y, ldy, scratch, kNoAllocScratchBytes,
                               stream);
}

}  // extern "C"

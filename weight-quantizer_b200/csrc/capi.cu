// C ABI entry points (include/wq_b200.h): argument validation in the order and
// with the messages of ptqkit's pybind11 entry point
// (src/ptqkit/csrc/dequant_gemm.cpp:222-300), then dispatch to the kernels.
// Nothing here allocates device memory or synchronizes the host.
#include <cuda.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/wq_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace wq {

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

// Fault word of this library on every device that loads it.
__device__ unsigned int g_wq_fault = 0;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

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

// Looked up once per device and CUDA context: a cudaDeviceReset gives the
// device a new context, and the address is then looked up again.
unsigned int* fault_word() {
    static unsigned int* cached[64] = {nullptr};
    static CUcontext cached_ctx[64] = {nullptr};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    CtxGetCurrentFn get = ctx_get_current();
    CUcontext ctx = nullptr;
    if (get != nullptr && get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (cached[dev] == nullptr || ctx == nullptr || cached_ctx[dev] != ctx) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_wq_fault) != cudaSuccess) return nullptr;
        if (get != nullptr && get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
        cached[dev] = static_cast<unsigned int*>(ptr);
        cached_ctx[dev] = ctx;
    }
    return cached[dev];
}

namespace {

// Waits on a shared-memory barrier that nothing arrives on, with the bounded
// poll loop of the pipeline kernels (here with a caller-chosen limit), and
// records the expiry in the fault word as they do.
__global__ void selftest_expired_wait_kernel(uint32_t max_polls, unsigned int* fault) {
    __shared__ __align__(8) unsigned long long bar_word;
    const uint32_t bar = smem_addr(&bar_word);
    mbar_init(bar, 1);
    fence_mbarrier_init();
    bool done = false;
    for (uint32_t n = 0; n < max_polls && !done; ++n) done = mbar_try_wait(bar, 0);
    if (!done) atomicOr(fault, 1u);
}

}  // namespace
}  // namespace wq

namespace {

thread_local char g_cuda_error[256] = "no error";

int cuda_fail(cudaError_t e) {
    std::snprintf(g_cuda_error, sizeof(g_cuda_error), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
    return WQ_E_CUDA;
}

constexpr int64_t kMaxDim = ((int64_t)1 << 31) - 1;

}  // namespace

extern "C" {

const char* wq_status_string(int status) {
    switch (status) {
        case WQ_OK: return "ok";
        case WQ_E_X_SHAPE: return "x must have shape [B, K]";
        case WQ_E_RANK: return "q, scales, and zeros must be rank 2";
        case WQ_E_BITS: return "bits must be 4 or 8";
        case WQ_E_GROUP_SIZE: return "group_size must be positive";
        case WQ_E_NEG_DIM: return "negative dimension";
        case WQ_E_PACKED_COLS: return "packed code row length does not match K";
        case WQ_E_ZEROS_SHAPE: return "zeros shape must match scales";
        case WQ_E_SCALE_ROWS: return "scale rows must be 1 or M";
        case WQ_E_SCALE_GROUPS: return "scale groups must equal ceil(K / group_size)";
        case WQ_E_CHANNEL_SHAPE: return "channel_scale must have shape [K]";
        case WQ_E_NULL: return "a required device pointer is null";
        case WQ_E_WORKSPACE: return "workspace is smaller than the size the workspace query returned";
        case WQ_E_TOO_LARGE: return "a dimension exceeds the range the kernels index";
        case WQ_E_CUDA: return "CUDA error (see wq_last_cuda_error)";
        case WQ_E_NOT_FINITE: return "weight must be finite";
        case WQ_E_PRE_SCALE_LEN: return "pre_scale must have one entry per input channel";
        case WQ_E_PRE_SCALE_VAL: return "pre_scale must be finite and positive";
        case WQ_E_INT4_RANGE: return "int4 codes must lie in [0, 15]";
        case WQ_E_GROUP_MODE: return "group_size must be None, 0, or positive";
        case WQ_E_LD: return "output row stride is smaller than the output row length";
        case WQ_E_NOALLOC_LIMIT:
            return "problem needs more scratch than the no-allocation entry point holds; use wq_dequant_gemm_f32";
        case WQ_E_OUTPUTS: return "output count must be between 1 and WQ_MAX_OUTPUTS";
        default: return "unknown status";
    }
}

const char* wq_last_cuda_error(void) { return g_cuda_error; }

int wq_kernel_info(int device, wq_kernel_info_t* out) {
    if (out == nullptr) return WQ_E_NULL;
    std::memset(out, 0, sizeof(*out));
    out->abi_version = WQ_ABI_VERSION;
    out->compiled_sm = 100;
    out->device = device;
    out->tcgen05 = 1;
    cudaDeviceProp prop;
    cudaError_t e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return cuda_fail(e);
    out->device_cc = prop.major * 10 + prop.minor;
    out->sm_count = prop.multiProcessorCount;
    std::snprintf(out->device_name, sizeof(out->device_name), "%.95s", prop.name);
    return WQ_OK;
}

int wq_fault_status(int reset, uint32_t* out) {
    if (out == nullptr) return WQ_E_NULL;
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, wq::g_wq_fault, sizeof(v));
    if (e != cudaSuccess) return cuda_fail(e);
    *out = v;
    if (reset && v != 0) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(wq::g_wq_fault, &zero, sizeof(zero));
        if (e != cudaSuccess) return cuda_fail(e);
    }
    return WQ_OK;
}

int wq_selftest_expired_wait(uint32_t max_polls, void* stream) {
    if (max_polls < 1 || max_polls > wq::kMaxPolls) return WQ_E_TOO_LARGE;
    unsigned int* fault = wq::fault_word();
    if (fault == nullptr) return cuda_fail(cudaErrorInvalidDevicePointer);
    wq::selftest_expired_wait_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(max_polls, fault);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

size_t wq_dequant_gemm_workspace_bytes(int64_t B, int64_t M, int64_t K, int group_size, int bits) {
    if (B <= 0 || K <= 0 || group_size <= 0 || (bits != 4 && bits != 8)) return 0;
    // the larger of the two paths a problem of this size can take (which one
    // runs also depends on the pointers' alignment)
    size_t need = 0;
    if (B <= wq::kGemvMaxBatch) {
        need = wq::gemv_workspace_bytes(B, K, bits);
    } else {
        const bool single_group = group_size >= K;
        if (single_group || group_size % 64 == 0) need = wq::tc_workspace_bytes(B, M, K, group_size, bits);
    }
    const size_t wide = wq::wide_workspace_bytes(B, M, K, group_size, bits);
    return wide > need ? wide : need;
}

}  // extern "C"

namespace {

// Validation in the reference's order, then dispatch; y_out[0] is the primary
// output, y_out[1..n_out) receive the same values.
int run_gemm(const float* x, int64_t B, int64_t K, const uint8_t* q, int64_t M, int64_t q_cols,
             const float* scales, int64_t scale_rows, int64_t groups, const float* zeros, int64_t zero_rows,
             int64_t zero_groups, const float* channel_scale, int64_t channel_len, int group_size, int bits,
             float* const* y_out, int n_out, int64_t ldy, float* y_all, const float* bias, void* workspace,
             size_t workspace_bytes, void* stream) {
    // dequant_gemm.cpp:241-276, same order
    if (bits != 4 && bits != 8) return WQ_E_BITS;
    if (group_size <= 0) return WQ_E_GROUP_SIZE;
    if (K < 0 || M < 0 || B < 0) return WQ_E_NEG_DIM;
    const int64_t packed_cols = bits == 4 ? (K + 1) / 2 : K;
    if (q_cols != packed_cols) return WQ_E_PACKED_COLS;
    if (zero_rows != scale_rows || zero_groups != groups) return WQ_E_ZEROS_SHAPE;
    if (scale_rows != 1 && scale_rows != M) return WQ_E_SCALE_ROWS;
    const int64_t n_groups = K == 0 ? 0 : (K + group_size - 1) / group_size;
    if (K > 0 && groups != n_groups) return WQ_E_SCALE_GROUPS;
    if (channel_scale != nullptr && channel_len != K) return WQ_E_CHANNEL_SHAPE;
    // beyond the reference: output count and stride, pointers, index range
    if (n_out < 1 || n_out > WQ_MAX_OUTPUTS) return WQ_E_OUTPUTS;
    if (ldy < M) return WQ_E_LD;
    if (B > kMaxDim || M > kMaxDim || K > kMaxDim || groups > kMaxDim) return WQ_E_TOO_LARGE;
    if (B == 0 || M == 0) return WQ_OK;
    if (y_out == nullptr) return WQ_E_NULL;
    for (int i = 0; i < n_out; ++i)
        if (y_out[i] == nullptr) return WQ_E_NULL;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (K == 0) {
        for (int i = 0; i < n_out; ++i) {
            cudaError_t e = bias != nullptr ? wq::launch_fill_bias(y_out[i], B, M, ldy, bias, s)
                                            : wq::launch_fill_zero(y_out[i], B, M, ldy, s);
            if (e != cudaSuccess) return cuda_fail(e);
        }
        return WQ_OK;
    }
    if (x == nullptr || q == nullptr || scales == nullptr || zeros == nullptr) return WQ_E_NULL;

    wq::GemmProblem p;
    p.x = x;
    p.q = q;
    p.scales = scales;
    p.zeros = zeros;
    p.channel = channel_scale;
    p.y = y_out[0];
    p.n_extra = 0;
    p.y_all = nullptr;
    p.bias = bias;
    for (int i = 0; i < 7; ++i) p.y_extra[i] = nullptr;
    p.B = B;
    p.M = M;
    p.K = K;
    p.q_stride = q_cols;
    p.ldy = ldy;
    p.scale_rows = (int)scale_rows;
    p.groups = (int)groups;
    p.group_size = group_size;
    p.bits = bits;

    cudaError_t e;
    bool copies = n_out > 1;   // paths without a multi-output epilogue copy afterwards
    // the decode and tensor-core kernels store into every output themselves
    auto fan_out = [&]() {
        if (y_all != nullptr) {
            p.y_all = y_all;
        } else {
            p.n_extra = n_out - 1;
            for (int i = 1; i < n_out; ++i) p.y_extra[i - 1] = y_out[i];
        }
        copies = false;
    };
    if (wq::wide_supported(p)) {
        const size_t need = wq::wide_workspace_bytes(B, M, K, group_size, bits);
        if (workspace_bytes < need || workspace == nullptr) return WQ_E_WORKSPACE;
        if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return WQ_E_WORKSPACE;
        fan_out();
        e = wq::launch_wide(p, workspace, s);
    } else if (wq::gemv_supported(p)) {
        const size_t need = wq::gemv_workspace_bytes(B, K, bits);
        if (workspace_bytes < need || (need > 0 && workspace == nullptr)) return WQ_E_WORKSPACE;
        fan_out();
        e = wq::launch_gemv(p, workspace, s);
    } else if (wq::tc_supported(p)) {
        const size_t need = wq::tc_workspace_bytes(B, M, K, group_size, bits);
        if (workspace_bytes < need || workspace == nullptr) return WQ_E_WORKSPACE;
        if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return WQ_E_WORKSPACE;
        fan_out();
        e = wq::launch_tc(p, workspace, s);
    } else {
        e = wq::launch_gemm_simt(p, s);
    }
    if (e != cudaSuccess) return cuda_fail(e);
    if (copies) {
        for (int i = 1; i < n_out; ++i) {
            e = cudaMemcpy2DAsync(y_out[i], (size_t)ldy * sizeof(float), y_out[0], (size_t)ldy * sizeof(float),
                                  (size_t)M * sizeof(float), (size_t)B, cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) return cuda_fail(e);
        }
    }
    return WQ_OK;
}

using MemGetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

MemGetAddressRangeFn address_range_fn() {
    static MemGetAddressRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<MemGetAddressRangeFn>(ptr);
    });
    return fn;
}

}  // namespace

extern "C" {

int wq_dequant_gemm_f32(const float* x, int64_t B, int64_t K,
                        const uint8_t* q, int64_t M, int64_t q_cols,
                        const float* scales, int64_t scale_rows, int64_t groups,
                        const float* zeros, int64_t zero_rows, int64_t zero_groups,
                        const float* channel_scale, int64_t channel_len,
                        int group_size, int bits,
                        float* y, int64_t ldy,
                        void* workspace, size_t workspace_bytes,
                        void* stream) {
    float* const outs[1] = {y};
    return run_gemm(x, B, K, q, M, q_cols, scales, scale_rows, groups, zeros, zero_rows, zero_groups, channel_scale,
                    channel_len, group_size, bits, y == nullptr ? nullptr : outs, 1, ldy, nullptr, nullptr, workspace,
                    workspace_bytes, stream);
}

int wq_dequant_gemm_f32_multi(const float* x, int64_t B, int64_t K,
                              const uint8_t* q, int64_t M, int64_t q_cols,
                              const float* scales, int64_t scale_rows, int64_t groups,
                              const float* zeros, int64_t zero_rows, int64_t zero_groups,
                              const float* channel_scale, int64_t channel_len,
                              int group_size, int bits,
                              float* const* y_out, int n_out, int64_t ldy, float* y_all, const float* bias,
                              void* workspace, size_t workspace_bytes,
                              void* stream) {
    return run_gemm(x, B, K, q, M, q_cols, scales, scale_rows, groups, zeros, zero_rows, zero_groups, channel_scale,
                    channel_len, group_size, bits, y_out, n_out, ldy, y_all, bias, workspace, workspace_bytes, stream);
}

size_t wq_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int wq_ipc_get_handle(const void* ptr, void* handle_out, int64_t* offset_out) {
    if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr) return WQ_E_NULL;
    MemGetAddressRangeFn range = address_range_fn();
    if (range == nullptr) return cuda_fail(cudaErrorNotSupported);
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return cuda_fail(cudaErrorInvalidValue);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) return cuda_fail(e);
    std::memcpy(handle_out, &h, sizeof(h));
    *offset_out = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return WQ_OK;
}

int wq_ipc_open_handle(const void* handle, int64_t offset, void** ptr_out) {
    if (handle == nullptr || ptr_out == nullptr) return WQ_E_NULL;
    if (offset < 0) return WQ_E_NEG_DIM;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e);
    *ptr_out = static_cast<unsigned char*>(base) + offset;
    return WQ_OK;
}

int wq_ipc_close_handle(void* ptr, int64_t offset) {
    if (ptr == nullptr) return WQ_E_NULL;
    cudaError_t e = cudaIpcCloseMemHandle(static_cast<unsigned char*>(ptr) - offset);
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

size_t wq_rtn_workspace_bytes(int64_t M, int64_t K, int group_mode) {
    return wq::rtn_workspace_bytes(M, K, group_mode);
}

int wq_rtn_flags_status(int32_t flags) {
    if (flags & 1) return WQ_E_NOT_FINITE;
    if (flags & 2) return WQ_E_PRE_SCALE_VAL;
    return WQ_OK;
}

int wq_rtn_quantize_f32(const float* w, const float* pre_scale, int64_t M, int64_t K,
                        int bits, int symmetric, int group_mode,
                        uint8_t* q_out, float* scales_out, float* zeros_out,
                        float* channel_out, int32_t* flags,
                        void* workspace, size_t workspace_bytes, void* stream) {
    if (bits != 4 && bits != 8) return WQ_E_BITS;
    if (group_mode < -1) return WQ_E_GROUP_MODE;
    if (M < 0 || K < 0) return WQ_E_NEG_DIM;
    if (M > kMaxDim || K > kMaxDim || M * K > ((int64_t)1 << 62)) return WQ_E_TOO_LARGE;
    if (K > 200 * 1024) return WQ_E_TOO_LARGE;
    if (flags == nullptr) return WQ_E_NULL;
    if (pre_scale != nullptr && channel_out == nullptr) return WQ_E_NULL;
    if (M > 0 && K > 0 && (w == nullptr || q_out == nullptr || scales_out == nullptr || zeros_out == nullptr))
        return WQ_E_NULL;
    const size_t need = wq::rtn_workspace_bytes(M, K, group_mode);
    if (workspace_bytes < need || (need > 0 && workspace == nullptr)) return WQ_E_WORKSPACE;
    wq::RtnProblem p;
    p.w = w;
    p.pre_scale = pre_scale;
    p.M = M;
    p.K = K;
    p.bits = bits;
    p.symmetric = symmetric ? 1 : 0;
    p.group_mode = group_mode;
    p.q_out = q_out;
    p.scales_out = scales_out;
    p.zeros_out = zeros_out;
    p.channel_out = channel_out;
    p.flags = flags;
    cudaError_t e = wq::launch_rtn(p, workspace, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

int wq_pack_int4(const int32_t* codes, int64_t M, int64_t K, uint8_t* packed, int32_t* minmax, void* stream) {
    if (M < 0 || K < 0) return WQ_E_NEG_DIM;
    if (minmax == nullptr) return WQ_E_NULL;
    if (M > 0 && K > 0 && (codes == nullptr || packed == nullptr)) return WQ_E_NULL;
    cudaError_t e = wq::launch_pack_int4(codes, M, K, packed, minmax, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

int wq_unpack_int4(const uint8_t* packed, int64_t M, int64_t packed_cols, int64_t K, uint8_t* codes,
                   void* stream) {
    if (M < 0 || K < 0) return WQ_E_NEG_DIM;
    if (packed_cols < (K + 1) / 2) return WQ_E_PACKED_COLS;
    if (M > 0 && K > 0 && (codes == nullptr || packed == nullptr)) return WQ_E_NULL;
    cudaError_t e = wq::launch_unpack_int4(packed, M, packed_cols, K, codes, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

int wq_dequantize_f32(const uint8_t* q, int64_t M, int64_t K, int64_t q_cols,
                      const float* scales, int64_t scale_rows, int64_t groups,
                      const float* zeros, const float* channel_scale,
                      int group_size, int bits, float* w_out, void* stream) {
    if (bits != 4 && bits != 8) return WQ_E_BITS;
    if (group_size <= 0) return WQ_E_GROUP_SIZE;
    if (K < 0 || M < 0) return WQ_E_NEG_DIM;
    const int64_t packed_cols = bits == 4 ? (K + 1) / 2 : K;
    if (q_cols < packed_cols) return WQ_E_PACKED_COLS;
    if (scale_rows != 1 && scale_rows != M) return WQ_E_SCALE_ROWS;
    if (K > 0 && groups != (K + group_size - 1) / group_size) return WQ_E_SCALE_GROUPS;
    if (M == 0 || K == 0) return WQ_OK;
    if (q == nullptr || scales == nullptr || zeros == nullptr || w_out == nullptr) return WQ_E_NULL;
    cudaError_t e = wq::launch_dequantize(q, M, K, q_cols, scales, (int)scale_rows, (int)groups, zeros,
                                          channel_scale, group_size, bits, w_out,
                                          static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

int wq_gather_permute_f32(const float* src, int64_t P, int64_t B, int64_t Mp, float* dst, void* stream) {
    if (P < 0 || B < 0 || Mp < 0) return WQ_E_NEG_DIM;
    if (P * B * Mp > 0 && (src == nullptr || dst == nullptr)) return WQ_E_NULL;
    cudaError_t e = wq::launch_gather_permute(src, P, B, Mp, dst, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

int wq_widen_f16_f32(const uint16_t* src, float* dst, int64_t n, void* stream) {
    if (n < 0) return WQ_E_NEG_DIM;
    if (n > 0 && (src == nullptr || dst == nullptr)) return WQ_E_NULL;
    cudaError_t e = wq::launch_widen_f16_f32(src, dst, n, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

int wq_narrow_f32_f16(const float* src, uint16_t* dst, int64_t n, void* stream) {
    if (n < 0) return WQ_E_NEG_DIM;
    if (n > 0 && (src == nullptr || dst == nullptr)) return WQ_E_NULL;
    cudaError_t e = wq::launch_narrow_f32_f16(src, dst, n, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

int wq_channel_abs_sum_f64(const float* x, int64_t n, int64_t K, int64_t ldx, double* acc, void* stream) {
    if (n < 0 || K < 0) return WQ_E_NEG_DIM;
    if (ldx < K) return WQ_E_LD;
    if (K > 0 && (acc == nullptr || (n > 0 && x == nullptr))) return WQ_E_NULL;
    if (n == 0 || K == 0) return WQ_OK;
    cudaError_t e = wq::launch_channel_abs_sum(x, n, K, ldx, acc, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

int wq_awq_pre_scale_f32(const float* mag, int64_t K, float alpha, float* pre, void* stream) {
    if (K < 0) return WQ_E_NEG_DIM;
    if (K > 0 && ((alpha != 0.0f && mag == nullptr) || pre == nullptr)) return WQ_E_NULL;
    cudaError_t e = wq::launch_pre_scale(mag, K, alpha, pre, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

size_t wq_sq_err_workspace_bytes(void) { return wq::sq_err_workspace_bytes(); }

int wq_sq_err_sum_f64(const float* a, const float* b, int64_t n, double* out, void* workspace, size_t workspace_bytes,
                      void* stream) {
    if (n < 0) return WQ_E_NEG_DIM;
    if (out == nullptr || (n > 0 && (a == nullptr || b == nullptr))) return WQ_E_NULL;
    if (workspace == nullptr || workspace_bytes < wq::sq_err_workspace_bytes()) return WQ_E_WORKSPACE;
    cudaError_t e = wq::launch_sq_err_sum(a, b, n, out, workspace, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

size_t wq_gptq_qparams_workspace_bytes(int64_t rows) { return rows > 0 ? wq::gptq_qparams_workspace_bytes(rows) : 0; }

int wq_gptq_qparams_f64(const double* w, int64_t rows, int64_t ld, int64_t c0, int64_t c1, int bits, int symmetric,
                        int per_tensor, double* scale_out, double* zero_out, int64_t out_stride, void* workspace,
                        size_t workspace_bytes, void* stream) {
    if (rows < 0 || c0 < 0 || c1 < c0 || out_stride < 0) return WQ_E_NEG_DIM;
    if (bits != 4 && bits != 8) return WQ_E_BITS;
    if (ld < c1) return WQ_E_LD;
    if (rows == 0) return WQ_OK;
    if (w == nullptr || scale_out == nullptr || zero_out == nullptr) return WQ_E_NULL;
    if (per_tensor && (workspace == nullptr || workspace_bytes < wq::gptq_qparams_workspace_bytes(rows)))
        return WQ_E_WORKSPACE;
    cudaError_t e = wq::launch_gptq_qparams(w, rows, ld, c0, c1, bits, symmetric, per_tensor, scale_out, zero_out,
                                            out_stride, static_cast<double*>(workspace),
                                            static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

int wq_gptq_block_f64(const double* w, int64_t rows, int64_t ld, const double* hinv, int64_t ldh, int64_t s0,
                      int count, const double* scale, const double* zero, int64_t qp_stride, int bits,
                      int32_t* codes, int64_t ldc, double* err_block, const uint8_t* zero_err, int32_t* bad_col,
                      void* stream) {
    if (rows < 0 || s0 < 0 || count < 0 || qp_stride < 0) return WQ_E_NEG_DIM;
    if (bits != 4 && bits != 8) return WQ_E_BITS;
    if (count > wq::gptq_max_block() || rows > kMaxDim) return WQ_E_TOO_LARGE;
    if (ld < s0 + count || ldh < s0 + count || ldc < s0 + count) return WQ_E_LD;
    if (rows == 0 || count == 0) return WQ_OK;
    if (w == nullptr || hinv == nullptr || scale == nullptr || zero == nullptr || codes == nullptr ||
        err_block == nullptr)
        return WQ_E_NULL;
    cudaError_t e = wq::launch_gptq_block(w, rows, ld, hinv, ldh, s0, count, scale, zero, qp_stride, bits, codes, ldc,
                                          err_block, zero_err, bad_col, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

int wq_gptq_tail_f64(double* w, int64_t rows, int64_t ld, int64_t c0, int64_t ncols, const double* err_block,
                     int count, const double* hinv, int64_t ldh, int64_t s0, void* stream) {
    if (rows < 0 || c0 < 0 || ncols < 0 || count < 0 || s0 < 0) return WQ_E_NEG_DIM;
    if (ld < c0 + ncols || ldh < c0 + ncols) return WQ_E_LD;
    if (rows == 0 || ncols == 0 || count == 0) return WQ_OK;
    if (w == nullptr || err_block == nullptr || hinv == nullptr) return WQ_E_NULL;
    if ((rows + 63) / 64 > 65535) return WQ_E_TOO_LARGE;
    cudaError_t e = wq::launch_gptq_tail(w, rows, ld, c0, ncols, err_block, count, hinv, ldh, s0,
                                         static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

size_t wq_chol_inverse_upper_workspace_bytes(int64_t n) {
    return n <= 0 ? 0 : wq::chol_inverse_upper_workspace_bytes(n);
}

int wq_chol_inverse_upper_f64(const double* a, int64_t n, int64_t lda, double* u, int64_t ldu, void* workspace,
                              size_t workspace_bytes, int32_t* info, void* stream) {
    if (n < 0) return WQ_E_NEG_DIM;
    if (info == nullptr) return WQ_E_NULL;
    if (n > 0 && (lda < n || ldu < n)) return WQ_E_LD;
    if (n > 0 && (a == nullptr || u == nullptr || workspace == nullptr)) return WQ_E_NULL;
    if (n > 0 && workspace_bytes < wq::chol_inverse_upper_workspace_bytes(n)) return WQ_E_WORKSPACE;
    if (n > 46340) return WQ_E_TOO_LARGE;   // n * n elements indexed by the rotation's grid
    cudaError_t e = wq::launch_chol_inverse_upper(a, n, lda, u, ldu, static_cast<double*>(workspace), info,
                                                  static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WQ_OK : cuda_fail(e);
}

}  // extern "C"

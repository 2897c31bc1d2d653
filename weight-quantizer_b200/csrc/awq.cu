// AWQ search reductions (ptqkit src/ptqkit/awq.py:39-81, convert.py:35-63).
//
// The alpha search quantizes W diag(s(alpha)) with the RTN kernels and scores
// it with the dequant-GEMM; what remains are three reductions, each written
// here as a deterministic kernel (fixed summation order, no atomics on data):
//
//   channel_abs_sum   acc[k] += sum_i |x[i, k]|, in fp64, rows in order: the
//                     activation statistic of ActivationStats.update
//                     (convert.py:40-49, x64.abs().sum(dim=0)) and, divided
//                     by n, awq.py:61's activations.abs().mean(dim=0).
//   pre_scale         s_k = m_k^alpha / max(mean(m^alpha), 1e-8), m already
//                     clamped to >= 1e-8 (awq.py:70-74); alpha = 0 gives 1.
//   sq_err_sum        sum_i (a_i - b_i)^2 in fp64 (awq.py:76-77), partials
//                     per block, then one block adds them in block order.
#include "common.cuh"
#include "kernels.h"

namespace wq {
namespace {

constexpr int kColThreads = 128;
constexpr int kSqBlocks = 592;    // 4 per SM on B200; fixed so that the order is too
constexpr int kSqThreads = 256;

__global__ void __launch_bounds__(kColThreads) channel_abs_sum_kernel(const float* __restrict__ x, int64_t n,
                                                                    int64_t K, int64_t ldx,
                                                                    double* __restrict__ acc) {
    const int64_t k = (int64_t)blockIdx.x * kColThreads + threadIdx.x;
    if (k >= K) return;
    const float* col = x + k;
    double s = 0.0;
    int64_t i = 0;
    // eight rows in flight per thread; the additions stay in row order
    for (; i + 8 <= n; i += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __ldg(col + (i + j) * ldx);
#pragma unroll
        for (int j = 0; j < 8; ++j) s += (double)fabsf(v[j]);
    }
    for (; i < n; ++i) s += (double)fabsf(__ldg(col + i * ldx));
    acc[k] += s;
}

// One block: s_k = m_k^alpha, then the mean in fp64 over a fixed tree, then
// s_k / max(mean, 1e-8) rounded to fp32. The power is taken in fp64 and
// rounded once to fp32, which gives the correctly rounded fp32 power except
// where the exact value lies within a few fp64 ulps of a rounding boundary:
// a value defined by the mathematics, not by one math library's fp32 pow.
constexpr int kPreThreads = 1024;
__global__ void __launch_bounds__(kPreThreads) pre_scale_kernel(const float* __restrict__ mag, int64_t K, float alpha,
                                                               float* __restrict__ pre) {
    __shared__ double part[kPreThreads / 32];
    if (alpha == 0.0f) {
        for (int64_t k = threadIdx.x; k < K; k += kPreThreads) pre[k] = 1.0f;
        return;
    }
    double s = 0.0;
    for (int64_t k = threadIdx.x; k < K; k += kPreThreads) {
        const float p = (float)pow((double)mag[k], (double)alpha);
        pre[k] = p;
        s += (double)p;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        double v = part[threadIdx.x];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) part[0] = v;
    }
    __syncthreads();
    float mean = (float)(part[0] / (double)K);
    mean = mean < 1e-8f ? 1e-8f : mean;
    for (int64_t k = threadIdx.x; k < K; k += kPreThreads) pre[k] = __fdiv_rn(pre[k], mean);
}

__global__ void __launch_bounds__(kSqThreads) sq_err_partial_kernel(const float* __restrict__ a,
                                                                   const float* __restrict__ b, int64_t n,
                                                                   double* __restrict__ partial) {
    __shared__ double part[kSqThreads / 32];
    double s = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * kSqThreads + threadIdx.x; i < n; i += (int64_t)kSqBlocks * kSqThreads) {
        const double d = (double)__ldg(a + i) - (double)__ldg(b + i);
        s = fma(d, d, s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double v = 0.0;
        for (int w = 0; w < kSqThreads / 32; ++w) v += part[w];
        partial[blockIdx.x] = v;
    }
}

__global__ void __launch_bounds__(32) sq_err_final_kernel(const double* __restrict__ partial, double* __restrict__ out) {
    double s = 0.0;
    for (int i = threadIdx.x; i < kSqBlocks; i += 32) s += partial[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) *out = s;
}

}  // namespace

cudaError_t launch_channel_abs_sum(const float* x, int64_t n, int64_t K, int64_t ldx, double* acc, cudaStream_t s) {
    if (K == 0) return cudaSuccess;
    const int64_t blocks = (K + kColThreads - 1) / kColThreads;
    channel_abs_sum_kernel<<<(unsigned)blocks, kColThreads, 0, s>>>(x, n, K, ldx, acc);
    return cudaGetLastError();
}

cudaError_t launch_pre_scale(const float* mag, int64_t K, float alpha, float* pre, cudaStream_t s) {
    if (K == 0) return cudaSuccess;
    pre_scale_kernel<<<1, kPreThreads, 0, s>>>(mag, K, alpha, pre);
    return cudaGetLastError();
}

size_t sq_err_workspace_bytes() { return (size_t)kSqBlocks * sizeof(double); }

cudaError_t launch_sq_err_sum(const float* a, const float* b, int64_t n, double* out, void* workspace,
                              cudaStream_t s) {
    double* partial = static_cast<double*>(workspace);
    sq_err_partial_kernel<<<kSqBlocks, kSqThreads, 0, s>>>(a, b, n, partial);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    sq_err_final_kernel<<<1, 32, 0, s>>>(partial, out);
    return cudaGetLastError();
}

}  // namespace wq

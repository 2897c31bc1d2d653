// Generic tiled dequant-GEMM on the SIMT fp32 pipe: every shape, alignment and
// group size ptqkit's storage allows (odd K, odd group starts, unaligned rows,
// scale_rows == 1 broadcast, K == 1). It is the path for the layouts the
// streaming and tensor-core kernels do not take.
//
// Each weight element is reconstructed exactly as the reference does it,
// w = ((float)code - zero) * scale [* channel[k]]
// (src/ptqkit/csrc/dequant_gemm.cpp:57-120; nibble rule :49-55, broadcast :30-34),
// staged in shared memory as a 64 x 32 tile, and multiplied against a 64 x 32
// tile of x with fp32 FMAs (4 x 4 outputs per thread).
#include "common.cuh"
#include "kernels.h"

namespace wq {
namespace {

constexpr int BM = 64;  // weight rows per CTA
constexpr int BN = 64;  // batch rows per CTA
constexpr int BK = 32;

__device__ __forceinline__ int code_at(const uint8_t* row, int64_t k, int bits) {
    if (bits == 8) return (int)row[k];
    const uint8_t byte = row[k >> 1];
    return (k & 1) == 0 ? (int)(byte & 0x0F) : (int)(byte >> 4);
}

__global__ void __launch_bounds__(256) gemm_simt_kernel(const GemmProblem p) {
    __shared__ float ws[BK][BM + 4];
    __shared__ float xs[BK][BN + 4];
    const int tid = threadIdx.x;
    const int tm = tid & 15;   // 4 weight rows each
    const int tb = tid >> 4;   // 4 batch rows each
    const int64_t m0 = (int64_t)blockIdx.x * BM;
    const int64_t b0 = (int64_t)blockIdx.y * BN;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

    for (int64_t k0 = 0; k0 < p.K; k0 += BK) {
#pragma unroll
        for (int i = 0; i < (BM * BK) / 256; ++i) {
            const int e = tid + i * 256;
            const int mm = e / BK, kk = e % BK;
            const int64_t m = m0 + mm, k = k0 + kk;
            float w = 0.0f;
            if (m < p.M && k < p.K) {
                const int64_t g = k / p.group_size;
                const int64_t srow = p.scale_rows == 1 ? 0 : m;
                const int64_t gi = p.groups == 1 ? 0 : g;
                const float scale = p.scales[srow * p.groups + gi];
                const float zero = p.zeros[srow * p.groups + gi];
                w = ((float)code_at(p.q + m * p.q_stride, k, p.bits) - zero) * scale;
                if (p.channel != nullptr) w = w * p.channel[k];
            }
            ws[kk][mm] = w;
        }
#pragma unroll
        for (int i = 0; i < (BN * BK) / 256; ++i) {
            const int e = tid + i * 256;
            const int bb = e / BK, kk = e % BK;
            const int64_t b = b0 + bb, k = k0 + kk;
            xs[kk][bb] = (b < p.B && k < p.K) ? p.x[b * p.K + k] : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < BK; ++kk) {
            float a[4], bx[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = ws[kk][tm * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bx[j] = xs[kk][tb * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bx[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int64_t b = b0 + tb * 4 + j;
        if (b >= p.B) continue;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t m = m0 + tm * 4 + i;
            if (m < p.M) {
                float v = acc[i][j];
                if (p.bias != nullptr) v = __fadd_rn(v, p.bias[m]);   // linear.py:99-100, one fp32 add
                p.y[b * p.ldy + m] = v;
            }
        }
    }
}

__global__ void fill_zero_kernel(float* y, int64_t B, int64_t M, int64_t ldy) {
    const int64_t n = B * M;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = i / M, m = i - b * M;
        y[b * ldy + m] = 0.0f;
    }
}

// y = 0 + bias[m]: the reference's zero result plus its bias add.
__global__ void fill_bias_kernel(float* y, int64_t B, int64_t M, int64_t ldy, const float* bias) {
    const int64_t n = B * M;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = i / M, m = i - b * M;
        y[b * ldy + m] = 0.0f + bias[m];
    }
}

}  // namespace

cudaError_t launch_gemm_simt(const GemmProblem& p, cudaStream_t s) {
    const int64_t gm = (p.M + BM - 1) / BM;
    const int64_t gb = (p.B + BN - 1) / BN;
    if (gm > 0x7fffffff || gb > 65535) return cudaErrorInvalidValue;
    dim3 grid((unsigned)gm, (unsigned)gb);
    gemm_simt_kernel<<<grid, 256, 0, s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_fill_zero(float* y, int64_t B, int64_t M, int64_t ldy, cudaStream_t s) {
    const int64_t n = B * M;
    if (n == 0) return cudaSuccess;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    fill_zero_kernel<<<(unsigned)blocks, 256, 0, s>>>(y, B, M, ldy);
    return cudaGetLastError();
}

cudaError_t launch_fill_bias(float* y, int64_t B, int64_t M, int64_t ldy, const float* bias, cudaStream_t s) {
    const int64_t n = B * M;
    if (n == 0) return cudaSuccess;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    fill_bias_kernel<<<(unsigned)blocks, 256, 0, s>>>(y, B, M, ldy, bias);
    return cudaGetLastError();
}

}  // namespace wq

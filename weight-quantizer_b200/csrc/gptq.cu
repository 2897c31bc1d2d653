// GPTQ column sweep (ptqkit src/ptqkit/gptq.py:86-191) on the device, fp64.
//
// Given the upper Cholesky factor U of the damped inverse Hessian (computed
// by the caller), GPTQ quantizes the columns of W left to right and corrects
// the not-yet-quantized columns of every row with the OBS step
//
//     err_r = (w_ri - w_hat_ri) / U_ii,      w_rj -= err_r * U_ij   (j > i).
//
// Rows never interact, so a block of up to 128 columns is swept with one warp
// per weight row: lane l holds columns l, l+32, l+64, l+96 of the block in
// registers, each column's value is broadcast from its lane, every lane
// computes the (row-uniform) code and error and updates its own columns with
// U's row i, staged in shared memory. The arithmetic follows the reference
// operation by operation (divide, round half to even, add the zero, clamp;
// product then difference, never fused), so one block sweep is bit-exact
// with ptqkit's _obs_block given the same inputs. The update of the columns
// past the block is one fp64 GEMM, done by the caller (gptq.py:124-125).
//
// qparams_rows / qparams_tensor restate quant.py:146-172 in fp64 over a
// column range of the updated weights (gptq.py:162-178): per row (group and
// channel granularity) or over the whole matrix (tensor granularity).
#include <cfloat>

#include "common.cuh"
#include "kernels.h"

namespace wq {
namespace {

constexpr int kGptqWarps = 8;     // rows per CTA in the block sweep
constexpr int kGptqBlock = 128;   // most columns one sweep holds (4 per lane)

// min and max of a row segment; a minimum of zero keeps the sign of the
// first zero met (the reference reduces in an unspecified order; only the
// stored zero point's sign bit can depend on it)
struct MinMax {
    double mn, mx;
};

__device__ __forceinline__ MinMax combine(MinMax a, MinMax b) {
    MinMax r;
    r.mn = (b.mn < a.mn) ? b.mn : a.mn;
    r.mx = (b.mx > a.mx) ? b.mx : a.mx;
    return r;
}

__device__ __forceinline__ void qparams_from(double mn, double mx, int symmetric, int qmax, double& scale,
                                             double& zero) {
    if (symmetric) {
        const double amax = fmax(fabs(mn), fabs(mx));
        scale = amax > 0.0 ? __ddiv_rn(__dmul_rn(2.0, amax), (double)qmax) : 1.0;
        zero = (double)(qmax + 1) / 2.0;
        return;
    }
    double xmin = mn > 0.0 ? 0.0 : mn;   // torch.minimum(xmin, 0): a zero minimum keeps its sign
    double xmax = mx > 0.0 ? mx : 0.0;   // torch.maximum(xmax, 0)
    if (xmin == 0.0 && xmax == 0.0) {
        xmin = -1.0;
        xmax = 1.0;
    }
    double s = __ddiv_rn(__dsub_rn(xmax, xmin), (double)qmax);
    s = s > 0.0 ? s : 1.0;
    double z = rint(__ddiv_rn(-xmin, s));
    z = z < 0.0 ? 0.0 : (z > (double)qmax ? (double)qmax : z);
    scale = s;
    zero = z;
}

// One warp per row: min/max over columns [c0, c1), then the row's scale and
// zero (per_row) or the partial (min, max) for the tensor reduction.
__global__ void __launch_bounds__(256) qparams_rows_kernel(const double* __restrict__ w, int64_t rows, int64_t ld,
                                                           int64_t c0, int64_t c1, int symmetric, int qmax,
                                                           int per_row, double* __restrict__ scale_out,
                                                           double* __restrict__ zero_out, int64_t out_stride,
                                                           double* __restrict__ partial) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= rows) return;
    const double* p = w + row * ld;
    MinMax m{DBL_MAX, -DBL_MAX};
    bool any = false;
    for (int64_t c = c0 + lane; c < c1; c += 32) {
        const double v = p[c];
        if (!any) {
            m.mn = v;
            m.mx = v;
            any = true;
        } else {
            if (v < m.mn) m.mn = v;
            if (v > m.mx) m.mx = v;
        }
    }
    // lanes in order, so that among equal zeros the lowest column's sign is kept
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        MinMax other;
        other.mn = __shfl_down_sync(0xffffffffu, m.mn, o);
        other.mx = __shfl_down_sync(0xffffffffu, m.mx, o);
        const bool other_any = __shfl_down_sync(0xffffffffu, any ? 1 : 0, o) != 0;
        if (lane + o < 32 && other_any) {
            m = any ? combine(m, other) : other;
            any = true;
        }
    }
    if (lane != 0) return;
    if (per_row) {
        double s, z;
        qparams_from(m.mn, m.mx, symmetric, qmax, s, z);
        scale_out[row * out_stride] = s;
        zero_out[row * out_stride] = z;
    } else {
        partial[2 * row] = m.mn;
        partial[2 * row + 1] = m.mx;
    }
}

// One thread reduces the rows' partials in row order (tensor granularity).
__global__ void qparams_tensor_kernel(const double* __restrict__ partial, int64_t rows, int symmetric, int qmax,
                                      double* __restrict__ scale_out, double* __restrict__ zero_out) {
    MinMax m{partial[0], partial[1]};
    for (int64_t r = 1; r < rows; ++r) m = combine(m, MinMax{partial[2 * r], partial[2 * r + 1]});
    double s, z;
    qparams_from(m.mn, m.mx, symmetric, qmax, s, z);
    scale_out[0] = s;
    zero_out[0] = z;
}

__global__ void __launch_bounds__(kGptqWarps * 32) gptq_block_kernel(
    const double* __restrict__ w, int64_t rows, int64_t ld, const double* __restrict__ hinv, int64_t ldh,
    int64_t s0, int count, const double* __restrict__ scale, const double* __restrict__ zero, int64_t qp_stride,
    int qmax, int32_t* __restrict__ codes, int64_t ldc, double* __restrict__ err_block,
    const uint8_t* __restrict__ zero_err, int* __restrict__ bad_col) {
    extern __shared__ double h_s[];   // [count][count]: U[s0 + i][s0 + j]
    for (int idx = threadIdx.x; idx < count * count; idx += blockDim.x) {
        const int i = idx / count, j = idx - i * count;
        h_s[idx] = hinv[(s0 + i) * ldh + s0 + j];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kGptqWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    const double* wr = w + row * ld + s0;
    double v[kGptqBlock / 32];
#pragma unroll
    for (int s = 0; s < kGptqBlock / 32; ++s) {
        const int j = s * 32 + lane;
        v[s] = j < count ? wr[j] : 0.0;
    }
    const double sc = scale[row * qp_stride];
    const double zz = zero[row * qp_stride];
    int32_t* crow = codes + row * ldc + s0;
    double* erow = err_block + row * (int64_t)count;
#pragma unroll
    for (int s = 0; s < kGptqBlock / 32; ++s) {
#pragma unroll 1
        for (int l = 0; l < 32; ++l) {
            const int i = s * 32 + l;
            if (i >= count) break;
            const double col = __shfl_sync(0xffffffffu, v[s], l);
            // integer_codes (quant.py:175-184): round(w / scale) + zero, clamped
            double q = __dadd_rn(rint(__ddiv_rn(col, sc)), zz);
            q = q < 0.0 ? 0.0 : (q > (double)qmax ? (double)qmax : q);
            const double deq = __dmul_rn(sc, __dsub_rn(q, zz));
            const double d = h_s[i * count + i];
            double err = __ddiv_rn(__dsub_rn(col, deq), d < 1e-8 ? 1e-8 : d);
            // _obs_block zeroes a column's whole error when any row's is not
            // finite (gptq.py:114-115). A row cannot see the other rows here,
            // so the first such column is reported and the caller sweeps the
            // block again with that column's error set to zero.
            if (zero_err != nullptr && zero_err[i] != 0) {
                err = 0.0;
            } else if (bad_col != nullptr && !isfinite(err) && lane == l) {
                atomicMin(bad_col, i);
            }
            if (lane == l) {
                crow[i] = (int32_t)q;
                erow[i] = err;
            }
            // block[:, i:] -= err * U[i, i:] (gptq.py:117-118), columns past i
#pragma unroll
            for (int s2 = 0; s2 < kGptqBlock / 32; ++s2) {
                const int j = s2 * 32 + lane;
                if (s2 >= s && j > i && j < count) v[s2] = __dsub_rn(v[s2], __dmul_rn(err, h_s[i * count + j]));
            }
        }
    }
}

// work[r, c0 + j] -= sum_i err[r, i] * hinv[s0 + i, c0 + j]: the tail update
// after one block (gptq.py:124-125), a 64 x 64 output tile per CTA, 4 x 4 per
// thread, the i sum in order (deterministic), then one subtraction.
constexpr int kTailT = 64, kTailK = 16;
__global__ void __launch_bounds__(256) gptq_tail_kernel(double* __restrict__ work, int64_t rows, int64_t ld, int64_t c0,
                                                        int64_t ncols, const double* __restrict__ err, int count,
                                                        const double* __restrict__ hinv, int64_t ldh, int64_t s0) {
    __shared__ double es[kTailK][kTailT + 1];   // err^T tile: [i][row]
    __shared__ double hs[kTailK][kTailT];       // hinv tile: [i][col]
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t r0 = (int64_t)blockIdx.y * kTailT, j0 = (int64_t)blockIdx.x * kTailT;
    double acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = 0.0;
    for (int k0 = 0; k0 < count; k0 += kTailK) {
        for (int idx = threadIdx.x; idx < kTailK * kTailT; idx += 256) {
            const int kk = idx % kTailK, rr = idx / kTailK;   // consecutive threads walk i of one row
            const int64_t r = r0 + rr;
            es[kk][rr] = (r < rows && k0 + kk < count) ? err[r * count + k0 + kk] : 0.0;
            const int cc = idx % kTailT, k2 = idx / kTailT;
            const int64_t j = j0 + cc;
            hs[k2][cc] = (j < ncols && k0 + k2 < count) ? hinv[(s0 + k0 + k2) * ldh + c0 + j] : 0.0;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kTailK; ++kk) {
            double ev[4], hv[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) ev[a] = es[kk][ty * 4 + a];
#pragma unroll
            for (int b = 0; b < 4; ++b) hv[b] = hs[kk][tx * 4 + b];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = fma(ev[a], hv[b], acc[a][b]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int64_t r = r0 + ty * 4 + a;
        if (r >= rows) continue;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int64_t j = j0 + tx * 4 + b;
            if (j < ncols) work[r * ld + c0 + j] = __dsub_rn(work[r * ld + c0 + j], acc[a][b]);
        }
    }
}

}  // namespace

cudaError_t launch_gptq_tail(double* work, int64_t rows, int64_t ld, int64_t c0, int64_t ncols, const double* err,
                             int count, const double* hinv, int64_t ldh, int64_t s0, cudaStream_t s) {
    if (rows == 0 || ncols == 0 || count == 0) return cudaSuccess;
    const dim3 grid((unsigned)((ncols + kTailT - 1) / kTailT), (unsigned)((rows + kTailT - 1) / kTailT));
    gptq_tail_kernel<<<grid, 256, 0, s>>>(work, rows, ld, c0, ncols, err, count, hinv, ldh, s0);
    return cudaGetLastError();
}

size_t gptq_qparams_workspace_bytes(int64_t rows) { return (size_t)rows * 2 * sizeof(double); }

cudaError_t launch_gptq_qparams(const double* w, int64_t rows, int64_t ld, int64_t c0, int64_t c1, int bits,
                                int symmetric, int per_tensor, double* scale_out, double* zero_out,
                                int64_t out_stride, double* workspace, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    const int qmax = (1 << bits) - 1;
    const unsigned grid = (unsigned)((rows + 7) / 8);
    qparams_rows_kernel<<<grid, 256, 0, s>>>(w, rows, ld, c0, c1, symmetric, qmax, per_tensor ? 0 : 1, scale_out,
                                             zero_out, out_stride, workspace);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || !per_tensor) return e;
    qparams_tensor_kernel<<<1, 1, 0, s>>>(workspace, rows, symmetric, qmax, scale_out, zero_out);
    return cudaGetLastError();
}

int gptq_max_block() { return kGptqBlock; }

cudaError_t launch_gptq_block(const double* w, int64_t rows, int64_t ld, const double* hinv, int64_t ldh,
                              int64_t s0, int count, const double* scale, const double* zero, int64_t qp_stride,
                              int bits, int32_t* codes, int64_t ldc, double* err_block, const uint8_t* zero_err,
                              int* bad_col, cudaStream_t s) {
    if (rows == 0 || count == 0) return cudaSuccess;
    const size_t smem = (size_t)count * count * sizeof(double);
    cudaError_t e = cudaFuncSetAttribute(gptq_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const unsigned grid = (unsigned)((rows + kGptqWarps - 1) / kGptqWarps);
    gptq_block_kernel<<<grid, kGptqWarps * 32, smem, s>>>(w, rows, ld, hinv, ldh, s0, count, scale, zero, qp_stride,
                                                          (1 << bits) - 1, codes, ldc, err_block, zero_err, bad_col);
    return cudaGetLastError();
}

}  // namespace wq

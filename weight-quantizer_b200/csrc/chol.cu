// Upper Cholesky factor of an inverse, fp64: the factor GPTQ sweeps with.
//
// ptqkit (src/ptqkit/gptq.py:59-66) takes the damped Hessian H, factors it
// (H = L L^T), forms H^-1 from that factor and factors H^-1 again, upper
// (H^-1 = U^T U). The same U comes from one factorization and one triangular
// inverse. With J the matrix that reverses the order of rows and columns,
// factor the reversed matrix: J H J = M M^T (M lower). Then H = R R^T with
// R = J M J upper, so H^-1 = R^-T R^-1 = (R^-1)^T R^-1, and R^-1 = J M^-1 J is
// upper with a positive diagonal: by uniqueness of the Cholesky factor it is
// U. The steps:
//
//   1. M = chol(J H J), blocked right-looking in 64-column blocks: the
//      diagonal block factored in shared memory by one CTA, the panel below it
//      by forward substitution (one thread per row), the trailing lower
//      triangle updated with 64 x 64 tiles (4 x 4 per thread);
//   2. X = M^-1, blocked from the bottom-right block up: the diagonal block
//      inverted in shared memory, the panel below it as
//      X21 = -(X22 M21) X11 with X22 already inverted;
//   3. U = J X J (a 180-degree rotation of the matrix, in place), zero below
//      the diagonal.
//
// A pivot that is not positive and finite records 1 + its column (of the
// reversed matrix) in the caller's info word; the caller damps H more and
// tries again, as gptq.py:67-70 does.
#include "common.cuh"
#include "kernels.h"

namespace wq {
namespace {

constexpr int kNB = 64;   // block size of both blocked algorithms

// L[i, j] = A[n-1-i, n-1-j] for j <= i (the lower triangle of J A J)
__global__ void __launch_bounds__(256) reverse_lower_kernel(const double* __restrict__ a, int64_t lda,
                                                            double* __restrict__ l, int64_t n) {
    const int64_t i = blockIdx.x;
    const double* src = a + (n - 1 - i) * lda + (n - 1);
    for (int64_t j = threadIdx.x; j <= i; j += blockDim.x) l[i * n + j] = src[-j];
}

// Cholesky of the diagonal block [j0, j0 + b) in shared memory (lower).
__global__ void __launch_bounds__(256) potrf_diag_kernel(double* __restrict__ l, int64_t n, int64_t j0, int b,
                                                         int* __restrict__ info) {
    __shared__ double s[kNB][kNB + 1];
    const int tid = threadIdx.x;
    for (int idx = tid; idx < b * b; idx += 256) {
        const int r = idx / b, c = idx % b;
        s[r][c] = c <= r ? l[(j0 + r) * n + j0 + c] : 0.0;
    }
    __syncthreads();
    for (int k = 0; k < b; ++k) {
        const double piv = s[k][k];
        if (tid == 0 && !(piv > 0.0 && isfinite(piv))) atomicCAS(info, 0, (int)(j0 + k + 1));
        const double d = sqrt(piv);
        __syncthreads();   // every thread has read the pivot
        if (tid == 0) s[k][k] = d;
        for (int i = k + 1 + tid; i < b; i += 256) s[i][k] = s[i][k] / d;
        __syncthreads();
        const int m = b - k - 1;
        for (int idx = tid; idx < m * m; idx += 256) {
            const int r = k + 1 + idx / m, c = k + 1 + idx % m;
            if (c <= r) s[r][c] = s[r][c] - s[r][k] * s[c][k];
        }
        __syncthreads();
    }
    for (int idx = tid; idx < b * b; idx += 256) {
        const int r = idx / b, c = idx % b;
        if (c <= r) l[(j0 + r) * n + j0 + c] = s[r][c];
    }
}

// Panel below the diagonal block: rows i >= j0 + b solve x L11^T = a, one
// warp of 32 rows per CTA, one row per lane, the row in shared memory.
constexpr int kTrsmRows = 32;
__global__ void __launch_bounds__(kTrsmRows) trsm_panel_kernel(double* __restrict__ l, int64_t n, int64_t j0, int b) {
    __shared__ double ld[kNB][kNB];          // the factored diagonal block
    __shared__ double xs[kNB][kTrsmRows];    // [k][lane]: the lane's row
    const int lane = threadIdx.x;
    for (int idx = lane; idx < b * b; idx += kTrsmRows) {
        const int r = idx / b, c = idx % b;
        ld[r][c] = c <= r ? l[(j0 + r) * n + j0 + c] : 0.0;
    }
    const int64_t i = j0 + b + (int64_t)blockIdx.x * kTrsmRows + lane;
    const bool valid = i < n;
    for (int k = 0; k < b; ++k) xs[k][lane] = valid ? l[i * n + j0 + k] : 0.0;
    __syncthreads();
    for (int k = 0; k < b; ++k) {
        double v = xs[k][lane];
        for (int q = 0; q < k; ++q) v = v - xs[q][lane] * ld[k][q];
        xs[k][lane] = v / ld[k][k];
    }
    if (valid)
        for (int k = 0; k < b; ++k) l[i * n + j0 + k] = xs[k][lane];
}

// Trailing update: L[i, j] -= sum_c P[i, c] P[j, c] for j <= i, both >= j0 + b,
// P = L[:, j0 : j0 + b]; 64 x 64 tiles on and below the diagonal.
constexpr int kT = 64, kKc = 16;
__global__ void __launch_bounds__(256) syrk_kernel(double* __restrict__ l, int64_t n, int64_t j0, int b) {
    const int tr = blockIdx.y, tc = blockIdx.x;
    if (tc > tr) return;
    __shared__ double ps[kKc][kT + 1];   // [c][row of tile tr]
    __shared__ double qs[kKc][kT + 1];   // [c][row of tile tc]
    const int64_t s = j0 + b;
    const int64_t r0 = s + (int64_t)tr * kT, c0 = s + (int64_t)tc * kT;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    double acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[a][q] = 0.0;
    for (int k0 = 0; k0 < b; k0 += kKc) {
        for (int idx = threadIdx.x; idx < kKc * kT; idx += 256) {
            const int kk = idx % kKc, rr = idx / kKc;
            const bool kin = k0 + kk < b;
            ps[kk][rr] = (kin && r0 + rr < n) ? l[(r0 + rr) * n + j0 + k0 + kk] : 0.0;
            qs[kk][rr] = (kin && c0 + rr < n) ? l[(c0 + rr) * n + j0 + k0 + kk] : 0.0;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kKc; ++kk) {
            double pv[4], qv[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) pv[a] = ps[kk][ty * 4 + a];
#pragma unroll
            for (int q = 0; q < 4; ++q) qv[q] = qs[kk][tx * 4 + q];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[a][q] = fma(pv[a], qv[q], acc[a][q]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int64_t i = r0 + ty * 4 + a;
        if (i >= n) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int64_t j = c0 + tx * 4 + q;
            if (j <= i) l[i * n + j] = l[i * n + j] - acc[a][q];
        }
    }
}

// Inverse of the lower diagonal block [j0, j0 + b) of L into X (zeros above
// its diagonal); thread c solves column c. Both triangles packed in shared
// memory: element (i, j), j <= i, at i (i + 1) / 2 + j.
__device__ __forceinline__ int tri(int i, int j) { return i * (i + 1) / 2 + j; }
__global__ void __launch_bounds__(kNB) trtri_diag_kernel(const double* __restrict__ l, int64_t n,
                                                         double* __restrict__ x, int64_t ldx, int64_t j0, int b) {
    __shared__ double lp[kNB * (kNB + 1) / 2];
    __shared__ double xp[kNB * (kNB + 1) / 2];
    const int c = threadIdx.x;
    for (int idx = c; idx < b * b; idx += kNB) {
        const int r = idx / b, q = idx % b;
        if (q <= r) lp[tri(r, q)] = l[(j0 + r) * n + j0 + q];
    }
    __syncthreads();
    if (c < b) {
        for (int i = c; i < b; ++i) {
            double v = i == c ? 1.0 : 0.0;
            for (int q = c; q < i; ++q) v = v - lp[tri(i, q)] * xp[tri(q, c)];
            xp[tri(i, c)] = v / lp[tri(i, i)];
        }
    }
    __syncthreads();
    for (int idx = c; idx < b * b; idx += kNB) {
        const int r = idx / b, q = idx % b;
        x[(j0 + r) * ldx + j0 + q] = q <= r ? xp[tri(r, q)] : 0.0;
    }
}

// Panel of the inverse: rows i >= s = j0 + b, columns [j0, j0 + b):
// X[i, :] = -(sum_{s <= k <= i} X[i, k] L[k, :]) X11, one 64-row tile of
// rows per CTA (4 x 4 outputs per thread). Dynamic shared memory: the two
// staging tiles of the first product, then Y and X11 for the second.
constexpr size_t kTrmmSmem = (size_t)(kT * (kT + 1) + kNB * kNB) * sizeof(double);
__global__ void __launch_bounds__(256) trmm_panel_kernel(const double* __restrict__ l, int64_t n,
                                                         double* __restrict__ x, int64_t ldx, int64_t j0, int b) {
    extern __shared__ double smem_d[];
    double (*es)[kT + 1] = reinterpret_cast<double (*)[kT + 1]>(smem_d);                 // [k][row]
    double (*hs)[kT] = reinterpret_cast<double (*)[kT]>(smem_d + kKc * (kT + 1));        // [k][col]
    const int64_t s = j0 + b, m = n - s;
    const int64_t rt0 = (int64_t)blockIdx.x * kT;   // first row of the tile, relative to s
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    double acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[a][q] = 0.0;
    const int64_t kend = min(m, rt0 + kT);   // X[i, k] = 0 for k > i
    for (int64_t k0 = 0; k0 < kend; k0 += kKc) {
        for (int idx = threadIdx.x; idx < kKc * kT; idx += 256) {
            const int kk = idx % kKc, rr = idx / kKc;
            const int64_t ri = rt0 + rr, k = k0 + kk;
            es[kk][rr] = (ri < m && k <= ri) ? x[(s + ri) * ldx + s + k] : 0.0;
            const int cc = idx % kT, k2 = idx / kT;
            const int64_t kb = k0 + k2;
            hs[k2][cc] = (kb < m && cc < b) ? l[(s + kb) * n + j0 + cc] : 0.0;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kKc; ++kk) {
            double ev[4], hv[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) ev[a] = es[kk][ty * 4 + a];
#pragma unroll
            for (int q = 0; q < 4; ++q) hv[q] = hs[kk][tx * 4 + q];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[a][q] = fma(ev[a], hv[q], acc[a][q]);
        }
        __syncthreads();
    }
    // second product: out = -Y X11 (X11 lower, from this step's diagonal inverse)
    double (*ys)[kT + 1] = reinterpret_cast<double (*)[kT + 1]>(smem_d);
    double (*x11)[kNB] = reinterpret_cast<double (*)[kNB]>(smem_d + kT * (kT + 1));
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int q = 0; q < 4; ++q) ys[ty * 4 + a][tx * 4 + q] = acc[a][q];
    for (int idx = threadIdx.x; idx < kNB * kNB; idx += 256) {
        const int r = idx / kNB, q = idx % kNB;
        x11[r][q] = (r < b && q <= r) ? x[(j0 + r) * ldx + j0 + q] : 0.0;
    }
    __syncthreads();
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[a][q] = 0.0;
    for (int p = 0; p < b; ++p) {
        double yv[4], xv[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) yv[a] = ys[ty * 4 + a][p];
#pragma unroll
        for (int q = 0; q < 4; ++q) xv[q] = x11[p][tx * 4 + q];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[a][q] = fma(yv[a], xv[q], acc[a][q]);
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int64_t ri = rt0 + ty * 4 + a;
        if (ri >= m) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int cc = tx * 4 + q;
            if (cc < b) x[(s + ri) * ldx + j0 + cc] = -acc[a][q];
        }
    }
}

// In place: U[i, j] = X[n-1-i, n-1-j] for j >= i, 0 below the diagonal.
// Thread p swaps element p of the row-major order with its mirror.
__global__ void __launch_bounds__(256) rotate_upper_kernel(double* __restrict__ u, int64_t ldu, int64_t n,
                                                           int64_t half) {
    const int64_t p = (int64_t)blockIdx.x * 256 + threadIdx.x;
    if (p >= half) return;
    const int64_t i = p / n, j = p - i * n;
    const int64_t i2 = n - 1 - i, j2 = n - 1 - j;
    const double v = u[i * ldu + j], w = u[i2 * ldu + j2];
    u[i * ldu + j] = j >= i ? w : 0.0;
    u[i2 * ldu + j2] = j2 >= i2 ? v : 0.0;
}

}  // namespace

size_t chol_inverse_upper_workspace_bytes(int64_t n) { return (size_t)n * (size_t)n * sizeof(double); }

cudaError_t launch_chol_inverse_upper(const double* a, int64_t n, int64_t lda, double* u, int64_t ldu,
                                      double* work, int* info, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(info, 0, sizeof(int), s);
    if (e != cudaSuccess || n == 0) return e;
    double* l = work;
    reverse_lower_kernel<<<(unsigned)n, 256, 0, s>>>(a, lda, l, n);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    // 1. M = chol(J A J)
    for (int64_t j0 = 0; j0 < n; j0 += kNB) {
        const int b = (int)min((int64_t)kNB, n - j0);
        potrf_diag_kernel<<<1, 256, 0, s>>>(l, n, j0, b, info);
        const int64_t m = n - j0 - b;
        if (m > 0) {
            trsm_panel_kernel<<<(unsigned)((m + kTrsmRows - 1) / kTrsmRows), kTrsmRows, 0, s>>>(l, n, j0, b);
            const unsigned t = (unsigned)((m + kT - 1) / kT);
            syrk_kernel<<<dim3(t, t), 256, 0, s>>>(l, n, j0, b);
        }
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    // 2. X = M^-1 into u, from the last block up
    e = cudaFuncSetAttribute(trmm_panel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTrmmSmem);
    if (e != cudaSuccess) return e;
    for (int64_t j0 = ((n - 1) / kNB) * kNB; j0 >= 0; j0 -= kNB) {
        const int b = (int)min((int64_t)kNB, n - j0);
        trtri_diag_kernel<<<1, kNB, 0, s>>>(l, n, u, ldu, j0, b);
        const int64_t m = n - j0 - b;
        if (m > 0)
            trmm_panel_kernel<<<(unsigned)((m + kT - 1) / kT), 256, kTrmmSmem, s>>>(l, n, u, ldu, j0, b);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    // 3. U = J X J, upper
    const int64_t half = (n * n + 1) / 2;
    rotate_upper_kernel<<<(unsigned)((half + 255) / 256), 256, 0, s>>>(u, ldu, n, half);
    return cudaGetLastError();
}

}  // namespace wq

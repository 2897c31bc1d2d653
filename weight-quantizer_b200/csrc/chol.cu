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
//   2. X = M^-1 by doubling: every 64 x 64 diagonal block inverted in shared
//      memory (one launch), then levels of S = 1, 2, 4, ... blocks: each pair
//      of neighbouring inverted diagonal sections A (upper) and C (lower) of
//      S blocks gets its off-diagonal part X_CA = -X_C (M_CA X_A), two batched
//      64 x 64-tile products per level over all pairs at once;
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
        // trailing triangle of the block: a 16 x 16 grid of threads over (r, c)
        for (int r = k + 1 + (tid >> 4); r < b; r += 16) {
            const double lrk = s[r][k];
            for (int c = k + 1 + (tid & 15); c <= r; c += 16) s[r][c] = s[r][c] - lrk * s[c][k];
        }
        __syncthreads();
    }
    for (int idx = tid; idx < b * b; idx += 256) {
        const int r = idx / b, c = idx % b;
        if (c <= r) l[(j0 + r) * n + j0 + c] = s[r][c];
    }
}

// Panel below the diagonal block: rows i >= j0 + b solve x L11^T = a by
// forward substitution, one warp of 32 rows per CTA, one row per lane, the
// row in shared memory.
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
    // column-oriented: once x_k is final, it updates every later x_q (those
    // updates are independent of one another)
    for (int k = 0; k < b; ++k) {
        const double xk = xs[k][lane] / ld[k][k];
        xs[k][lane] = xk;
        for (int q = k + 1; q < b; ++q) xs[q][lane] = xs[q][lane] - xk * ld[q][k];
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
                                                         double* __restrict__ x, int64_t ldx) {
    __shared__ double lp[kNB * (kNB + 1) / 2];
    __shared__ double xp[kNB * (kNB + 1) / 2];
    const int64_t j0 = (int64_t)blockIdx.x * kNB;
    const int b = (int)min((int64_t)kNB, n - j0);
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

// One doubling level of the inverse. Pair g: A = rows/columns [a0, c0), C =
// rows/columns [c0, c1) with a0 = 2 g S 64, c0 = a0 + S 64. Phase 1:
// T[i, j] = sum_k M[i, k] X[k, j] (i in C, j, k in A, k >= j's tile); phase 2:
// X[i, j] = -sum_k X[i, k] T[k, j] (i, k in C, k up to i's tile). X's
// diagonal 64-blocks hold zeros above their diagonals, and no product reads
// a block of X above the block diagonal. 64 x 64 output tiles (4 x 4 per
// thread), the k sum in order in chunks of 16.
template <bool PHASE2>
__global__ void __launch_bounds__(256) inv_level_kernel(const double* __restrict__ mm, double* __restrict__ x,
                                                        int64_t ldx, double* __restrict__ t, int64_t n, int64_t S) {
    const int64_t a0 = (int64_t)blockIdx.y * 2 * S * kT, c0 = a0 + S * kT;
    if (c0 >= n) return;
    const int64_t c1 = min(c0 + S * kT, n);
    const int64_t ti = (int64_t)blockIdx.x / S, tj = (int64_t)blockIdx.x % S;
    const int64_t i0 = c0 + ti * kT, j0 = a0 + tj * kT;
    if (i0 >= c1) return;
    __shared__ double es[kKc][kT + 1];   // [k][row]
    __shared__ double hs[kKc][kT];       // [k][col]
    const double* aop = PHASE2 ? x : mm;
    const int64_t lda = PHASE2 ? ldx : n;
    const double* bop = PHASE2 ? t : x;
    const int64_t ldb = PHASE2 ? n : ldx;
    const int64_t klo = PHASE2 ? c0 : j0;
    const int64_t khi = PHASE2 ? min(i0 + kT, c1) : c0;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    double acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[a][q] = 0.0;
    for (int64_t k0 = klo; k0 < khi; k0 += kKc) {
        for (int idx = threadIdx.x; idx < kKc * kT; idx += 256) {
            const int kk = idx % kKc, rr = idx / kKc;
            const int64_t i = i0 + rr, k = k0 + kk;
            es[kk][rr] = (i < c1 && k < khi) ? aop[i * lda + k] : 0.0;
            const int cc = idx % kT, k2 = idx / kT;
            const int64_t j = j0 + cc, kb = k0 + k2;
            hs[k2][cc] = (j < c0 && kb < khi) ? bop[kb * ldb + j] : 0.0;
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
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int64_t i = i0 + ty * 4 + a;
        if (i >= c1) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int64_t j = j0 + tx * 4 + q;
            if (j >= c0) continue;
            if constexpr (PHASE2) x[i * ldx + j] = -acc[a][q];
            else t[i * n + j] = acc[a][q];
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

// workspace: M (n x n), then the doubling levels' products T (n x n)
size_t chol_inverse_upper_workspace_bytes(int64_t n) { return 2 * (size_t)n * (size_t)n * sizeof(double); }

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
    // 2. X = M^-1 into u: diagonal blocks, then doubling levels
    const int64_t nb = (n + kNB - 1) / kNB;
    trtri_diag_kernel<<<(unsigned)nb, kNB, 0, s>>>(l, n, u, ldu);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    double* t = work + n * n;
    for (int64_t S = 1; S < nb; S *= 2) {
        const dim3 grid((unsigned)(S * S), (unsigned)((nb + 2 * S - 1) / (2 * S)));
        inv_level_kernel<false><<<grid, 256, 0, s>>>(l, u, ldu, t, n, S);
        inv_level_kernel<true><<<grid, 256, 0, s>>>(l, u, ldu, t, n, S);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    // 3. U = J X J, upper
    const int64_t half = (n * n + 1) / 2;
    rotate_upper_kernel<<<(unsigned)((half + 255) / 256), 256, 0, s>>>(u, ldu, n, half);
    return cudaGetLastError();
}

}  // namespace wq

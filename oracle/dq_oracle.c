/*
 * CPU oracle (test infrastructure only; never part of the product path).
 * See dq_oracle.h for what it restates and how it is pinned.
 *
 * Compiled with -ffp-contract=off: every fused multiply-add below is an
 * explicit fmaf() that stands for a fused multiply-add of the reference build
 * (an _mm256_fmadd_ps, or a tail product the compiler contracted), and every
 * other expression rounds after each operation, as the reference does.
 */
#include "dq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------- */
/* dequant-GEMM                                                              */
/* ------------------------------------------------------------------------- */

/* Broadcast read of a [rows, cols] table (dequant_gemm.cpp:30-34). */
static float at2(const float* a, int rows, int cols, int m, int g) {
    const int r = rows == 1 ? 0 : m;
    const int c = cols == 1 ? 0 : g;
    return a[(size_t)r * (size_t)cols + (size_t)c];
}

/* Code k of one stored row: int8 byte, or int4 nibble with even k in the low
 * nibble (dequant_gemm.cpp:49-55, pack.py:1-12). */
static int code_at(const uint8_t* row, int k, int bits) {
    if (bits == 8) return (int)row[k];
    const uint8_t byte = row[k >> 1];
    return (k & 1) == 0 ? (int)(byte & 0x0F) : (int)(byte >> 4);
}

/* One row of W_hat in fp32 (dequant_gemm.cpp:57-120). The AVX2 and scalar
 * branches there compute the same per-element expression,
 * ((float)code - zero) * scale, then * channel[k]; each op rounds. */
static void dequant_row(const uint8_t* row, int m, int K, int bits, const float* scales,
                        const float* zeros, int scale_rows, int groups, int group_size,
                        const float* channel, float* dst) {
    const int n_groups = (K + group_size - 1) / group_size;
    for (int g = 0; g < n_groups; ++g) {
        const int k0 = g * group_size;
        const int k1 = k0 + group_size < K ? k0 + group_size : K;
        const float scale = at2(scales, scale_rows, groups, m, g);
        const float zero = at2(zeros, scale_rows, groups, m, g);
        for (int k = k0; k < k1; ++k) {
            float w = ((float)code_at(row, k, bits) - zero) * scale;
            if (channel != NULL) w = w * channel[k];
            dst[k] = w;
        }
    }
}

/* Horizontal sum of 8 fp32 lanes in the order of hsum256
 * (dequant_gemm.cpp:37-46): ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7)). */
static float hsum8(const float a[8]) {
    const float l0 = a[0] + a[4], l1 = a[1] + a[5], l2 = a[2] + a[6], l3 = a[3] + a[7];
    return (l0 + l1) + (l2 + l3);
}

/* Scalar tail `s += a[k] * b[k]` as the reference's build (g++ -O3 -mavx2
 * -mfma) evaluates it: a first block of 4 elements is an in-order vectorized
 * reduction (products rounded, then added one by one), the remaining 0-3
 * elements are contracted into fused multiply-adds. */
static float tail_dot(float s, const float* a, const float* b, int k, int K, size_t stride_b) {
    if (k + 4 <= K) {
        for (int l = 0; l < 4; ++l) {
            const float p = a[k + l] * b[(size_t)(k + l) * stride_b];
            s = s + p;
        }
        k += 4;
    }
    for (; k < K; ++k) s = fmaf(a[k], b[(size_t)k * stride_b], s);
    return s;
}

/* 8-lane FMA dot product plus scalar tail (dot_scalar, dequant_gemm.cpp:122-136). */
static float dot_scalar(const float* a, const float* b, int K) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int k = 0;
    for (; k + 8 <= K; k += 8)
        for (int l = 0; l < 8; ++l) acc[l] = fmaf(a[k + l], b[k + l], acc[l]);
    return tail_dot(hsum8(acc), a, b, k, K, 1);
}

/* Four batch rows at a time, then dot_scalar for the rest
 * (dots_into, dequant_gemm.cpp:138-174). */
static void dots_into(const float* row, const float* x, float* y, int B, int M, int K, int m) {
    int b = 0;
    for (; b + 4 <= B; b += 4) {
        float acc[4][8];
        memset(acc, 0, sizeof(acc));
        int k = 0;
        for (; k + 8 <= K; k += 8)
            for (int j = 0; j < 4; ++j) {
                const float* xb = x + (size_t)(b + j) * (size_t)K;
                for (int l = 0; l < 8; ++l) acc[j][l] = fmaf(row[k + l], xb[k + l], acc[j][l]);
            }
        for (int j = 0; j < 4; ++j)
            y[(size_t)(b + j) * (size_t)M + m] =
                tail_dot(hsum8(acc[j]), row, x + (size_t)(b + j) * (size_t)K, k, K, 1);
    }
    for (; b < B; ++b) y[(size_t)b * (size_t)M + m] = dot_scalar(row, x + (size_t)b * (size_t)K, K);
}

int orc_dequant_gemm(const float* x, const uint8_t* q, const float* scales, const float* zeros,
                     const float* channel, float* y, int B, int M, int K, int scale_rows,
                     int groups, int group_size, int bits, int nthreads) {
    if ((bits != 4 && bits != 8) || group_size <= 0 || B < 0 || M < 0 || K < 0) return ORC_EINVAL;
    if (scale_rows != 1 && scale_rows != M) return ORC_EINVAL;
    if (K > 0 && groups != (K + group_size - 1) / group_size) return ORC_EINVAL;
    const int packed_cols = bits == 4 ? (K + 1) / 2 : K;
#ifdef _OPENMP
    if (nthreads < 1) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads)
#else
    (void)nthreads;
#endif
    {
        float* row = (float*)malloc(sizeof(float) * (size_t)(K > 0 ? K : 1));
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int m = 0; m < M; ++m) {
            const uint8_t* qrow = q + (size_t)m * (size_t)packed_cols;
            dequant_row(qrow, m, K, bits, scales, zeros, scale_rows, groups, group_size, channel, row);
            dots_into(row, x, y, B, M, K, m);
        }
        free(row);
    }
    return ORC_OK;
}

/* ------------------------------------------------------------------------- */
/* RTN quantize + pack                                                       */
/* ------------------------------------------------------------------------- */

/* Block statistics of qparams (quant.py:146-172) over the elements
 * w[r * ld + k] for r in [r0, r1), k in [k0, k1), scanned in row-major order.
 * The min scan keeps the first of equal values (strict <), so a block whose
 * smallest value is a zero takes the sign of its first zero; torch's CPU
 * reduction does the same for narrow blocks. */
static void qparams_block(const float* w, size_t ld, int r0, int r1, int k0, int k1, int symmetric,
                          int bits, float* scale_out, float* zero_out) {
    const int qmax = (1 << bits) - 1;
    if (symmetric) {
        float amax = 0.0f;
        int first = 1;
        for (int r = r0; r < r1; ++r)
            for (int k = k0; k < k1; ++k) {
                const float a = fabsf(w[(size_t)r * ld + (size_t)k]);
                if (first || a > amax) amax = a;
                first = 0;
            }
        /* torch.where(amax > 0, (2 * amax) / qmax, 1) */
        *scale_out = amax > 0.0f ? (2.0f * amax) / (float)qmax : 1.0f;
        *zero_out = (float)(qmax + 1) / 2.0f;
        return;
    }
    float xmin = 0.0f, xmax = 0.0f;
    int first = 1;
    for (int r = r0; r < r1; ++r)
        for (int k = k0; k < k1; ++k) {
            const float v = w[(size_t)r * ld + (size_t)k];
            if (first) {
                xmin = v;
                xmax = v;
                first = 0;
            } else {
                if (v < xmin) xmin = v;
                if (v > xmax) xmax = v;
            }
        }
    /* torch.minimum(xmin, 0) keeps a -0.0 minimum; torch.maximum(xmax, 0). */
    if (xmin > 0.0f) xmin = 0.0f;
    if (xmax < 0.0f) xmax = 0.0f;
    if (xmin == 0.0f && xmax == 0.0f) {
        xmin = -1.0f;
        xmax = 1.0f;
    }
    float scale = (xmax - xmin) / (float)qmax;
    if (!(scale > 0.0f)) scale = 1.0f;
    float zero = rintf(-xmin / scale);
    /* torch.clamp(zero, 0, qmax): a -0.0 stays -0.0 */
    if (zero < 0.0f) zero = 0.0f;
    if (zero > (float)qmax) zero = (float)qmax;
    *scale_out = scale;
    *zero_out = zero;
}

/* integer_codes (quant.py:175-184): clamp(round(w / scale) + zero, 0, qmax). */
static int32_t code_of(float v, float scale, float zero, int qmax) {
    float q = rintf(v / scale) + zero;
    if (q < 0.0f) q = 0.0f;
    if (q > (float)qmax) q = (float)qmax;
    return (int32_t)rintf(q);
}

int orc_rtn_quantize(const float* w, const float* pre_scale, int M, int K, int bits,
                     int symmetric, int group_mode, int32_t* codes, float* scales,
                     float* zeros, float* channel_out) {
    if ((bits != 4 && bits != 8) || M < 0 || K < 0 || group_mode < -1) return ORC_EINVAL;
    const size_t n = (size_t)M * (size_t)K;
    /* quant.py:239-241 */
    for (size_t i = 0; i < n; ++i)
        if (!isfinite(w[i])) return ORC_ENONFINITE;
    const float* src = w;
    float* folded = NULL;
    if (pre_scale != NULL) {
        /* quant.py:242-250: w * s, stored channel = 1 / s */
        for (int k = 0; k < K; ++k)
            if (!isfinite(pre_scale[k]) || pre_scale[k] <= 0.0f) return ORC_EPRESCALE;
        folded = (float*)malloc(sizeof(float) * (n > 0 ? n : 1));
        for (int m = 0; m < M; ++m)
            for (int k = 0; k < K; ++k)
                folded[(size_t)m * K + k] = w[(size_t)m * K + k] * pre_scale[k];
        if (channel_out != NULL)
            for (int k = 0; k < K; ++k) channel_out[k] = 1.0f / pre_scale[k];
        src = folded;
    }
    const int qmax = (1 << bits) - 1;
    if (group_mode == 0) {
        /* per-tensor: qparams(w.reshape(1, -1)) */
        float s, z;
        qparams_block(src, (size_t)K, 0, M, 0, K, symmetric, bits, &s, &z);
        scales[0] = s;
        zeros[0] = z;
        for (size_t i = 0; i < n; ++i) codes[i] = code_of(src[i], s, z, qmax);
    } else {
        const int gs = group_mode < 0 ? (K > 0 ? K : 1) : group_mode;
        const int groups = group_mode < 0 ? 1 : (K + gs - 1) / gs;
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
        for (int m = 0; m < M; ++m)
            for (int g = 0; g < groups; ++g) {
                const int k0 = g * gs;
                const int k1 = k0 + gs < K ? k0 + gs : K;
                float s, z;
                qparams_block(src, (size_t)K, m, m + 1, k0, k1, symmetric, bits, &s, &z);
                scales[(size_t)m * groups + g] = s;
                zeros[(size_t)m * groups + g] = z;
                for (int k = k0; k < k1; ++k)
                    codes[(size_t)m * K + k] = code_of(src[(size_t)m * K + k], s, z, qmax);
            }
    }
    free(folded);
    return ORC_OK;
}

int orc_pack_int4(const int32_t* codes, int M, int K, uint8_t* packed) {
    const int cols = (K + 1) / 2;
    for (size_t i = 0; i < (size_t)M * (size_t)K; ++i)
        if (codes[i] < 0 || codes[i] > 15) return ORC_EINVAL;
    for (int m = 0; m < M; ++m)
        for (int j = 0; j < cols; ++j) {
            const int lo = codes[(size_t)m * K + 2 * j] & 0x0F;
            const int hi = 2 * j + 1 < K ? codes[(size_t)m * K + 2 * j + 1] & 0x0F : 0;
            packed[(size_t)m * cols + j] = (uint8_t)(lo | (hi << 4));
        }
    return ORC_OK;
}

void orc_unpack_int4(const uint8_t* packed, int M, int K, uint8_t* codes) {
    const int cols = (K + 1) / 2;
    for (int m = 0; m < M; ++m)
        for (int k = 0; k < K; ++k) {
            const uint8_t byte = packed[(size_t)m * cols + (k >> 1)];
            codes[(size_t)m * K + k] = (k & 1) == 0 ? (uint8_t)(byte & 0x0F) : (uint8_t)(byte >> 4);
        }
}

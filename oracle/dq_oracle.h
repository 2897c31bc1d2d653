/*
 * CPU oracle for the dequant-GEMM hot path and its RTN quantize+pack producer.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is
 * compared against; the product never links, loads or calls it. Only the test
 * suite, the smoke check and the benchmark's CPU-baseline leg use it.
 *
 * It restates, in plain C, the algorithm of ptqkit (cvs0/weight-quantizer):
 *   - orc_dequant_gemm  : src/ptqkit/csrc/dequant_gemm.cpp:57-218 (AVX2 build),
 *                         with the reference's exact fp32 operation order, so its
 *                         output is bitwise equal to the reference kernel's.
 *   - orc_rtn_quantize  : src/ptqkit/quant.py:146-184 (qparams, integer_codes)
 *                         and :225-289 (quantize_weight).
 *   - orc_pack_int4 / orc_unpack_int4 : src/ptqkit/pack.py:17-55.
 *
 * Pinning: tests/golden/ holds outputs of the reference itself (its Python RTN and
 * its compiled C++ kernel) on seeded inputs; the CPU test suite checks this
 * oracle against them bit for bit.
 */
#ifndef DQ_ORACLE_H
#define DQ_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (0 = ok). */
#define ORC_OK 0
#define ORC_EINVAL 1
#define ORC_ENONFINITE 2
#define ORC_EPRESCALE 3

/* y[b, m] = sum_k scale[m, g] * (code[m, k] - zero[m, g]) * channel[k] * x[b, k].
 * x [B, K] fp32; q uint8 [M, K] (bits 8) or [M, (K+1)/2] (bits 4);
 * scales/zeros fp32 [scale_rows, groups]; channel fp32 [K] or NULL; y [B, M].
 * nthreads <= 0 uses the OpenMP default; the result does not depend on it. */
int orc_dequant_gemm(const float* x, const uint8_t* q, const float* scales, const float* zeros,
                     const float* channel, float* y, int B, int M, int K, int scale_rows,
                     int groups, int group_size, int bits, int nthreads);

/* Round-to-nearest quantization of w [M, K] (fp32).
 * group_mode: > 0 group size along K, 0 per-tensor, -1 per-channel.
 * pre_scale [K] or NULL: quantizes w * pre_scale and writes 1 / pre_scale to
 * channel_out [K] (channel_out may be NULL when pre_scale is NULL).
 * codes int32 [M, K]; scales/zeros fp32 [rows, groups] where rows = 1 for
 * per-tensor else M, groups = 1 for tensor/channel else ceil(K / group_mode). */
int orc_rtn_quantize(const float* w, const float* pre_scale, int M, int K, int bits,
                     int symmetric, int group_mode, int32_t* codes, float* scales,
                     float* zeros, float* channel_out);

/* codes int32 [M, K] in [0, 15] -> packed uint8 [M, (K+1)/2]; odd K pads a 0 code. */
int orc_pack_int4(const int32_t* codes, int M, int K, uint8_t* packed);
/* packed uint8 [M, (K+1)/2] -> codes uint8 [M, K]; the pad nibble is dropped. */
void orc_unpack_int4(const uint8_t* packed, int M, int K, uint8_t* codes);

#ifdef __cplusplus
}
#endif
#endif

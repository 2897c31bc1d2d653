// Internal launch interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace wq {

// One dequant-GEMM problem in ptqkit's storage layout (see include/wq_b200.h).
struct GemmProblem {
    const float* x;        // [B, K]
    const uint8_t* q;      // [M, q_stride] bytes
    const float* scales;   // [scale_rows, groups]
    const float* zeros;    // [scale_rows, groups]
    const float* channel;  // [K] or nullptr
    float* y;              // [B, ldy]
    float* y_extra[7];     // further outputs with y's layout (peer-mapped or local)
    int n_extra;           // entries of y_extra in use
    float* y_all;          // NVLink-switch address reaching every rank's y, or nullptr
    const float* bias;     // [M] added to every output row, or nullptr
    int64_t B, M, K;
    int64_t q_stride;      // bytes per stored row: K (int8) or (K+1)/2 (int4)
    int64_t ldy;
    int scale_rows, groups, group_size, bits;
};

// --- K1: streaming decode kernel (small batch, weight-stream bound) --------
// Batches up to 4; the C ABI sends batches 3-4 to K1w first when it applies.
constexpr int kGemvMaxBatch = 4;
// Workspace the decode path needs for this problem (0 if it does not apply).
size_t gemv_workspace_bytes(int64_t B, int64_t K, int bits);
// True when the decode kernel can run this problem (alignment, group shape,
// batch, shared-memory fit).
bool gemv_supported(const GemmProblem& p);
cudaError_t launch_gemv(const GemmProblem& p, void* workspace, cudaStream_t s);
// int4 codes at batches 1-2 on the integer tensor-core path (mma.sync
// m16n8k32 u8 x s8: codes widened to bytes, x' as three signed base-256
// digits), when groups are multiples of 64 (or one group), K <= 8192 and the
// tables can be bulk-copied; launch_gemv routes these problems to it, and
// batches 3-4 that K1w does not take as two launches.
bool gemv_imma_supported(const GemmProblem& p);
cudaError_t launch_gemv_imma(const GemmProblem& p, cudaStream_t s);

// --- K1w: batches 3-32 on the integer tensor-core path ----------------------
// int4 (groups a multiple of 64, or one group) and int8 (groups a multiple of
// 64, or one group) codes with 16-byte aligned code rows: x' as three signed
// base-256 digits per fold block, written by a prep kernel in the order the
// MMA fragments read them; the weight is cut into units of 256 rows x one
// fold block and every CTA takes an equal contiguous run of units
// (stream-K), partial rows summed in a fixed order by the last CTA to arrive.
// Above 16 batch rows it takes only layers of at least 2^25 codes (smaller
// ones run faster on the tcgen05 kernel with split-K).
// Workspace: the digit records, the partial rows, one counter per row block.
constexpr int kWideMinBatch = 3;
constexpr int kWideMaxBatch = 32;
bool wide_supported(const GemmProblem& p);
size_t wide_workspace_bytes(int64_t B, int64_t M, int64_t K, int group_size, int bits);
cudaError_t launch_wide(const GemmProblem& p, void* workspace, cudaStream_t s);

// --- K2: tcgen05/TMEM tensor-core kernel (batches above 32, and 5-32 where K1w does not run)
// Applies when rows are 16-byte aligned and groups are multiples of 64 (or a
// single group). Workspace: the fp16 hi/lo planes of x', 1/S_b, the
// per-group sums of x' (for zero points that are not integers) and, when
// the output tiles are too few to fill the GPU, split-K partial tiles and
// arrival counters.
bool tc_supported(const GemmProblem& p);
size_t tc_workspace_bytes(int64_t B, int64_t M, int64_t K, int group_size, int bits);
cudaError_t launch_tc(const GemmProblem& p, void* workspace, cudaStream_t s);

// --- generic tiled SIMT kernel: any shape, reference per-element formula ---
cudaError_t launch_gemm_simt(const GemmProblem& p, cudaStream_t s);

// --- y for K == 0: zeros, or the bias in every row ---------------------------
cudaError_t launch_fill_zero(float* y, int64_t B, int64_t M, int64_t ldy, cudaStream_t s);
cudaError_t launch_fill_bias(float* y, int64_t B, int64_t M, int64_t ldy, const float* bias, cudaStream_t s);

// --- RTN quantize + pack -----------------------------------------------------
struct RtnProblem {
    const float* w;          // [M, K]
    const float* pre_scale;  // [K] or nullptr
    int64_t M, K;
    int bits, symmetric, group_mode;  // group_mode: >0 group, 0 tensor, -1 channel
    uint8_t* q_out;
    float* scales_out;
    float* zeros_out;
    float* channel_out;
    int32_t* flags;
};
size_t rtn_workspace_bytes(int64_t M, int64_t K, int group_mode);
cudaError_t launch_rtn(const RtnProblem& p, void* workspace, cudaStream_t s);

cudaError_t launch_pack_int4(const int32_t* codes, int64_t M, int64_t K, uint8_t* packed,
                             int32_t* minmax, cudaStream_t s);
cudaError_t launch_unpack_int4(const uint8_t* packed, int64_t M, int64_t packed_cols, int64_t K,
                               uint8_t* codes, cudaStream_t s);
cudaError_t launch_dequantize(const uint8_t* q, int64_t M, int64_t K, int64_t q_stride,
                              const float* scales, int scale_rows, int groups,
                              const float* zeros, const float* channel, int group_size, int bits,
                              float* w_out, cudaStream_t s);
cudaError_t launch_gather_permute(const float* src, int64_t P, int64_t B, int64_t Mp, float* dst,
                                  cudaStream_t s);

// --- compressed format: fp16 payload <-> fp32 kernel arrays ----------------
cudaError_t launch_widen_f16_f32(const uint16_t* src, float* dst, int64_t n, cudaStream_t s);
cudaError_t launch_narrow_f32_f16(const float* src, uint16_t* dst, int64_t n, cudaStream_t s);

// --- AWQ search reductions (awq.cu) ----------------------------------------
cudaError_t launch_channel_abs_sum(const float* x, int64_t n, int64_t K, int64_t ldx, double* acc, cudaStream_t s);
cudaError_t launch_pre_scale(const float* mag, int64_t K, float alpha, float* pre, cudaStream_t s);
size_t sq_err_workspace_bytes();
cudaError_t launch_sq_err_sum(const float* a, const float* b, int64_t n, double* out, void* workspace,
                              cudaStream_t s);

// --- GPTQ column sweep (gptq.cu) ----------------------------------------------
size_t gptq_qparams_workspace_bytes(int64_t rows);
cudaError_t launch_gptq_qparams(const double* w, int64_t rows, int64_t ld, int64_t c0, int64_t c1, int bits,
                                int symmetric, int per_tensor, double* scale_out, double* zero_out,
                                int64_t out_stride, double* workspace, cudaStream_t s);
int gptq_max_block();
cudaError_t launch_gptq_block(const double* w, int64_t rows, int64_t ld, const double* hinv, int64_t ldh,
                              int64_t s0, int count, const double* scale, const double* zero, int64_t qp_stride,
                              int bits, int32_t* codes, int64_t ldc, double* err_block, const uint8_t* zero_err,
                              int* bad_col, cudaStream_t s);
// upper Cholesky factor of an inverse (chol.cu)
size_t chol_inverse_upper_workspace_bytes(int64_t n);
cudaError_t launch_chol_inverse_upper(const double* a, int64_t n, int64_t lda, double* u, int64_t ldu,
                                      double* work, int* info, cudaStream_t s);
cudaError_t launch_gptq_tail(double* work, int64_t rows, int64_t ld, int64_t c0, int64_t ncols, const double* err,
                             int count, const double* hinv, int64_t ldh, int64_t s0, cudaStream_t s);

// Number of SMs of the current device (cached per device).
int sm_count();

// cuTensorMapEncodeTiled from the driver (nullptr if unavailable), and a 2D
// map over a row-major array: `inner` elements per row, `outer` rows,
// `row_bytes` apart, boxes of box_inner x box_outer.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn();
bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz);

// Device address (current device) of the library's fault word: kernels OR in
// 1 when a bounded pipeline mbarrier wait expires. nullptr if the symbol
// cannot be resolved.
unsigned int* fault_word();

}  // namespace wq

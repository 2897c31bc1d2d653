/*
 * wq_b200 — C ABI of the B200 (sm_100a) dequant-GEMM and RTN quantize+pack path.
 *
 * Drop-in replacement for the native kernel of ptqkit (cvs0/weight-quantizer),
 * the pybind11 module `ptqkit._kernels` built from src/ptqkit/csrc/dequant_gemm.cpp,
 * plus device versions of its RTN producer (src/ptqkit/quant.py) and int4 packing
 * (src/ptqkit/pack.py). Storage layouts are ptqkit's, byte for byte:
 *
 *   x        fp32  [B, K]                      row-major activations
 *   q        uint8 [M, K]          (bits 8)    one code per byte
 *            uint8 [M, (K+1)/2]    (bits 4)    code 2j in the low nibble of byte j,
 *                                              code 2j+1 in the high nibble; odd K
 *                                              pads a zero nibble that is never read
 *   scales   fp32  [scale_rows, groups]        scale_rows in {1, M}, groups = ceil(K/G)
 *   zeros    fp32  [scale_rows, groups]
 *   channel  fp32  [K] or absent               AWQ channel scale (stored 1/s)
 *   y        fp32  [B, M]
 *
 *   y[b, m] = sum_k scale[m, g] * (q[m, k] - zero[m, g]) * channel[k] * x[b, k],  g = k / G
 *
 * Conventions
 *   - All data pointers are DEVICE pointers of the current CUDA device. They are
 *     borrowed, never freed. Shapes are element counts.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     Work is enqueued on it; no entry point synchronizes the host.
 *   - Every entry point returns 0 (WQ_OK) or a WQ_E_* status; wq_status_string()
 *     gives the message. Argument errors are detected on the host before any
 *     launch and use the reference's own messages where it has one.
 *   - Results are deterministic: the same inputs and shapes give the same bits
 *     on every call (no atomics in any reduction).
 */
#ifndef WQ_B200_H
#define WQ_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define WQ_API __attribute__((visibility("default")))
#else
#define WQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum wq_status {
    WQ_OK = 0,
    WQ_E_X_SHAPE = 1,        /* "x must have shape [B, K]" (dequant_gemm.cpp:235-237) */
    WQ_E_RANK = 2,           /* "q, scales, and zeros must be rank 2" (:238-240) */
    WQ_E_BITS = 3,           /* "bits must be 4 or 8" (:241-243) */
    WQ_E_GROUP_SIZE = 4,     /* "group_size must be positive" (:244-246) */
    WQ_E_NEG_DIM = 5,        /* "negative dimension" (:252-254) */
    WQ_E_PACKED_COLS = 6,    /* "packed code row length does not match K" (:255-258) */
    WQ_E_ZEROS_SHAPE = 7,    /* "zeros shape must match scales" (:259-261) */
    WQ_E_SCALE_ROWS = 8,     /* "scale rows must be 1 or M" (:262-264) */
    WQ_E_SCALE_GROUPS = 9,   /* "scale groups must equal ceil(K / group_size)" (:265-268) */
    WQ_E_CHANNEL_SHAPE = 10, /* "channel_scale must have shape [K]" (:271-276) */
    WQ_E_NULL = 11,          /* a required pointer is NULL */
    WQ_E_WORKSPACE = 12,     /* workspace smaller than the *_workspace_bytes() query */
    WQ_E_TOO_LARGE = 13,     /* a dimension is beyond what the kernels index */
    WQ_E_CUDA = 14,          /* a CUDA call failed; wq_last_cuda_error() has the text */
    WQ_E_NOT_FINITE = 15,    /* "weight must be finite" (quant.py:240-241) */
    WQ_E_PRE_SCALE_LEN = 16, /* "pre_scale must have one entry per input channel" (quant.py:245-246) */
    WQ_E_PRE_SCALE_VAL = 17, /* "pre_scale must be finite and positive" (quant.py:247-248) */
    WQ_E_INT4_RANGE = 18,    /* "int4 codes must lie in [0, 15]" (pack.py:22-26) */
    WQ_E_GROUP_MODE = 19,    /* "group_size must be None, 0, or positive" (quant.py:75-76) */
    WQ_E_LD = 20,            /* output row stride smaller than the row length */
    WQ_E_NOALLOC_LIMIT = 21, /* problem needs more scratch than wq_dequant_gemm_f32_noalloc holds */
    WQ_E_OUTPUTS = 22        /* output count outside [1, WQ_MAX_OUTPUTS] */
};

/* Message for a status code (static storage; never NULL). */
WQ_API const char* wq_status_string(int status);
/* Text of the last CUDA error seen by this library on the calling thread. */
WQ_API const char* wq_last_cuda_error(void);

/* Fault word of the current device. Bit 0: a bounded wait on a pipeline
 * barrier expired (the launch then completed without waiting again, and its
 * output is not valid). Other bits are reserved and stay 0. Synchronizes with
 * the device. `reset` nonzero clears the word after reading it. No
 * counterpart in the reference, whose CPU kernel has no asynchronous waits. */
WQ_API int wq_fault_status(int reset, uint32_t* out);

/* Self-test of the fault reporting: one thread initializes a shared-memory
 * barrier that nothing ever arrives on and waits for it with the library's
 * bounded wait, giving up after `max_polls` polls (1 <= max_polls <= 2^22).
 * When the wait gives up, bit 0 of the fault word is set, exactly as when a
 * pipeline wait of a real kernel expires; nothing else is touched and no copy
 * is in flight. Enqueued on `stream`. No counterpart in the reference. */
WQ_API int wq_selftest_expired_wait(uint32_t max_polls, void* stream);

/* Build/device facts, the counterpart of `_kernels.kernel_info()`
 * (dequant_gemm.cpp:302-315, which reports {"avx2", "openmp"}). */
typedef struct wq_kernel_info_t {
    int abi_version;       /* WQ_ABI_VERSION of the library */
    int compiled_sm;       /* 100 for sm_100a */
    int device;            /* device queried */
    int device_cc;         /* major*10 + minor of that device */
    int sm_count;          /* multiprocessors on that device */
    int tcgen05;           /* 1 if the tcgen05 tensor-core path is built in */
    char device_name[96];
} wq_kernel_info_t;
#define WQ_ABI_VERSION 1
WQ_API int wq_kernel_info(int device, wq_kernel_info_t* out);

/* ------------------------------------------------------------------------ */
/* Dequant-GEMM: replaces `_kernels.dequant_gemm(x, q, scales, zeros,        */
/* channel_scale, group_size, bits, nthreads)` (dequant_gemm.cpp:222-300,    */
/* _kernels.pyi:3-12). `nthreads` has no counterpart: the launch shape is    */
/* chosen from the problem. The array shapes are passed so that the same     */
/* validation as the reference runs here (q is [M, q_cols], scales is        */
/* [scale_rows, groups], zeros is [zero_rows, zero_groups], channel_scale is */
/* [channel_len] or NULL with channel_len = -1). y is [B, M] with row        */
/* stride ldy >= M elements (ldy = M for a dense output).                    */
/* ------------------------------------------------------------------------ */
WQ_API size_t wq_dequant_gemm_workspace_bytes(int64_t B, int64_t M, int64_t K, int group_size, int bits);

WQ_API int wq_dequant_gemm_f32(const float* x, int64_t B, int64_t K,
                        const uint8_t* q, int64_t M, int64_t q_cols,
                        const float* scales, int64_t scale_rows, int64_t groups,
                        const float* zeros, int64_t zero_rows, int64_t zero_groups,
                        const float* channel_scale, int64_t channel_len,
                        int group_size, int bits,
                        float* y, int64_t ldy,
                        void* workspace, size_t workspace_bytes,
                        void* stream);

/* Same computation as wq_dequant_gemm_f32, for callers that cannot allocate
 * device memory where they run the layer (a server that reserves all device
 * memory at start-up and forbids allocation on its request path, or a runtime
 * that only holds the buffers its caller gives it). No counterpart in the
 * reference, whose CPU kernel allocates its output itself.
 *
 * Instead of a caller-provided workspace it uses one static scratch array of
 * 32 MiB (33554432 bytes) inside the library; every GPU that
 * loads the library holds that array until the process exits. It allocates
 * nothing. A problem whose wq_dequant_gemm_workspace_bytes() exceeds the array
 * returns WQ_E_NOALLOC_LIMIT (about 4 * B * K bytes are needed on the
 * tensor-core path: for K = 8192, up to 896 batch rows). All calls on a
 * device share the array and every call writes the scratch it reads before
 * reading it, but calls whose work overlaps on the GPU race on it. The first
 * call on each device resolves the array's device address
 * (cudaGetSymbolAddress); make it before capturing a stream. The address is
 * kept per device and CUDA context, so after a cudaDeviceReset the next call
 * resolves it again. */
WQ_API int wq_dequant_gemm_f32_noalloc(const float* x, int64_t B, int64_t K,
                                       const uint8_t* q, int64_t M, int64_t q_cols,
                                       const float* scales, int64_t scale_rows, int64_t groups,
                                       const float* zeros, int64_t zero_rows, int64_t zero_groups,
                                       const float* channel_scale, int64_t channel_len,
                                       int group_size, int bits,
                                       float* y, int64_t ldy,
                                       void* stream);

/* ------------------------------------------------------------------------ */
/* RTN quantize + pack: replaces `quantize_weight(weight, config,            */
/* pre_scale=)` (quant.py:225-289) up to and including assemble_quantized's  */
/* packing (quant.py:187-222, pack.py:17-33), bit for bit.                   */
/*   w          fp32 [M, K] device                                           */
/*   pre_scale  fp32 [K] or NULL (AWQ fold: quantizes w*s, writes 1/s)       */
/*   group_mode > 0: group size; 0: per-tensor; -1: per-channel (None)       */
/*   q_out      uint8 [M, (K+1)/2] (bits 4) or [M, K] (bits 8)               */
/*   scales_out, zeros_out fp32 [rows, groups]: rows = 1 (tensor) or M,      */
/*              groups = 1 (tensor/channel) or ceil(K / group_mode)          */
/*   channel_out fp32 [K] (required iff pre_scale != NULL)                   */
/*   flags      int32 [1] device word; the call zeroes it, and the kernels   */
/*              OR in 1 (non-finite weight) or 2 (bad pre_scale). The caller */
/*              reads it after the stream completes; nonzero means the       */
/*              outputs are not valid (wq_rtn_flags_status maps it).         */
/* ------------------------------------------------------------------------ */
WQ_API size_t wq_rtn_workspace_bytes(int64_t M, int64_t K, int group_mode);
WQ_API int wq_rtn_quantize_f32(const float* w, const float* pre_scale, int64_t M, int64_t K,
                        int bits, int symmetric, int group_mode,
                        uint8_t* q_out, float* scales_out, float* zeros_out,
                        float* channel_out, int32_t* flags,
                        void* workspace, size_t workspace_bytes, void* stream);
/* WQ_OK for flags == 0, else the status of the first condition set. */
WQ_API int wq_rtn_flags_status(int32_t flags);

/* int4 packing (pack.py:17-33): codes int32 [M, K] -> packed uint8 [M, (K+1)/2].
 * Range errors are reported through `minmax` (int32 [2] device: the call
 * writes min and max of the codes; the caller raises WQ_E_INT4_RANGE if they
 * fall outside [0, 15], as pack_int4 does). */
WQ_API int wq_pack_int4(const int32_t* codes, int64_t M, int64_t K, uint8_t* packed,
                 int32_t* minmax, void* stream);
/* int4 unpacking (pack.py:36-55): packed uint8 [M, packed_cols] -> codes uint8 [M, K]. */
WQ_API int wq_unpack_int4(const uint8_t* packed, int64_t M, int64_t packed_cols, int64_t K,
                   uint8_t* codes, void* stream);

/* Dense reconstruction W_hat fp32 [M, K] (quant.py:292-308, the operand of
 * the reference's `impl="reference"` matmul, gemm.py:41-42). */
WQ_API int wq_dequantize_f32(const uint8_t* q, int64_t M, int64_t K, int64_t q_cols,
                      const float* scales, int64_t scale_rows, int64_t groups,
                      const float* zeros, const float* channel_scale,
                      int group_size, int bits, float* w_out, void* stream);

/* Row-major [P, B, Mp] -> [B, P*Mp] permute, used after an all-gather of
 * row-sharded outputs (each of P ranks produced y[:, p*Mp:(p+1)*Mp]). */
WQ_API int wq_gather_permute_f32(const float* src, int64_t P, int64_t B, int64_t Mp,
                          float* dst, void* stream);

/* ------------------------------------------------------------------------ */
/* Compressed format (version 1, src/ptqkit/convert.py:296-336): codes are   */
/* stored as they are; scales, zeros and the channel scale in fp16. ptqkit   */
/* has no loader; these two passes serve this library's loader (one upload  */
/* of every layer's fp16 payload, widened in one launch into the fp32        */
/* arrays the dequant-GEMM reads) and its writer.                            */
/* ------------------------------------------------------------------------ */
/* dst[i] = (float)src[i] for n fp16 values (exact). */
WQ_API int wq_widen_f16_f32(const uint16_t* src, float* dst, int64_t n, void* stream);
/* dst[i] = fp16(src[i]), round to nearest even, overflow to infinity: the
 * `.to(dtype=torch.float16)` of compressed_state (convert.py:318-323). */
WQ_API int wq_narrow_f32_f16(const float* src, uint16_t* dst, int64_t n, void* stream);

/* ------------------------------------------------------------------------ */
/* AWQ alpha search (src/ptqkit/awq.py:39-81) and its calibration statistic  */
/* (src/ptqkit/convert.py:35-63). The search quantizes W diag(s) with        */
/* wq_rtn_quantize_f32 and scores it with wq_dequant_gemm_f32; these are the */
/* reductions around them. All are deterministic (fixed summation order).    */
/* ------------------------------------------------------------------------ */
/* acc[k] += sum_i |x[i, k]| over the n rows of x (fp32, row stride ldx      */
/* >= K), summed in fp64 in row order: ActivationStats.update's               */
/* x64.abs().sum(dim=0) (convert.py:47-48); divided by n it is awq.py:61's    */
/* activations.abs().mean(dim=0). acc is fp64 [K] on the device.             */
WQ_API int wq_channel_abs_sum_f64(const float* x, int64_t n, int64_t K, int64_t ldx, double* acc, void* stream);
/* pre[k] = mag[k]^alpha / max(mean_j mag[j]^alpha, 1e-8) (awq.py:70-74, mag */
/* already clamped to >= 1e-8 by the caller as awq.py:61-65 does); alpha = 0 */
/* writes 1 (awq.py:68-69). The mean is taken in fp64 and rounded to fp32.    */
WQ_API int wq_awq_pre_scale_f32(const float* mag, int64_t K, float alpha, float* pre, void* stream);
/* out[0] = sum_i (a[i] - b[i])^2 over n fp32 values, in fp64: the numerator */
/* of awq.py:76-77's err.square().mean(). workspace: device memory of        */
/* wq_sq_err_workspace_bytes() bytes.                                         */
WQ_API size_t wq_sq_err_workspace_bytes(void);
WQ_API int wq_sq_err_sum_f64(const float* a, const float* b, int64_t n, double* out,
                             void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* GPTQ column sweep (src/ptqkit/gptq.py:86-191), fp64. The caller factors   */
/* the damped inverse Hessian (gptq.py:44-71); these are the per-row sweep   */
/* and each block's update of the later columns (gptq.py:124-125).           */
/* ------------------------------------------------------------------------ */
/* Grid of quant.py:146-172 in fp64 over columns [c0, c1) of w (fp64 [rows,  */
/* ld]): per row (per_tensor = 0; scale_out/zero_out[r * out_stride]) or for */
/* the whole range of every row (per_tensor = 1; one value at [0]). The      */
/* workspace (per_tensor only) holds wq_gptq_qparams_workspace_bytes(rows).   */
WQ_API size_t wq_gptq_qparams_workspace_bytes(int64_t rows);
WQ_API int wq_gptq_qparams_f64(const double* w, int64_t rows, int64_t ld, int64_t c0, int64_t c1,
                               int bits, int symmetric, int per_tensor,
                               double* scale_out, double* zero_out, int64_t out_stride,
                               void* workspace, size_t workspace_bytes, void* stream);
/* One block of _obs_block (gptq.py:86-125) without its last line: columns   */
/* [s0, s0 + count) of every row of w are quantized left to right with the   */
/* row's scale/zero (scale[r * qp_stride]; qp_stride 0 = one pair for all    */
/* rows), each column's OBS error corrects the block's later columns with    */
/* U = hinv (fp64 [K, ldh], upper Cholesky factor of the damped inverse), in */
/* the reference's operation order. Writes int32 codes[r * ldc + s0 + i] and  */
/* the errors err_block (fp64 [rows, count]); w is read only. count <= 128.   */
/* zero_err (uint8 [count] or NULL): columns whose error is taken as 0 for    */
/* every row, as _obs_block does when a column's error is not finite          */
/* (gptq.py:114-115). bad_col (int32 device word or NULL; the caller sets it  */
/* to INT32_MAX): receives the first column, not masked, whose error is not   */
/* finite in some row; the caller then sweeps the block again with that       */
/* column masked.                                                             */
WQ_API int wq_gptq_block_f64(const double* w, int64_t rows, int64_t ld, const double* hinv, int64_t ldh,
                             int64_t s0, int count, const double* scale, const double* zero, int64_t qp_stride,
                             int bits, int32_t* codes, int64_t ldc, double* err_block, const uint8_t* zero_err,
                             int32_t* bad_col, void* stream);
/* The tail update after one block (gptq.py:124-125), fp64:                   */
/* w[r, c0 + j] -= sum_i err_block[r, i] * hinv[s0 + i, c0 + j] for j < ncols,  */
/* i < count; the sum in i order, then one subtraction.                       */
WQ_API int wq_gptq_tail_f64(double* w, int64_t rows, int64_t ld, int64_t c0, int64_t ncols,
                            const double* err_block, int count, const double* hinv, int64_t ldh, int64_t s0,
                            void* stream);

/* Upper Cholesky factor of the inverse of a symmetric positive definite     */
/* matrix: U with U^T U = A^-1, the factor the sweep above reads (replaces    */
/* the torch.linalg.cholesky, cholesky_inverse and upper cholesky calls of    */
/* src/ptqkit/gptq.py:59-66). A fp64 [n, lda] device (only the upper triangle */
/* is read), U fp64 [n, ldu] device (zeros below the diagonal), workspace of  */
/* wq_chol_inverse_upper_workspace_bytes(n). info (int32 device word): the    */
/* call sets it to 0, and to 1 + a column index when a pivot is not positive  */
/* and finite (A not numerically positive definite; U is then not valid).     */
/* U = J M^-1 J with M M^T = J A J (J reverses rows and columns): one blocked */
/* factorization and one blocked triangular inverse, all on this library's    */
/* kernels; the caller reads info after the stream completes.                 */
WQ_API size_t wq_chol_inverse_upper_workspace_bytes(int64_t n);
WQ_API int wq_chol_inverse_upper_f64(const double* a, int64_t n, int64_t lda, double* u, int64_t ldu,
                                     void* workspace, size_t workspace_bytes, int32_t* info, void* stream);

/* ------------------------------------------------------------------------ */
/* Row-sharded layers across the GPUs of one node. No counterpart in ptqkit, */
/* whose kernel runs on one CPU and splits rows across OpenMP threads        */
/* (dequant_gemm.cpp:196-205). Each rank computes its rows of y; the         */
/* tensor-core kernel's epilogue stores every finished value into the full   */
/* y buffer of every rank (its own and its peers', mapped with the IPC calls */
/* below), so the exchange over NVLink overlaps the computation and no       */
/* gather or permute pass follows. The caller orders the ranks around the    */
/* call (every rank done reading its y before any rank starts, and every     */
/* rank's call complete before y is read), e.g. with a one-element NCCL      */
/* all-reduce on each side of it.                                            */
/* ------------------------------------------------------------------------ */
#define WQ_MAX_OUTPUTS 8

/* Bytes of an IPC handle (cudaIpcMemHandle_t). */
WQ_API size_t wq_ipc_handle_bytes(void);
/* Handle of the device allocation that contains `ptr`, and ptr's byte offset
 * inside that allocation (caching allocators hand out interior pointers). */
WQ_API int wq_ipc_get_handle(const void* ptr, void* handle_out, int64_t* offset_out);
/* Maps another process's allocation into this one (peer access enabled
 * lazily); *ptr_out = mapped base + offset. */
WQ_API int wq_ipc_open_handle(const void* handle, int64_t offset, void** ptr_out);
/* Unmaps a pointer returned by wq_ipc_open_handle with the same offset. */
WQ_API int wq_ipc_close_handle(void* ptr, int64_t offset);

/* wq_dequant_gemm_f32 with the output written to n_out buffers (1 <= n_out
 * <= WQ_MAX_OUTPUTS, a host array of device pointers, local or peer-mapped),
 * each holding the [B, M] result at row stride ldy. The decode and
 * tensor-core kernels store into all of them as they finish each value; the
 * tiled fallback computes into y_out[0] and copies it to the rest on the same
 * stream. y_all, when not NULL, is an NVLink-switch address (NVLS) that
 * reaches the same position in every rank's buffer: the decode and
 * tensor-core kernels then issue one multimem.st per value instead of n_out
 * stores, and y_out is used only by the fallback. bias, when not NULL, is an
 * fp32 [M] vector added to every output row by the kernels' epilogues (the
 * reference adds it after the GEMM in Python, linear.py:99-100: the same
 * single fp32 add). */
WQ_API int wq_dequant_gemm_f32_multi(const float* x, int64_t B, int64_t K,
                                     const uint8_t* q, int64_t M, int64_t q_cols,
                                     const float* scales, int64_t scale_rows, int64_t groups,
                                     const float* zeros, int64_t zero_rows, int64_t zero_groups,
                                     const float* channel_scale, int64_t channel_len,
                                     int group_size, int bits,
                                     float* const* y_out, int n_out, int64_t ldy, float* y_all,
                                     const float* bias,
                                     void* workspace, size_t workspace_bytes,
                                     void* stream);

#ifdef __cplusplus
}
#endif
#endif /* WQ_B200_H */

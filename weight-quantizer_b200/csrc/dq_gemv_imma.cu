// K1i — int4 decode dequant-GEMM for batches 1-2 (3-4 as two launches) on the
// integer tensor-core path (mma.sync u8 x s8 -> s32).
//
// Same math as ptqkit's CPU kernel (src/ptqkit/csrc/dequant_gemm.cpp:57-218,
// run_gemm / dequant_row / dots_into), y[b,m] = sum_g scale[m,g] * sum_{k in g}
// (q[m,k] - zero[m,g]) * x'[b,k] with x' = x * channel, reorganized so that the
// products of codes and activations are exact integer products:
//
//   * x' is cut into fold blocks of F = 128 (or 64) consecutive k. In each
//     block, x' is written as a 23-bit signed fixed-point integer relative to
//     the block's largest magnitude, x'_k = X_k * 2^(e-22) with |X_k| <= 2^22
//     (round to nearest; the error per element is at most 2^-23 of the block
//     maximum), and X_k is split into three signed base-256 digits,
//     X_k = sum_l d_lk 256^l with d_lk in [-128, 127].
//   * The packed codes (ptqkit's int4 layout, unchanged) are widened to bytes
//     in registers: a 32-bit word of codes 8c..8c+7 gives the even codes
//     (w & 0x0F0F0F0F) and the odd codes ((w >> 4) & 0x0F0F0F0F), 3 ALU
//     operations per 8 codes. One mma.sync.m16n8k32 multiplies 16 rows x 32
//     codes by the 32 x 8 digit matrix whose column 4b + l (l < 3) is limb l
//     of batch row b; columns 4b + 3 are empty. Products and s32 accumulators
//     are exact, so C[m, 4b+l] = sum_k q[m,k] d_lk(b).
//   * Per fold block and row: sum_k q x'_b = 2^(e-22) sum_l 256^l C[m, 4b+l],
//     and the zero point enters as zero * sum_k X_k (the integer sum of the
//     same block). A lane's two C columns belong to one batch row: limbs 0-1
//     (combined as C0 + 256 C1, exact in s32), or limb 2 and the empty
//     column, in which that lane folds the zero-point term. Each lane folds
//     into one fp32 accumulator per row with the row's scale.
//
// The integer MMA runs at the full legacy tensor rate on sm_100 (the 4-bit
// u4 x s4 form does not: it is about 20x slower there), and one MMA covers
// 512 codes with ~11 ALU instructions, a small fraction of a SIMT
// multiply-add loop's cost, which leaves the kernel bound by the weight stream.
//
// Mapping. 8 multiply warps and one producer warp per CTA, one CTA per SM
// (persistent). Multiply warp w owns the fold blocks [w*nfb/8, (w+1)*nfb/8)
// of every row and keeps their digit fragments (the MMA's B operand) in
// registers for the whole launch: lane (g, t) = (lane/4, lane%4) holds column
// g of the codes that thread-in-group t supplies. Rows stream past in row
// blocks of 8-16 rows (chosen so that the last wave is full; the MMA's other
// rows are ignored): the producer issues one bulk asynchronous copy
// (cp.async.bulk) per row of codes, and per table or per table row, into a
// ring of shared-memory stages, completing on an mbarrier. Shared-memory rows
// are padded so that the fragment loads (16 or 8 bytes per lane) are free of
// bank conflicts. Each multiply warp folds its slice's accumulators, adds the
// lanes of one batch row with shuffles and leaves one partial per row and
// batch row in shared memory; the producer adds the 8 partials in a fixed
// order (deterministic, no atomics), writes y and refills the stage. The x'
// loads are issued before the weight stream so that they do not queue behind
// it. Every mbarrier wait is bounded; on expiry the kernel sets bit 0 of the
// library's fault word and runs to completion without waiting again.
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace wq {
namespace {

constexpr int kImmaWarps = 8;                  // warps that multiply
constexpr int kImmaThreads = (kImmaWarps + 1) * 32;   // + one producer warp
constexpr int kImmaRows = 16;                  // rows an MMA (and a stage) holds; a row block uses rb <= 16
constexpr int kSliceCodes = 1024;              // most codes of a row one warp covers
constexpr int kLimbs = 3;                      // base-256 digits of a 23-bit signed integer
constexpr int kDigRow = kSliceCodes / 8 * 2 + 4;  // words per limb row: (even, odd) per octet, +16 B skew
constexpr int kImmaMaxStages = 4;
constexpr int kOctIters = kSliceCodes / 8 / 32;   // octets per lane in the x' staging
constexpr uint32_t kDigitBias = 0x808080u;     // + 128 in each of the three digits

enum ImmaTables : int {
    kTabPerRow = 0,     // scale_rows == M, groups % 4 == 0: one bulk copy per table row (padded)
    kTabColumn = 1,     // scale_rows == M, groups == 1: one contiguous copy per table
    kTabShared = 2,     // scale_rows == 1: one table for every row, loaded once
    kTabBlock = 3,      // scale_rows == M, one group per fold block: one contiguous copy per table
};

struct ImmaParams {
    const float* x;
    const uint8_t* q;
    const float* scales;
    const float* zeros;
    const float* channel;
    float* y;
    float* y_extra[7];
    int n_extra;
    float* y_all;
    const float* bias;
    unsigned int* fault;
    int M, K;
    int64_t q_stride, ldy;
    int groups, group_size;
    int nfb;            // fold blocks per row, ceil(K / F)
    int tables;         // ImmaTables
    int ts;             // floats per table row inside a stage (0: shared table)
    int rs;             // bytes per code row inside a stage
    int ns;             // stages
    int rb;             // rows per row block (<= 16; the MMA's other rows are ignored)
    int defer_last;     // the digit table borrows the last stage, which is filled after staging
    uint32_t stage_bytes;
    uint32_t shared_tab_bytes;
    uint32_t dig_off;   // byte offset of the digit table
    uint32_t fbt_off;   // byte offset of the fold-block table
    int x_vec4;         // x rows and channel 16-byte aligned and K % 4 == 0
};

__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int NB, int FBW>
struct ImmaLayout {
    __host__ __device__ static size_t dig_bytes() { return (size_t)kImmaWarps * NB * kLimbs * kDigRow * 4; }
    __host__ __device__ static size_t fbt_bytes() { return (size_t)kImmaWarps * NB * FBW * 8; }
    __host__ __device__ static size_t red_bytes(int ns) { return (size_t)ns * kImmaWarps * kImmaRows * NB * 4; }
};

// Digit-matrix columns: 4b + l (l < 3) is limb l of batch row b, 4b + 3 is
// empty (zero digits). Lane (g, t) of the C fragment holds columns 2t and
// 2t + 1 of rows g and g + 8: lanes with t even the limbs 0 and 1 of batch row
// t / 2, lanes with t odd its limb 2 and the empty column, in which those
// lanes accumulate the zero-point term instead.
__device__ __forceinline__ uint32_t lo_nibbles(uint32_t w) { return w & 0x0F0F0F0Fu; }
__device__ __forceinline__ uint32_t hi_nibbles(uint32_t w) { return (w >> 4) & 0x0F0F0F0Fu; }

// F: codes per fold block (128 or 64). FBW: fold blocks per warp (the most,
// or exactly, when FAST). FAST: every warp holds exactly FBW fold blocks,
// one quantization group per fold block, tables copied as one block per
// stage (kTabBlock) and read once per row block as 16-byte loads.
template <int NB, int F, int FBW, bool FAST>
__global__ void __launch_bounds__(kImmaThreads, 1) gemv_imma_kernel(const ImmaParams p) {
    using L = ImmaLayout<NB, FBW>;
    constexpr int MPF = F / 32;   // MMAs per fold block (32 codes each)
    constexpr int LPF = F / 8;    // octets of codes per fold block (one per lane in the x' staging)
    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char* stages = smem_raw;
    float* shared_sc = reinterpret_cast<float*>(smem_raw + (size_t)p.ns * p.stage_bytes);
    float* shared_zr = shared_sc + (p.tables == kTabShared ? p.groups : 0);
    uint32_t* dig = reinterpret_cast<uint32_t*>(smem_raw + p.dig_off);
    float2* fbt = reinterpret_cast<float2*>(smem_raw + p.fbt_off);
    float* red = reinterpret_cast<float*>(smem_raw + p.fbt_off + L::fbt_bytes());
    uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + p.fbt_off + L::fbt_bytes() + L::red_bytes(p.ns));
    uint64_t* consumed = full + p.ns;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const bool producer = warp == kImmaWarps;
    // Programmatic dependent launch: the next kernel on the stream may be
    // scheduled now (its CTAs take an SM as ours leave it, and run up to their
    // own wait), and this one reads nothing in global memory before every
    // earlier kernel on the stream has completed and its writes are visible.
    // Without the launch attribute both instructions do nothing.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int n_blocks = (p.M + p.rb - 1) / p.rb;
    const uint32_t full0 = smem_addr(full);
    const uint32_t cons0 = smem_addr(consumed);
    const uint32_t tab_bytes = p.tables == kTabShared ? 0u : (uint32_t)(kImmaRows * p.ts * 4);

    // Bulk copies of row block `blk` into stage `s`, issued by the producer
    // warp's lanes (lane 0 registers the byte count first).
    // per stage: bit s of `filled` once a fill was issued, bit s of `fill_par`
    // the parity of the number of fills (producer lane 0)
    uint32_t filled = 0, fill_par = 0;
    auto issue = [&](int blk, int s) {
        const int row0 = blk * p.rb;
        const int rows = (p.M - row0) < p.rb ? (p.M - row0) : p.rb;
        const uint32_t dst = smem_addr(stages + (size_t)s * p.stage_bytes);
        const uint32_t bar = full0 + 8u * (uint32_t)s;
        uint32_t tb = 0;
        if (p.tables == kTabPerRow || p.tables == kTabBlock) tb = (uint32_t)(rows * p.groups * 4);
        if (p.tables == kTabColumn) tb = (uint32_t)(rows * 4);
        if (lane == 0) {
            mbar_arrive_expect_tx(bar, (uint32_t)rows * (uint32_t)p.q_stride + 2u * tb);
            filled |= 1u << s;
            fill_par ^= 1u << s;
        }
        __syncwarp();
        const uint32_t tdst = dst + (uint32_t)kImmaRows * (uint32_t)p.rs;
        if (lane < rows) {
            bulk_copy_g2s(dst + (uint32_t)lane * (uint32_t)p.rs, p.q + (int64_t)(row0 + lane) * p.q_stride,
                          (uint32_t)p.q_stride, bar);
            if (p.tables == kTabPerRow) {
                const uint32_t rowb = (uint32_t)(p.groups * 4);
                const uint32_t roff = (uint32_t)lane * (uint32_t)(p.ts * 4);
                bulk_copy_g2s(tdst + roff, p.scales + (int64_t)(row0 + lane) * p.groups, rowb, bar);
                bulk_copy_g2s(tdst + tab_bytes + roff, p.zeros + (int64_t)(row0 + lane) * p.groups, rowb, bar);
            }
        }
        if ((p.tables == kTabColumn || p.tables == kTabBlock) && lane == 16) {
            const int64_t toff = (int64_t)row0 * (p.tables == kTabBlock ? p.groups : 1);
            bulk_copy_g2s(tdst, p.scales + toff, tb, bar);
            bulk_copy_g2s(tdst + tab_bytes, p.zeros + toff, tb, bar);
        }
    };

    // ---- x' loads first, ahead of the weight stream in the memory queues ----
    const int fb0 = (warp * p.nfb) / kImmaWarps;
    const int nfbw = FAST ? FBW : ((warp + 1) * p.nfb) / kImmaWarps - fb0;
    const int n_oct = nfbw * LPF;
    float xv[NB][kOctIters][8];
    if (!producer) {
#pragma unroll
        for (int it = 0; it < kOctIters; ++it) {
            const int o = it * 32 + lane;
            const int k0 = fb0 * F + o * 8;
            const bool valid = o < n_oct;
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const float* xb = p.x + (int64_t)b * p.K;
                if (valid && p.x_vec4 && k0 + 8 <= p.K) {
                    const float4 v0 = __ldg(reinterpret_cast<const float4*>(xb + k0));
                    const float4 v1 = __ldg(reinterpret_cast<const float4*>(xb + k0 + 4));
                    xv[b][it][0] = v0.x; xv[b][it][1] = v0.y; xv[b][it][2] = v0.z; xv[b][it][3] = v0.w;
                    xv[b][it][4] = v1.x; xv[b][it][5] = v1.y; xv[b][it][6] = v1.z; xv[b][it][7] = v1.w;
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) xv[b][it][j] = (valid && k0 + j < p.K) ? __ldg(xb + k0 + j) : 0.0f;
                }
            }
            if (p.channel != nullptr) {
                float cv[8];
                if (valid && p.x_vec4 && k0 + 8 <= p.K) {
                    const float4 c0 = __ldg(reinterpret_cast<const float4*>(p.channel + k0));
                    const float4 c1 = __ldg(reinterpret_cast<const float4*>(p.channel + k0 + 4));
                    cv[0] = c0.x; cv[1] = c0.y; cv[2] = c0.z; cv[3] = c0.w;
                    cv[4] = c1.x; cv[5] = c1.y; cv[6] = c1.z; cv[7] = c1.w;
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) cv[j] = (valid && k0 + j < p.K) ? __ldg(p.channel + k0 + j) : 0.0f;
                }
#pragma unroll
                for (int b = 0; b < NB; ++b)
#pragma unroll
                    for (int j = 0; j < 8; ++j) xv[b][it][j] *= cv[j];
            }
        }
    } else {
        // ---- barriers, then the weight stream -------------------------------
        if (lane == 0) {
            for (int s = 0; s < p.ns; ++s) {
                mbar_init(full0 + 8u * (uint32_t)s, 1);
                mbar_init(cons0 + 8u * (uint32_t)s, (uint32_t)kImmaWarps);
            }
            fence_mbarrier_init();
        }
        __syncwarp();
        for (int s = 0; s < p.ns - p.defer_last; ++s) {
            const int blk = (int)blockIdx.x + s * (int)gridDim.x;
            if (blk < n_blocks) issue(blk, s);
        }
    }
    if (p.tables == kTabShared) {
        for (int i = threadIdx.x; i < p.groups; i += kImmaThreads) {
            shared_sc[i] = __ldg(p.scales + i);
            shared_zr[i] = __ldg(p.zeros + i);
        }
    }

    // ---- per-block exponent, 23-bit integers, digit words per octet ---------
    uint32_t* dig_w = dig + (size_t)(producer ? 0 : warp) * NB * kLimbs * kDigRow;
    float2* fbt_w = fbt + (size_t)(producer ? 0 : warp) * NB * FBW;
    if (!producer) {
#pragma unroll
        for (int b = 0; b < NB; ++b) {
#pragma unroll
            for (int it = 0; it < kOctIters; ++it) {
                const int o = it * 32 + lane;
                const bool valid = o < n_oct;
                float m = 0.0f;
#pragma unroll
                for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(xv[b][it][j]));
#pragma unroll
                for (int off = 1; off < LPF; off <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
                // m < 2^e with e = biased exponent - 126 (m = 0 and subnormal m give
                // e <= -126, raised to -100 so that both scalings stay normal).
                const int E = (int)((__float_as_uint(m) >> 23) & 0xFFu);
                int e = E - 126;
                e = e < -100 ? -100 : e;
                const float sc = pow2i(22 - e);
                const float pw = E == 255 ? __int_as_float(0x7fc00000) : pow2i(e - 22);
                uint32_t u[8];
                int sx = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int xi = __float2int_rn(xv[b][it][j] * sc);   // exact scaling, then round half to even
                    sx += xi;
                    u[j] = (uint32_t)(xi + (int)kDigitBias);            // in [0, 2^24): three unsigned digits
                }
#pragma unroll
                for (int off = 1; off < LPF; off <<= 1) sx += __shfl_xor_sync(0xffffffffu, sx, off);
                if (valid) {
#pragma unroll
                    for (int l = 0; l < kLimbs; ++l) {
                        // digit l of the even codes (0, 2, 4, 6) and of the odd codes, one byte
                        // each; unsigned digit n encodes n - 128, as a signed byte that is n ^ 0x80
                        const uint32_t sel = (uint32_t)l | ((uint32_t)(4 + l) << 4);
                        const uint32_t ev =
                            __byte_perm(__byte_perm(u[0], u[2], sel), __byte_perm(u[4], u[6], sel), 0x5410);
                        const uint32_t od =
                            __byte_perm(__byte_perm(u[1], u[3], sel), __byte_perm(u[5], u[7], sel), 0x5410);
                        *reinterpret_cast<uint2*>(dig_w + ((size_t)b * kLimbs + l) * kDigRow + 2 * o) =
                            make_uint2(ev ^ 0x80808080u, od ^ 0x80808080u);
                    }
                    if ((lane & (LPF - 1)) == 0) fbt_w[b * FBW + o / LPF] = make_float2(pw, (float)sx);
                }
            }
        }
        __syncwarp();
    }

    // ---- this lane's B fragments and fold factors, kept for the launch -------
    const int g = lane >> 2;   // MMA group: rows g and g + 8, B column g
    const int t = lane & 3;    // thread in group: C columns 2t and 2t + 1
    const int col_b = g >> 2, col_l = g & 3;          // this lane's B column: batch row, limb
    const int lane_b = NB == 2 ? (t >> 1) : 0;        // batch row of this lane's C columns
    const bool zero_lane = (t & 1) && (NB == 2 || t == 1);
    const int mB = (t & 1) ? 0 : 256;                 // C columns -> integer: limb0 + 256 limb1, or limb2
    const float wC = (t & 1) ? 65536.0f : 1.0f;
    uint32_t bw[FBW][2 * MPF];
    float pw[FBW], zq[FBW];   // 2^(e-22) of the fold block; sum of X on zero-point lanes
    int gix[FBW];
    const int fold_per_group = p.groups > 1 ? p.group_size / F : 0;
#pragma unroll
    for (int i = 0; i < FBW; ++i) {
        gix[i] = (i < nfbw && fold_per_group > 0) ? (fb0 + i) / fold_per_group : 0;
#pragma unroll
        for (int v = 0; v < 2 * MPF; ++v) bw[i][v] = 0u;
        pw[i] = zq[i] = 0.0f;
        if (!producer && i < nfbw) {
            if (col_l < kLimbs && col_b < NB) {
                // octets i*LPF + t*MPF + [0, MPF): (even, odd) words = MPF MMAs' b0, b1
                const uint32_t* src = dig_w + ((size_t)col_b * kLimbs + col_l) * kDigRow + 2 * (i * LPF + t * MPF);
#pragma unroll
                for (int v = 0; v < 2 * MPF; v += 4) {
                    const uint4 q4 = *reinterpret_cast<const uint4*>(src + v);
                    bw[i][v] = q4.x; bw[i][v + 1] = q4.y; bw[i][v + 2] = q4.z; bw[i][v + 3] = q4.w;
                }
            }
            if constexpr (!FAST) {
                const float2 pf = fbt_w[lane_b * FBW + i];
                pw[i] = pf.x;
                zq[i] = zero_lane ? pf.y : 0.0f;
            }
        }
    }
    named_barrier(1, kImmaThreads);   // mbarrier init, shared table and every lane's reads of the digit table

    if (producer) {
        // ---- producer: refill stages, finish rows ---------------------------
        bool faulted = false;
        if (p.defer_last) {
            const int blk = (int)blockIdx.x + (p.ns - 1) * (int)gridDim.x;
            if (blk < n_blocks) {
                fence_proxy_async_smem();   // the digit table's generic accesses before the copies reuse it
                issue(blk, p.ns - 1);
            }
        }
        int s = 0;
        uint32_t phase = 0;
#pragma unroll 1
        for (int blk = (int)blockIdx.x; blk < n_blocks; blk += (int)gridDim.x) {
            if (lane == 0 && !faulted && !mbar_wait_bounded(cons0 + 8u * (uint32_t)s, phase)) {
                faulted = true;
                atomicOr(p.fault, 1u);
            }
            faulted = __shfl_sync(0xffffffffu, faulted ? 1 : 0, 0) != 0;
            __syncwarp();
            const float* rb = red + (size_t)s * kImmaWarps * kImmaRows * NB;
            const int r = lane & (kImmaRows - 1), b = lane >> 4;
            if (lane < kImmaRows * NB && r < p.rb) {
                const int row = blk * p.rb + r;
                float v = 0.0f;
#pragma unroll
                for (int w = 0; w < kImmaWarps; ++w) v += rb[(w * kImmaRows + r) * NB + b];
                if (row < p.M) {
                    if (p.bias != nullptr) v = __fadd_rn(v, p.bias[row]);   // linear.py:99-100
                    const int64_t off = (int64_t)b * p.ldy + row;
                    if (p.y_all != nullptr) {
                        asm volatile("multimem.st.global.f32 [%0], %1;" ::"l"(p.y_all + off), "f"(v) : "memory");
                    } else {
                        p.y[off] = v;
                        for (int d = 0; d < p.n_extra; ++d) p.y_extra[d][off] = v;
                    }
                }
            }
            __syncwarp();
            const int next = blk + p.ns * (int)gridDim.x;
            if (!faulted && next < n_blocks) {
                fence_proxy_async_smem();   // the CTA's reads of stage s before the copies refill it
                issue(next, s);
            }
            if (++s == p.ns) {
                s = 0;
                phase ^= 1u;
            }
        }
        // Copies issued before a fault may still be in flight into this CTA's
        // shared memory: wait (bounded) for the last fill of every stage. In a
        // fault-free run those phases have completed already.
        if (lane == 0) {
            for (int i = 0; i < p.ns; ++i) {
                // the last fill completes the phase of parity (number of fills - 1)
                if (((filled >> i) & 1u) && !mbar_wait_bounded(full0 + 8u * (uint32_t)i, ((fill_par >> i) & 1u) ^ 1u))
                    atomicOr(p.fault, 1u);
            }
        }
        return;
    }

    // ---- multiply warps: stream rows ----------------------------------------
    const float2* fbt_lane = fbt_w + lane_b * FBW;
    bool faulted = false;
    int s = 0;
    uint32_t phase = 0;
#pragma unroll 1
    for (int blk = (int)blockIdx.x; blk < n_blocks; blk += (int)gridDim.x) {
        if (!faulted && !mbar_wait_bounded(full0 + 8u * (uint32_t)s, phase)) {
            faulted = true;
            atomicOr(p.fault, 1u);
        }
        const unsigned char* stg = stages + (size_t)s * p.stage_bytes;
        const unsigned char* code_g = stg + (size_t)g * p.rs + t * (F / 8);
        const unsigned char* code_h = code_g + (size_t)8 * p.rs;
        const float* tsc = p.tables == kTabShared ? shared_sc
                                                  : reinterpret_cast<const float*>(stg + (size_t)kImmaRows * p.rs);
        const float* tzr = p.tables == kTabShared ? shared_zr : tsc + kImmaRows * p.ts;
        float acc0 = 0.0f, acc1 = 0.0f;   // rows g and g + 8
        if constexpr (FAST) {
            // one group per fold block: this warp's FBW consecutive groups of rows g, g + 8
            float sg[FBW], sh[FBW], zg[FBW], zh[FBW];
#pragma unroll
            for (int q = 0; q < FBW; q += 4) {
                const float4 a = *reinterpret_cast<const float4*>(tsc + g * p.ts + fb0 + q);
                const float4 b = *reinterpret_cast<const float4*>(tsc + (g + 8) * p.ts + fb0 + q);
                const float4 c = *reinterpret_cast<const float4*>(tzr + g * p.ts + fb0 + q);
                const float4 d = *reinterpret_cast<const float4*>(tzr + (g + 8) * p.ts + fb0 + q);
                sg[q] = a.x; sg[q + 1] = a.y; sg[q + 2] = a.z; sg[q + 3] = a.w;
                sh[q] = b.x; sh[q + 1] = b.y; sh[q + 2] = b.z; sh[q + 3] = b.w;
                zg[q] = c.x; zg[q + 1] = c.y; zg[q + 2] = c.z; zg[q + 3] = c.w;
                zh[q] = d.x; zh[q + 1] = d.y; zh[q + 2] = d.z; zh[q + 3] = d.w;
            }
#pragma unroll
            for (int i = 0; i < FBW; ++i) {
                const int boff = (fb0 + i) * (F / 2);
                uint32_t ag[MPF], ah[MPF];
                if constexpr (MPF == 4) {
                    const uint4 a = *reinterpret_cast<const uint4*>(code_g + boff);
                    const uint4 h = *reinterpret_cast<const uint4*>(code_h + boff);
                    ag[0] = a.x; ag[1] = a.y; ag[2] = a.z; ag[3] = a.w;
                    ah[0] = h.x; ah[1] = h.y; ah[2] = h.z; ah[3] = h.w;
                } else {
                    const uint2 a = *reinterpret_cast<const uint2*>(code_g + boff);
                    const uint2 h = *reinterpret_cast<const uint2*>(code_h + boff);
                    ag[0] = a.x; ag[1] = a.y;
                    ah[0] = h.x; ah[1] = h.y;
                }
                // two independent accumulation chains per fold block
                int c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
#pragma unroll
                for (int mm = 0; mm < MPF; mm += 2) {
                    mma_u8s8(c0, lo_nibbles(ag[mm]), lo_nibbles(ah[mm]), hi_nibbles(ag[mm]), hi_nibbles(ah[mm]),
                             bw[i][2 * mm], bw[i][2 * mm + 1]);
                    mma_u8s8(c1, lo_nibbles(ag[mm + 1]), lo_nibbles(ah[mm + 1]), hi_nibbles(ag[mm + 1]),
                             hi_nibbles(ah[mm + 1]), bw[i][2 * mm + 2], bw[i][2 * mm + 3]);
                }
                // the fold block's factors come from shared memory (a broadcast
                // load) rather than registers, which this variant has none to spare
                const float2 pf = fbt_lane[i];
                const float zqi = zero_lane ? pf.y : 0.0f;
                const float v0 = fmaf((float)((c0[0] + c1[0]) + mB * (c0[1] + c1[1])), wC, -zg[i] * zqi);
                const float v1 = fmaf((float)((c0[2] + c1[2]) + mB * (c0[3] + c1[3])), wC, -zh[i] * zqi);
                acc0 = fmaf(sg[i] * pf.x, v0, acc0);
                acc1 = fmaf(sh[i] * pf.x, v1, acc1);
            }
        } else {
            const float* tsc_g = tsc + g * p.ts;
            const float* tsc_h = tsc + (g + 8) * p.ts;
            const float* tzr_g = tzr + g * p.ts;
            const float* tzr_h = tzr + (g + 8) * p.ts;
#pragma unroll
            for (int i = 0; i < FBW; ++i) {
                if (i < nfbw) {
                    const int boff = (fb0 + i) * (F / 2);
                    uint32_t ag[MPF], ah[MPF];
                    if constexpr (MPF == 4) {
                        const uint4 a = *reinterpret_cast<const uint4*>(code_g + boff);
                        const uint4 h = *reinterpret_cast<const uint4*>(code_h + boff);
                        ag[0] = a.x; ag[1] = a.y; ag[2] = a.z; ag[3] = a.w;
                        ah[0] = h.x; ah[1] = h.y; ah[2] = h.z; ah[3] = h.w;
                    } else {
                        const uint2 a = *reinterpret_cast<const uint2*>(code_g + boff);
                        const uint2 h = *reinterpret_cast<const uint2*>(code_h + boff);
                        ag[0] = a.x; ag[1] = a.y;
                        ah[0] = h.x; ah[1] = h.y;
                    }
                    const float sc0 = tsc_g[gix[i]], sc1 = tsc_h[gix[i]];
                    const float zr0 = tzr_g[gix[i]], zr1 = tzr_h[gix[i]];
                    int c[4] = {0, 0, 0, 0};
#pragma unroll
                    for (int mm = 0; mm < MPF; ++mm)
                        mma_u8s8(c, lo_nibbles(ag[mm]), lo_nibbles(ah[mm]), hi_nibbles(ag[mm]), hi_nibbles(ah[mm]),
                                 bw[i][2 * mm], bw[i][2 * mm + 1]);
                    // c[0], c[1]: row g, columns 2t, 2t+1; c[2], c[3]: row g + 8
                    const float v0 = fmaf((float)(c[0] + mB * c[1]), wC, -zr0 * zq[i]);
                    const float v1 = fmaf((float)(c[2] + mB * c[3]), wC, -zr1 * zq[i]);
                    acc0 = fmaf(sc0 * pw[i], v0, acc0);
                    acc1 = fmaf(sc1 * pw[i], v1, acc1);
                }
            }
        }
        float* rb = red + (size_t)s * kImmaWarps * kImmaRows * NB;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float v = r == 0 ? acc0 : acc1;
            v += __shfl_xor_sync(0xffffffffu, v, 1);   // the two lanes of one batch row
            if (NB == 1) v += __shfl_xor_sync(0xffffffffu, v, 2);
            if ((t & 1) == 0 && (NB == 2 || t == 0)) rb[(warp * kImmaRows + g + 8 * r) * NB + lane_b] = v;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(cons0 + 8u * (uint32_t)s);
        if (++s == p.ns) {
            s = 0;
            phase ^= 1u;
        }
    }
}

// Shared memory one CTA may use on B200 (227 KB).
constexpr size_t kImmaSmemMax = 227 * 1024;

struct ImmaPlan {
    int F, FBW, fast, tables, ts, rs, ns, rb, nfb, defer_last;
    uint32_t stage_bytes, shared_tab_bytes, dig_off, fbt_off;
    size_t smem;
};

template <int NB, int FBW>
bool imma_layout(ImmaPlan& pl) {
    using L = ImmaLayout<NB, FBW>;
    for (int ns = kImmaMaxStages; ns >= 2; --ns) {
        const size_t stages = (size_t)ns * pl.stage_bytes;
        const bool defer = L::dig_bytes() <= pl.stage_bytes;
        size_t o = stages + pl.shared_tab_bytes;
        const size_t dig_off = defer ? (size_t)(ns - 1) * pl.stage_bytes : o;
        if (!defer) o += L::dig_bytes();
        const size_t fbt_off = o;
        o += L::fbt_bytes() + L::red_bytes(ns) + (size_t)ns * 16;
        if (o <= kImmaSmemMax) {
            pl.ns = ns;
            pl.defer_last = defer ? 1 : 0;
            pl.dig_off = (uint32_t)dig_off;
            pl.fbt_off = (uint32_t)fbt_off;
            pl.smem = o;
            return true;
        }
    }
    return false;
}

bool imma_plan(const GemmProblem& g, ImmaPlan& pl) {
    if (g.bits != 4 || g.B < 1 || g.B > 2 || g.M < 1 || g.K < 1) return false;
    if (g.q_stride % 16 != 0 || (reinterpret_cast<uintptr_t>(g.q) & 15) != 0) return false;
    if (g.M > ((int64_t)1 << 30) || g.K > kImmaWarps * kSliceCodes) return false;
    if (g.groups == 1) {
        pl.F = 128;
    } else if (g.group_size % 128 == 0) {
        pl.F = 128;
    } else if (g.group_size % 64 == 0) {
        pl.F = 64;
    } else {
        return false;
    }
    pl.nfb = (int)((g.K + pl.F - 1) / pl.F);
    pl.FBW = kSliceCodes / pl.F;
    // every warp's slice holds at most kSliceCodes codes
    if ((pl.nfb + kImmaWarps - 1) / kImmaWarps * pl.F > kSliceCodes) return false;
    const bool al_tab = ((reinterpret_cast<uintptr_t>(g.scales) & 15) == 0) &&
                        ((reinterpret_cast<uintptr_t>(g.zeros) & 15) == 0);
    // every warp holds exactly 8 (or 4) fold blocks of 128 codes, one group each
    pl.fast = 0;
    if (pl.F == 128 && g.group_size == 128 && g.scale_rows != 1 && al_tab &&
        (pl.nfb == kImmaWarps * 8 || pl.nfb == kImmaWarps * 4)) {
        pl.fast = 1;
        pl.FBW = pl.nfb / kImmaWarps;
        pl.tables = kTabBlock;
        pl.ts = g.groups;
    } else if (g.scale_rows == 1) {
        pl.tables = kTabShared;
        pl.ts = 0;
    } else if (g.groups % 4 == 0 && al_tab) {
        pl.tables = kTabPerRow;
        pl.ts = g.groups + 4;   // 16-byte pad: rows land 4 banks apart
    } else if (g.groups == 1 && g.M % 4 == 0 && al_tab) {
        pl.tables = kTabColumn;
        pl.ts = 1;
    } else {
        return false;
    }
    const int64_t row_read = (int64_t)pl.nfb * pl.F / 2;   // bytes a row's fragments span (>= q_stride)
    pl.rs = (int)((row_read + 127) / 128 * 128 + (pl.F == 128 ? 64 : 32));
    const size_t stage = (size_t)kImmaRows * pl.rs + (size_t)2 * kImmaRows * pl.ts * 4;
    pl.stage_bytes = (uint32_t)((stage + 127) / 128 * 128);
    pl.shared_tab_bytes = pl.tables == kTabShared ? (uint32_t)((2 * g.groups * 4 + 15) / 16 * 16) : 0u;
    if (g.B == 1) {
        if (pl.FBW == 4) return imma_layout<1, 4>(pl);
        if (pl.FBW == 8) return imma_layout<1, 8>(pl);
        return imma_layout<1, 16>(pl);
    }
    if (pl.FBW == 4) return imma_layout<2, 4>(pl);
    if (pl.FBW == 8) return imma_layout<2, 8>(pl);
    return imma_layout<2, 16>(pl);
}

// Rows per row block: the value in [8, 16] whose last wave is fullest, i.e.
// that minimizes (row blocks per CTA, rounded up) x rows per block; ties go
// to more rows. Per-channel tables are copied whole, so there the block must
// keep a multiple of 4 rows.
int imma_rows_per_block(int64_t M, int grid_max, int tables) {
    int best = kImmaRows;
    int64_t best_cost = -1;
    for (int rb = kImmaRows; rb >= 8; --rb) {
        if (tables == kTabColumn && rb % 4 != 0) continue;
        const int64_t nb = (M + rb - 1) / rb;
        const int64_t cost = (nb + grid_max - 1) / grid_max * rb;
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = rb;
        }
    }
    return best;
}

template <int NB, int F, int FBW, bool FAST>
cudaError_t launch_imma_t(ImmaParams p, size_t smem, cudaStream_t s) {
    auto kern = gemv_imma_kernel<NB, F, FBW, FAST>;
    // The shared-memory opt-in and the occupancy for it are looked up once per
    // device and shared-memory size (the last pair is kept).
    constexpr int kDevs = 32;
    static std::atomic<uint64_t> cache[kDevs];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int occ = 0;
    const uint64_t c = (dev >= 0 && dev < kDevs) ? cache[dev].load(std::memory_order_relaxed) : 0;
    if (c != 0 && (c >> 32) == (uint64_t)smem) {
        occ = (int)(c & 0xFFFFFFFFu);
    } else {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kImmaThreads, smem);
        if (e != cudaSuccess) return e;
        if (occ < 1) return cudaErrorInvalidConfiguration;
        if (dev >= 0 && dev < kDevs) cache[dev].store(((uint64_t)smem << 32) | (uint32_t)occ, std::memory_order_relaxed);
    }
    const int grid_max = sm_count() * occ;
    p.rb = imma_rows_per_block(p.M, grid_max, p.tables);
    const int n_blocks = (p.M + p.rb - 1) / p.rb;
    int grid = grid_max < n_blocks ? grid_max : n_blocks;
    if (grid < 1) grid = 1;
    // launched with programmatic stream serialization (see the kernel's first
    // lines): back-to-back decode layers overlap one launch's start with the
    // previous kernel's tail
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kImmaThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int NB>
cudaError_t launch_imma_nb(const ImmaPlan& pl, const ImmaParams& p, cudaStream_t s) {
    if (pl.fast) {
        return pl.FBW == 8 ? launch_imma_t<NB, 128, 8, true>(p, pl.smem, s)
                           : launch_imma_t<NB, 128, 4, true>(p, pl.smem, s);
    }
    return pl.F == 128 ? launch_imma_t<NB, 128, 8, false>(p, pl.smem, s)
                       : launch_imma_t<NB, 64, 16, false>(p, pl.smem, s);
}

}  // namespace

bool gemv_imma_supported(const GemmProblem& g) {
    ImmaPlan pl;
    return imma_plan(g, pl);
}

cudaError_t launch_gemv_imma(const GemmProblem& g, cudaStream_t s) {
    ImmaPlan pl;
    if (!imma_plan(g, pl)) return cudaErrorInvalidValue;
    ImmaParams p;
    p.x = g.x;
    p.q = g.q;
    p.scales = g.scales;
    p.zeros = g.zeros;
    p.channel = g.channel;
    p.y = g.y;
    for (int d = 0; d < 7; ++d) p.y_extra[d] = g.y_extra[d];
    p.n_extra = g.n_extra;
    p.y_all = g.y_all;
    p.bias = g.bias;
    p.fault = fault_word();
    if (p.fault == nullptr) return cudaErrorInvalidDevicePointer;
    p.M = (int)g.M;
    p.K = (int)g.K;
    p.q_stride = g.q_stride;
    p.ldy = g.ldy;
    p.groups = g.groups;
    p.group_size = g.group_size;
    p.nfb = pl.nfb;
    p.tables = pl.tables;
    p.ts = pl.ts;
    p.rs = pl.rs;
    p.ns = pl.ns;
    p.rb = kImmaRows;
    p.defer_last = pl.defer_last;
    p.stage_bytes = pl.stage_bytes;
    p.shared_tab_bytes = pl.shared_tab_bytes;
    p.dig_off = pl.dig_off;
    p.fbt_off = pl.fbt_off;
    p.x_vec4 = (g.K % 4 == 0) && ((reinterpret_cast<uintptr_t>(g.x) & 15) == 0) &&
               (g.channel == nullptr || (reinterpret_cast<uintptr_t>(g.channel) & 15) == 0);
    return g.B == 1 ? launch_imma_nb<1>(pl, p, s) : launch_imma_nb<2>(pl, p, s);
}

}  // namespace wq

// K1w — dequant-GEMM for batches 3-32 (int4 and int8 codes) on the integer
// tensor-core path (mma.sync m16n8k32 u8 x s8 -> s32), stream-K over the
// weight.
//
// Same math as ptqkit's CPU kernel (src/ptqkit/csrc/dequant_gemm.cpp:57-218,
// run_gemm / dequant_row / dots_into) and the same exact-integer formulation
// as the batch-1/2 decode kernel (dq_gemv_imma.cu): in each fold block of F
// consecutive k (F = 128 or 64, inside one quantization group),
// x'_k = X_k 2^(e-22) with |X_k| <= 2^22 (e from the block's largest |x'|,
// per batch row), X_k = d0 + 256 d1 + 65536 d2 in signed bytes; one mma.sync
// multiplies 16 rows x 32 codes by 32 codes x 8 batch rows of one digit,
// exactly in s32, and per fold block, row and batch row
//
//   sum_k (q - zero) x' = 2^(e-22) (C0 + 256 C1 + 65536 C2 - zero * sum_k X)
//
// is folded into an fp32 accumulator with the row's group scale (any fp32
// zero point).
//
// What differs from the batch-1/2 kernel is the shape. With up to 32 batch
// rows the digits of x (3 bytes per k and batch row) no longer fit in
// registers, and at batch 32 every 16 x 32 block of codes takes 12 MMAs (3
// digits x 4 tiles of 8 batch rows), so above ~16 batch rows the legacy
// tensor pipe (~1900 int8 MACs per clock per SM on B200), not the weight
// stream, sets the time. Roles are the other way round:
//
//   * A prep kernel writes, for every fold block, one record: the digit tiles
//     of all batch rows in the order of the MMA's B fragments (each lane's 16
//     bytes for two k-steps together, a warp's 512 bytes contiguous), then
//     (2^(e-22), sum X) per batch row. It also zeroes the row-block counters.
//   * The weight is cut into units of 256 rows x one fold block. CTA c of P
//     (one per SM) takes units [c U / P, (c + 1) U / P) in row-block-major
//     order (stream-K), so every SM streams the same number of code bytes
//     whatever the layer's shape. A producer warp brings each unit into a
//     ring of shared-memory stages: one 2D TMA box of codes (256 rows x F
//     codes, rows dense and unswizzled: 8 rows of a warp's 16- or 8-byte
//     fragment loads fill 128 consecutive bytes, so the loads are free of
//     bank conflicts) and one bulk copy of the fold block's record.
//   * 8 multiply warps own 32 rows each (two MMA row tiles) and all batch
//     rows: per fold block they load their code words once, widen int4 codes
//     to bytes in registers (w & 0x0F0F0F0F gives codes 0, 2, 4, 6 of a word
//     and (w >> 4) & 0x0F0F0F0F codes 1, 3, 5, 7; int8 codes are bytes
//     already) and run (F / 32) k-steps x 3 digits x ceil(B / 8) batch tiles x
//     2 row tiles MMAs, each B fragment (one 16-byte shared load for two
//     k-steps) serving both row tiles. Scale and zero of the fold block's
//     group are read from global memory before the stage is waited for.
//   * A CTA that holds a whole row block writes y. Otherwise every CTA that
//     holds part of it writes its partial rows to a workspace slot, and the
//     last of them to arrive (an atomic counter per row block) adds the slots
//     in CTA order, a fixed order, and writes y: the result does not depend
//     on which CTA finishes last.
//
// The code permutation. Within a k-step the MMA pairs A's k-index 4t + i
// (and 16 + 4t + i) with B's; any one-to-one map of those indices to codes
// that A and B share is the same sum. Thread t of a fragment group reads code
// word 4t + s (int4, F = 128), 2t + s (int4, F = 64) or words 4t + 2s and
// 4t + 2s + 1 (int8) of each fold block for k-step s, and the prep kernel
// writes each lane's digits in that word's code order.
//
// Every mbarrier wait is bounded; on expiry the kernel sets bit 0 of the
// library's fault word and runs to completion without waiting again. No wait
// depends on another CTA. TMA and bulk loads target this CTA's own shared
// memory only, without multicast.
#include <cuda.h>

#include <atomic>
#include <cstring>

#include "common.cuh"
#include "kernels.h"

namespace wq {
namespace {

constexpr int kWideRows = 256;                         // rows per row block: one TMA box
constexpr int kWideLimbs = 3;                          // base-256 digits of a 23-bit signed integer
constexpr int kWideMaxStages = 8;
constexpr uint32_t kWideBias = 0x808080u;              // + 128 in each of the three digits
constexpr int kWidePiece = 512;                        // one digit tile piece: 32 lanes x 16 bytes

struct WideParams {
    const unsigned char* rec;   // per fold block: digit tiles, then (2^(e-22), sum X) per batch row
    const float* scales;
    const float* zeros;
    const float* bias;          // [M] or nullptr
    float* y;
    float* y_extra[7];          // further outputs with y's layout (peer-mapped or local)
    int n_extra;
    float* y_all;               // NVLink-switch address reaching every rank's y, or nullptr
    float* part;                // partial rows: [2 * grid][threads][E] (2048 NT floats per slot)
    int* counters;              // arrivals per row block (zeroed by the prep kernel)
    unsigned int* fault;
    int M, B, nfb, nrb, groups, fold_per_group, scale_rows;   // fold_per_group 0: one group
    int64_t ldy;
    int64_t units;              // nrb * nfb
    uint32_t rec_bytes;         // bytes of one fold block's record
    uint32_t stage_bytes;
    uint32_t tab_off;           // stage offset of the scale and zero boxes (tab_box)
    int tab_box;                // 1: scales and zeros come with each unit as two TMA boxes
    int ns;
};

constexpr int kWideTabGroups = 4;   // groups per table box (16 bytes of a table row)
constexpr uint32_t kWideTabBytes = (uint32_t)kWideRows * kWideTabGroups * 4;

template <int F, int BITS>
struct WideShape {
    static constexpr int H = (BITS == 4 && F == 128) ? 2 : 1;   // 16-byte pieces per lane and digit tile
    static constexpr int KS = 2 * H;                           // k-steps (32 codes each) per fold block
    static constexpr int RB = F * BITS / 8;                     // code bytes per row per fold block
    static constexpr int WPT = RB / 16;                         // code words a thread reads per row
    static constexpr uint32_t CODE_BYTES = (uint32_t)kWideRows * RB;
    static_assert(BITS == 8 ? F == 64 : (F == 128 || F == 64), "fold block");
    static_assert(WPT == 4 || WPT == 2, "fragment load width");
    __host__ __device__ static constexpr uint32_t dig_bytes(int nt) {
        return (uint32_t)(kWideLimbs * nt * H * kWidePiece);
    }
    __host__ __device__ static constexpr uint32_t rec_bytes(int nt) { return dig_bytes(nt) + (uint32_t)(8 * nt * 8); }
};

// Not volatile: the MMA touches only its registers, so the compiler may
// interleave independent MMAs with each other and with the loads.
__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Stream-K bookkeeping: CTA c of P holds units [start(c), start(c + 1)).
__device__ __forceinline__ int64_t unit_start(int64_t c, int64_t units, int64_t P) { return c * units / P; }
__device__ __forceinline__ int64_t unit_owner(int64_t u, int64_t units, int64_t P) { return ((u + 1) * P - 1) / units; }

// ---- prep: digit records ---------------------------------------------------
// Block (f, n): fold block f, batch rows 8n .. 8n + 7 (one warp each).
template <int F, int BITS>
__global__ void __launch_bounds__(256) prep_digits_kernel(const float* x, const float* channel, int B, int K,
                                                          int nt, uint32_t rec_bytes, unsigned char* rec,
                                                          int* counters, int ncounters) {
    using S = WideShape<F, BITS>;
    __shared__ int xs[8][F];
    // x may be the previous kernel's output; the dequant kernel that follows
    // waits for this one to complete before it reads the records
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int f = blockIdx.x, n = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (f == 0 && n == 0)
        for (int i = threadIdx.x; i < ncounters; i += blockDim.x) counters[i] = 0;
    const int b = n * 8 + warp;
    const bool real = b < B;
    constexpr int V = F / 32;
    float v[V];
    float m = 0.0f;
    bool bad = false;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int k = f * F + i * 32 + lane;
        float tv = 0.0f;
        if (real && k < K) {
            tv = x[(int64_t)b * K + k];
            if (channel != nullptr) tv = tv * channel[k];
        }
        v[i] = tv;
        bad |= !(fabsf(tv) <= 3.4028235e38f);   // inf or NaN
        m = fmaxf(m, fabsf(tv));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    bad = __any_sync(0xffffffffu, bad);
    // m < 2^e with e = biased exponent - 126 (m = 0 and subnormal m give
    // e <= -126, raised to -100 so that both scalings stay normal)
    const int E = (int)((__float_as_uint(m) >> 23) & 0xFFu);
    int e = E - 126;
    e = e < -100 ? -100 : e;
    const float sc = pow2i(22 - e);
    const float pw = bad ? __int_as_float(0x7fc00000) : pow2i(e - 22);
    int sx = 0;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int xi = bad ? 0 : __float2int_rn(v[i] * sc);   // exact scaling, then round half to even
        sx += xi;
        xs[warp][i * 32 + lane] = xi;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sx += __shfl_xor_sync(0xffffffffu, sx, off);
    unsigned char* r = rec + (size_t)f * rec_bytes;
    if (lane == 0) *reinterpret_cast<float2*>(r + S::dig_bytes(nt) + (size_t)b * 8) = make_float2(pw, (float)sx);
    __syncwarp();
    // one 16-byte piece per lane: digit l, thread-in-group tq, piece h
    constexpr int NP = kWideLimbs * 4 * S::H;
    if (lane < NP) {
        const int l = lane / (4 * S::H), rem = lane % (4 * S::H);
        const int tq = rem / S::H, h = rem % S::H;
        const int p16 = (BITS == 4 && F == 128) ? 2 * tq + h : tq;   // the piece covers codes 16 p16 .. 16 p16 + 15
        const int* xp = &xs[warp][16 * p16];
        uint32_t wv[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t word = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int jj = 4 * q + j;
                // int4: per code word, its codes 0, 2, 4, 6 then 1, 3, 5, 7; int8: in order
                const int code = BITS == 4 ? (jj >> 3) * 8 + 2 * (jj & 3) + ((jj >> 2) & 1) : jj;
                const uint32_t u = (uint32_t)(xp[code] + (int)kWideBias);   // in [0, 2^24)
                // unsigned digit n encodes n - 128, as a signed byte that is n ^ 0x80
                word |= (((u >> (8 * l)) & 0xFFu) ^ 0x80u) << (8 * j);
            }
            wv[q] = word;
        }
        *reinterpret_cast<uint4*>(r + (size_t)((l * nt + n) * S::H + h) * kWidePiece + (size_t)(4 * warp + tq) * 16) =
            make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
}

// ---- the dequant-GEMM -------------------------------------------------------
// Warps: WARPS multiply warps of MT 16-row MMA tiles each (256 rows), then one
// producer warp. With the producer's own warp every stage is refilled the
// moment the last multiply warp releases it (at small batches the load
// stream, not the multiply warps, sets the pace), and nine warps leave 168
// registers a thread: batch tiles are accumulated in passes of NG.
template <int NT, int MT>
struct WideCfg {
    static constexpr int WARPS = 16 / MT;
    static constexpr int THREADS = WARPS * 32 + 32;   // + the producer warp
    static constexpr int MMA_THREADS = WARPS * 32;
    static constexpr int NG = NT < 2 ? NT : 2;        // batch tiles per accumulation pass
    static constexpr int E = 4 * MT * NT;             // fp32 accumulators per thread
    static_assert(WARPS * MT * 16 == kWideRows, "a row block is one TMA box of rows");
};

template <int NT, int F, int BITS, int MT>
__global__ void __launch_bounds__(WideCfg<NT, MT>::THREADS, 1)
    gemv_wide_kernel(const WideParams p, const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap ms,
                     const __grid_constant__ CUtensorMap mz) {
    using S = WideShape<F, BITS>;
    using C = WideCfg<NT, MT>;
    constexpr int E = C::E;
    constexpr int NG = C::NG;
    extern __shared__ unsigned char smem_raw[];
    // stages start on a 1024-byte boundary (TMA destinations need 128)
    const uint32_t raw = smem_addr(smem_raw);
    unsigned char* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    unsigned char* stages = base;
    uint64_t* full = reinterpret_cast<uint64_t*>(base + (size_t)p.ns * p.stage_bytes);
    uint64_t* consumed = full + p.ns;
    volatile int* flag = reinterpret_cast<volatile int*>(consumed + p.ns);
    const uint32_t full0 = smem_addr(full), cons0 = smem_addr(consumed);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int64_t P = gridDim.x, cta = blockIdx.x;
    const int64_t u0 = unit_start(cta, p.units, P), u1 = unit_start(cta + 1, p.units, P);
    if (warp == C::WARPS && lane == 0) {
        for (int s = 0; s < p.ns; ++s) {
            mbar_init(full0 + 8u * (uint32_t)s, 1);
            mbar_init(cons0 + 8u * (uint32_t)s, (uint32_t)C::WARPS);
        }
        fence_mbarrier_init();
    }
    __syncthreads();
    // the prep kernel's records and counters
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (warp == C::WARPS) {
        // ---- producer warp: one code box, two table boxes and one record per unit
        if (lane == 0) {
            bool faulted = false;
            uint32_t filled = 0, fill_par = 0;
            int s = 0;
            uint32_t round = 0;
            int rb = (int)(u0 / p.nfb), fb = (int)(u0 % p.nfb);
            for (int64_t u = u0; u < u1; ++u) {
                if (round > 0 && !mbar_wait_bounded(cons0 + 8u * (uint32_t)s, (round - 1u) & 1u)) {
                    faulted = true;
                    atomicOr(p.fault, 1u);
                }
                if (faulted) break;
                const uint32_t dst = smem_addr(stages + (size_t)s * p.stage_bytes);
                const uint32_t bar = full0 + 8u * (uint32_t)s;
                fence_proxy_async_smem();   // the consumers' reads of the stage before the copies refill it
                mbar_arrive_expect_tx(bar, S::CODE_BYTES + p.rec_bytes + (p.tab_box ? 2u * kWideTabBytes : 0u));
                tma_load_2d(dst, &mq, fb * S::RB, rb * kWideRows, bar);
                if (p.tab_box) {
                    // the 4-group column of both tables that holds this unit's group
                    const int gi = p.fold_per_group > 0 ? fb / p.fold_per_group : 0;
                    const int gx = gi & ~(kWideTabGroups - 1);
                    tma_load_2d(dst + p.tab_off, &ms, gx, rb * kWideRows, bar);
                    tma_load_2d(dst + p.tab_off + kWideTabBytes, &mz, gx, rb * kWideRows, bar);
                }
                bulk_copy_g2s(dst + S::CODE_BYTES, p.rec + (int64_t)fb * p.rec_bytes, p.rec_bytes, bar);
                filled |= 1u << s;
                fill_par ^= 1u << s;
                if (++fb == p.nfb) {
                    fb = 0;
                    ++rb;
                }
                if (++s == p.ns) {
                    s = 0;
                    ++round;
                }
            }
            // Copies issued before a fault may still be in flight into this
            // CTA's shared memory: wait (bounded) for the last fill of every
            // stage. In a fault-free run those phases have completed already.
            for (int i = 0; i < p.ns; ++i) {
                if (((filled >> i) & 1u) && !mbar_wait_bounded(full0 + 8u * (uint32_t)i, ((fill_par >> i) & 1u) ^ 1u))
                    atomicOr(p.fault, 1u);
            }
        }
        return;
    }

    // ---- multiply warps ---------------------------------------------------------
    // The CTA's run of units is walked one row-block segment at a time: the
    // units of a segment, then the segment's output. Per unit a warp waits for
    // the stage, loads its code words, runs the MMAs of every batch tile (in
    // passes of NG tiles, each folded into the fp32 accumulators right
    // after its MMAs) and releases the stage. With one batch tile (up to 8
    // batch rows) a unit is short, so two units are taken per iteration: their
    // loads, MMAs and folds interleave, which hides the shared-memory and
    // barrier latencies of one behind the work of the other.
    const int g = lane >> 2;   // MMA group: rows g and g + 8, B column g
    const int t = lane & 3;    // thread in group: C columns 2t and 2t + 1
    const int wrow = warp * (MT * 16);   // this warp's first row in the row block
    float acc[E];
#pragma unroll
    for (int i = 0; i < E; ++i) acc[i] = 0.0f;
    bool faulted = false;

    // y (+ bias) into every output of rows blk*256 + this thread's rows
    auto write_out = [&](int blk, const float (&val)[E]) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const int row = blk * kWideRows + wrow + mt * 16 + g + 8 * rr;
                if (row >= p.M) continue;
                const float bv = p.bias != nullptr ? p.bias[row] : 0.0f;
#pragma unroll
                for (int ng = 0; ng < NT; ++ng) {
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {
                        const int b = 8 * ng + 2 * t + cc;
                        if (b >= p.B) continue;
                        float v = val[((mt * 2 + rr) * NT + ng) * 2 + cc];
                        if (p.bias != nullptr) v = __fadd_rn(v, bv);   // linear.py:99-100
                        const int64_t off = (int64_t)b * p.ldy + row;
                        if (p.y_all != nullptr) {
                            asm volatile("multimem.st.global.f32 [%0], %1;" ::"l"(p.y_all + off), "f"(v) : "memory");
                        } else {
                            p.y[off] = v;
                            for (int d = 0; d < p.n_extra; ++d) p.y_extra[d][off] = v;
                        }
                    }
                }
            }
        }
    };

    // End of a row block's segment (units seg_first .. seg_last of row block
    // blk): write y, or this CTA's partial rows and, by the last CTA to arrive,
    // the fixed-order sum. Then the fp32 accumulators start again from zero.
    auto flush = [&](int blk, int64_t seg_first, int64_t seg_last) {
        const int64_t ub = (int64_t)blk * p.nfb, ue = ub + p.nfb;
        if (seg_first == ub && seg_last == ue - 1) {
            write_out(blk, acc);
        } else {
            // slot 1 when the CTA's run started in an earlier row block, else 0
            const int which = u0 < ub ? 1 : 0;
            float* dst = p.part + ((size_t)(2 * cta + which) * C::MMA_THREADS + threadIdx.x) * E;
#pragma unroll
            for (int i = 0; i < E; i += 4)
                __stcg(reinterpret_cast<float4*>(dst + i), make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]));
            __threadfence();
            named_barrier(1, C::MMA_THREADS);
            const int64_t cf = unit_owner(ub, p.units, P), cl = unit_owner(ue - 1, p.units, P);
            if (threadIdx.x == 0) {
                const int old = atomicAdd(p.counters + blk, 1);
                *flag = old == (int)(cl - cf) ? 1 : 0;
            }
            named_barrier(1, C::MMA_THREADS);
            if (*flag) {
                __threadfence();
                float sum[E];
#pragma unroll
                for (int i = 0; i < E; ++i) sum[i] = 0.0f;
                // Small layers give a row block dozens of contributors: the
                // slots are loaded U at a time (U x E floats in registers,
                // which the accumulators no longer hold) and added in CTA order.
                constexpr int U = E <= 8 ? 8 : (E <= 16 ? 4 : 2);
                auto slot = [&](int64_t c) {
                    const int wh = unit_start(c, p.units, P) < ub ? 1 : 0;
                    return p.part + ((size_t)(2 * c + wh) * C::MMA_THREADS + threadIdx.x) * E;
                };
                int64_t c = cf;
#pragma unroll 1
                for (; c + U - 1 <= cl; c += U) {
                    float4 q[U][E / 4];
#pragma unroll
                    for (int j = 0; j < U; ++j) {
                        const float* src = slot(c + j);
#pragma unroll
                        for (int i = 0; i < E / 4; ++i) q[j][i] = __ldcg(reinterpret_cast<const float4*>(src) + i);
                    }
#pragma unroll
                    for (int j = 0; j < U; ++j) {
#pragma unroll
                        for (int i = 0; i < E / 4; ++i) {
                            sum[4 * i] += q[j][i].x;
                            sum[4 * i + 1] += q[j][i].y;
                            sum[4 * i + 2] += q[j][i].z;
                            sum[4 * i + 3] += q[j][i].w;
                        }
                    }
                }
#pragma unroll 1
                for (; c <= cl; ++c) {
                    const float* src = slot(c);
#pragma unroll
                    for (int i = 0; i < E; i += 4) {
                        const float4 q = __ldcg(reinterpret_cast<const float4*>(src + i));
                        sum[i] += q.x;
                        sum[i + 1] += q.y;
                        sum[i + 2] += q.z;
                        sum[i + 3] += q.w;
                    }
                }
                write_out(blk, sum);
            }
        }
#pragma unroll
        for (int i = 0; i < E; ++i) acc[i] = 0.0f;
    };

    using Words = uint32_t[MT][2][S::WPT];
    using Tab = float[MT][2];
    using Acc = int[MT][kWideLimbs][NG][4];

    // stage ring position of the next unit
    int s = 0;
    uint32_t par = 0;
    auto next_stage = [&](int& st, uint32_t& pr) {
        st = s;
        pr = par;
        if (++s == p.ns) {
            s = 0;
            par ^= 1u;
        }
    };
    auto stage_wait = [&](int st, uint32_t pr) {
        if (!faulted && !mbar_wait_bounded(full0 + 8u * (uint32_t)st, pr)) {
            faulted = true;
            atomicOr(p.fault, 1u);
        }
    };
    auto release = [&](int st) {
        // mbarrier.arrive releases: this warp's shared-memory reads of the
        // stage, all earlier in program order, are ordered before the refill
        __syncwarp();
        if (lane == 0) mbar_arrive(cons0 + 8u * (uint32_t)st);
    };
    // this thread's code words of rows g, g + 8 of both row tiles
    auto load_codes = [&](const unsigned char* stg, Words& aw) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const unsigned char* src = stg + (size_t)(wrow + mt * 16 + g + 8 * rr) * S::RB + t * (S::RB / 4);
                if constexpr (S::WPT == 4) {
                    const uint4 q4 = *reinterpret_cast<const uint4*>(src);
                    aw[mt][rr][0] = q4.x;
                    aw[mt][rr][1] = q4.y;
                    aw[mt][rr][2] = q4.z;
                    aw[mt][rr][3] = q4.w;
                } else {
                    const uint2 q2 = *reinterpret_cast<const uint2*>(src);
                    aw[mt][rr][0] = q2.x;
                    aw[mt][rr][1] = q2.y;
                }
            }
        }
    };
    // scales and zeros of unit (blk, f), this thread's rows: from global memory
    // (issued before the stage wait), or from the stage's table boxes
    auto tables_global = [&](int blk, int f, Tab& sc, Tab& zr) {
        const int gi = p.fold_per_group > 0 ? f / p.fold_per_group : 0;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const int row = blk * kWideRows + wrow + mt * 16 + g + 8 * rr;
                sc[mt][rr] = zr[mt][rr] = 0.0f;
                if (row < p.M) {
                    const int64_t idx = p.scale_rows == 1 ? (int64_t)gi : (int64_t)row * p.groups + gi;
                    sc[mt][rr] = __ldg(p.scales + idx);
                    zr[mt][rr] = __ldg(p.zeros + idx);
                }
            }
        }
    };
    auto tables_stage = [&](const unsigned char* stg, int f, Tab& sc, Tab& zr) {
        const int gi = p.fold_per_group > 0 ? f / p.fold_per_group : 0;
        const float* ts = reinterpret_cast<const float*>(stg + p.tab_off);   // rows past M are zero-filled
        const float* tz = ts + kWideRows * kWideTabGroups;
        const int gc = gi & (kWideTabGroups - 1);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const int r = wrow + mt * 16 + g + 8 * rr;
                sc[mt][rr] = ts[r * kWideTabGroups + gc];
                zr[mt][rr] = tz[r * kWideTabGroups + gc];
            }
        }
    };
    // the MMAs of batch tiles ng0 .. ng0 + NG - 1 of one unit
    auto mma_pass = [&](const unsigned char* rec, const Words& aw, const int ng0, Acc& c) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int l = 0; l < kWideLimbs; ++l)
#pragma unroll
                for (int j = 0; j < NG; ++j)
#pragma unroll
                    for (int i = 0; i < 4; ++i) c[mt][l][j][i] = 0;
#pragma unroll
        for (int h = 0; h < S::H; ++h) {
            // A fragments of k-steps 2h and 2h + 1
            uint32_t af[MT][2][4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
                for (int ss = 0; ss < 2; ++ss) {
                    const int ks = 2 * h + ss;
                    if constexpr (BITS == 4) {
                        af[mt][ss][0] = aw[mt][0][ks] & 0x0F0F0F0Fu;
                        af[mt][ss][1] = aw[mt][1][ks] & 0x0F0F0F0Fu;
                        af[mt][ss][2] = (aw[mt][0][ks] >> 4) & 0x0F0F0F0Fu;
                        af[mt][ss][3] = (aw[mt][1][ks] >> 4) & 0x0F0F0F0Fu;
                    } else {
                        af[mt][ss][0] = aw[mt][0][2 * ks];
                        af[mt][ss][1] = aw[mt][1][2 * ks];
                        af[mt][ss][2] = aw[mt][0][2 * ks + 1];
                        af[mt][ss][3] = aw[mt][1][2 * ks + 1];
                    }
                }
            }
            // B fragments of both k-steps for every digit and batch tile
            uint4 bq[kWideLimbs][NG];
#pragma unroll
            for (int l = 0; l < kWideLimbs; ++l)
#pragma unroll
                for (int j = 0; j < NG; ++j)
                    if (ng0 + j < NT)
                        bq[l][j] = *reinterpret_cast<const uint4*>(
                            rec + (size_t)((l * NT + ng0 + j) * S::H + h) * kWidePiece + (size_t)lane * 16);
            // k-step outermost: consecutive MMAs write different accumulators
#pragma unroll
            for (int ss = 0; ss < 2; ++ss)
#pragma unroll
                for (int l = 0; l < kWideLimbs; ++l)
#pragma unroll
                    for (int j = 0; j < NG; ++j) {
                        if (ng0 + j >= NT) continue;
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt)
                            mma_u8s8(c[mt][l][j], af[mt][ss][0], af[mt][ss][1], af[mt][ss][2], af[mt][ss][3],
                                     ss ? bq[l][j].z : bq[l][j].x, ss ? bq[l][j].w : bq[l][j].y);
                    }
        }
    };
    // fold factors of this lane's batch columns 8 ng + 2t, 8 ng + 2t + 1
    auto load_fbt = [&](const unsigned char* rec, const int ng0, float4 (&f)[NG]) {
#pragma unroll
        for (int j = 0; j < NG; ++j)
            if (ng0 + j < NT)
                f[j] = *reinterpret_cast<const float4*>(rec + S::dig_bytes(NT) + (size_t)(8 * (ng0 + j) + 2 * t) * 8);
    };
    // fold: C[m, n] of digit l, row g or g + 8 (rr), batch column 2t + cc
    auto fold = [&](const Acc& c, const int ng0, const float4 (&f)[NG], const Tab& sc, const Tab& zr) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
#pragma unroll
                for (int j = 0; j < NG; ++j) {
                    if (ng0 + j >= NT) continue;
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {
                        const int i = 2 * rr + cc;
                        const int c01 = c[mt][0][j][i] + 256 * c[mt][1][j][i];   // exact in s32
                        float v = fmaf((float)c[mt][2][j][i], 65536.0f, (float)c01);
                        const float pw = cc ? f[j].z : f[j].x;
                        const float sx = cc ? f[j].w : f[j].y;
                        v = fmaf(-zr[mt][rr], sx, v);
                        float& a = acc[((mt * 2 + rr) * NT + ng0 + j) * 2 + cc];
                        a = fmaf(sc[mt][rr] * pw, v, a);
                    }
                }
            }
        }
    };

    // one unit (row block blk, fold block f)
    auto one_unit = [&](int blk, int f) {
        int st;
        uint32_t pr;
        next_stage(st, pr);
        Tab sc, zr;
        if (!p.tab_box) tables_global(blk, f, sc, zr);
        stage_wait(st, pr);
        const unsigned char* stg = stages + (size_t)st * p.stage_bytes;
        const unsigned char* rec = stg + S::CODE_BYTES;
        Words aw;
        load_codes(stg, aw);
        if (p.tab_box) tables_stage(stg, f, sc, zr);
#pragma unroll
        for (int ng0 = 0; ng0 < NT; ng0 += NG) {
            Acc c;
            mma_pass(rec, aw, ng0, c);
            float4 fbt[NG];
            load_fbt(rec, ng0, fbt);
            if (ng0 + NG >= NT) release(st);
            fold(c, ng0, fbt, sc, zr);
        }
    };
    // two consecutive units of one row block (one batch tile only)
    auto two_units = [&](int blk, int f) {
        int st0, st1;
        uint32_t pr0, pr1;
        next_stage(st0, pr0);
        next_stage(st1, pr1);
        Tab sc0, zr0, sc1, zr1;
        if (!p.tab_box) {
            tables_global(blk, f, sc0, zr0);
            tables_global(blk, f + 1, sc1, zr1);
        }
        stage_wait(st0, pr0);
        stage_wait(st1, pr1);
        const unsigned char* stg0 = stages + (size_t)st0 * p.stage_bytes;
        const unsigned char* stg1 = stages + (size_t)st1 * p.stage_bytes;
        Words aw0, aw1;
        load_codes(stg0, aw0);
        load_codes(stg1, aw1);
        if (p.tab_box) {
            tables_stage(stg0, f, sc0, zr0);
            tables_stage(stg1, f + 1, sc1, zr1);
        }
        Acc c0, c1;
        mma_pass(stg0 + S::CODE_BYTES, aw0, 0, c0);
        mma_pass(stg1 + S::CODE_BYTES, aw1, 0, c1);
        float4 f0[NG], f1[NG];
        load_fbt(stg0 + S::CODE_BYTES, 0, f0);
        load_fbt(stg1 + S::CODE_BYTES, 0, f1);
        release(st0);
        release(st1);
        fold(c0, 0, f0, sc0, zr0);   // in unit order, as one_unit would
        fold(c1, 0, f1, sc1, zr1);
    };

    int64_t u = u0;
#pragma unroll 1
    while (u < u1) {
        const int blk = (int)(u / p.nfb);
        const int64_t seg_first = u;
        const int64_t row_end = (int64_t)(blk + 1) * p.nfb;
        const int64_t seg_end = u1 < row_end ? u1 : row_end;
        int f = (int)(u - (int64_t)blk * p.nfb);
        if constexpr (NT == 1) {
#pragma unroll 1
            for (; u + 1 < seg_end; u += 2, f += 2) two_units(blk, f);
        }
#pragma unroll 1
        for (; u < seg_end; ++u, ++f) one_unit(blk, f);
        flush(blk, seg_first, seg_end - 1);
    }
}

// ---- host side ------------------------------------------------------------------
constexpr size_t kWideSmemMax = 227 * 1024;

struct WidePlan {
    int F, NT, H, RB;
    int nfb, nrb;
    int64_t units;
    int grid;
    uint32_t rec_bytes, stage_bytes, tab_off;
    int tab_box;
    int ns;
    size_t smem;
};

int64_t round256(int64_t v) { return (v + 255) / 256 * 256; }

// tab_box: the layer's scale and zero tables come by TMA with every unit
// (they only shape the stages, not the workspace).
bool wide_plan(int64_t B, int64_t M, int64_t K, int group_size, int bits, bool tab_box, WidePlan& pl) {
    if (B < kWideMinBatch || B > kWideMaxBatch || M < 1 || K < 1 || group_size < 1) return false;
    if (bits != 4 && bits != 8) return false;
    if (M > ((int64_t)1 << 30) || K > ((int64_t)1 << 30)) return false;
    const bool one_group = group_size >= K;
    if (bits == 4)
        pl.F = (one_group || group_size % 128 == 0) ? 128 : (group_size % 64 == 0 ? 64 : 0);
    else
        pl.F = (one_group || group_size % 64 == 0) ? 64 : 0;
    if (pl.F == 0) return false;
    pl.NT = (int)((B + 7) / 8);
    pl.H = (bits == 4 && pl.F == 128) ? 2 : 1;
    pl.RB = pl.F * bits / 8;
    pl.nfb = (int)((K + pl.F - 1) / pl.F);
    pl.nrb = (int)((M + kWideRows - 1) / kWideRows);
    pl.units = (int64_t)pl.nfb * pl.nrb;
    const int sms = sm_count();
    if (sms < 1) return false;
    pl.grid = pl.units < sms ? (int)pl.units : sms;
    pl.rec_bytes = (uint32_t)(kWideLimbs * pl.NT * pl.H * kWidePiece + 64 * pl.NT);
    uint32_t stage = (uint32_t)kWideRows * (uint32_t)pl.RB + pl.rec_bytes;
    pl.tab_box = tab_box ? 1 : 0;
    pl.tab_off = (stage + 127u) / 128u * 128u;
    if (tab_box) stage = pl.tab_off + 2u * kWideTabBytes;
    pl.stage_bytes = (stage + 1023u) / 1024u * 1024u;
    const size_t tail = 1024 + 16 * kWideMaxStages + 16;   // base alignment, barriers, flag
    size_t ns = (kWideSmemMax - tail) / pl.stage_bytes;
    if (ns > (size_t)kWideMaxStages) ns = kWideMaxStages;
    if (ns < 2) return false;
    pl.ns = (int)ns;
    pl.smem = ns * pl.stage_bytes + tail;
    return true;
}

// Workspace: [records: nfb * rec_bytes][partial rows: 2 * grid * 256 * 8 NT floats][counters: nrb ints]
struct WideWorkspace {
    unsigned char* rec;
    float* part;
    int* counters;
};

size_t wide_bytes(const WidePlan& pl) {
    return (size_t)(round256((int64_t)pl.nfb * pl.rec_bytes) +
                    round256((int64_t)2 * pl.grid * kWideRows * 8 * pl.NT * 4) + round256((int64_t)pl.nrb * 4));
}

WideWorkspace wide_carve(void* ws, const WidePlan& pl) {
    unsigned char* q = static_cast<unsigned char*>(ws);
    WideWorkspace w;
    w.rec = q;
    q += round256((int64_t)pl.nfb * pl.rec_bytes);
    w.part = reinterpret_cast<float*>(q);
    q += round256((int64_t)2 * pl.grid * kWideRows * 8 * pl.NT * 4);
    w.counters = reinterpret_cast<int*>(q);
    return w;
}

cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t s, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

template <int F, int BITS>
cudaError_t launch_prep(const GemmProblem& g, const WidePlan& pl, const WideWorkspace& w, cudaStream_t s) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_config(dim3((unsigned)pl.nfb, (unsigned)pl.NT), dim3(256), 0, s, attr);
    return cudaLaunchKernelEx(&cfg, prep_digits_kernel<F, BITS>, g.x, g.channel, (int)g.B, (int)g.K, pl.NT,
                              pl.rec_bytes, w.rec, w.counters, pl.nrb);
}

struct WideMaps {
    CUtensorMap q, s, z;
};

template <int NT, int F, int BITS>
cudaError_t launch_main(const WideParams& p, const WideMaps& m, const WidePlan& pl, cudaStream_t s) {
    constexpr int MT = 2;   // 8 multiply warps of two row tiles
    auto kern = gemv_wide_kernel<NT, F, BITS, MT>;
    // the shared-memory opt-in is set once per device and size (the last size is kept)
    constexpr int kDevs = 32;
    static std::atomic<size_t> opted[kDevs];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kDevs || opted[dev].load(std::memory_order_relaxed) != pl.smem) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < kDevs) opted[dev].store(pl.smem, std::memory_order_relaxed);
    }
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_config(dim3((unsigned)pl.grid), dim3(WideCfg<NT, MT>::THREADS), pl.smem, s, attr);
    return cudaLaunchKernelEx(&cfg, kern, p, m.q, m.s, m.z);
}

template <int F, int BITS>
cudaError_t launch_fb(const GemmProblem& g, const WidePlan& pl, const WideWorkspace& w, const WideParams& p,
                      const WideMaps& mq, cudaStream_t s) {
    cudaError_t e = launch_prep<F, BITS>(g, pl, w, s);
    if (e != cudaSuccess) return e;
    switch (pl.NT) {
        case 1: return launch_main<1, F, BITS>(p, mq, pl, s);
        case 2: return launch_main<2, F, BITS>(p, mq, pl, s);
        case 3: return launch_main<3, F, BITS>(p, mq, pl, s);
        default: return launch_main<4, F, BITS>(p, mq, pl, s);
    }
}

}  // namespace

// Above 16 batch rows this kernel is bound by its MMA count (3 digits x
// ceil(B / 8) tiles); there the tcgen05 kernel with split-K is faster on
// small layers (measured: 4096 x 4095 at batch 32, 47 us here against 37 us),
// and this one on large ones (28672 x 8192 at batch 32: 104 us against 136).
constexpr int64_t kWideMinCodesAbove16 = (int64_t)1 << 25;

bool wide_supported(const GemmProblem& g) {
    if (g.B > 16 && g.M * g.K < kWideMinCodesAbove16) return false;
    WidePlan pl;
    if (!wide_plan(g.B, g.M, g.K, g.group_size, g.bits, false, pl)) return false;
    if (g.groups > 1 && g.group_size % pl.F != 0) return false;
    if (g.q_stride % 16 != 0 || (reinterpret_cast<uintptr_t>(g.q) & 15) != 0) return false;
    return encode_fn() != nullptr;
}

size_t wide_workspace_bytes(int64_t B, int64_t M, int64_t K, int group_size, int bits) {
    WidePlan pl;
    if (!wide_plan(B, M, K, group_size, bits, false, pl)) return 0;
    return wide_bytes(pl) + 256;
}

cudaError_t launch_wide(const GemmProblem& g, void* workspace, cudaStream_t s) {
    // per-row tables whose rows are whole 16-byte multiples come by TMA
    const bool tab_box = g.scale_rows == g.M && g.groups % kWideTabGroups == 0 &&
                         (reinterpret_cast<uintptr_t>(g.scales) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(g.zeros) & 15) == 0;
    WidePlan pl;
    if (!wide_plan(g.B, g.M, g.K, g.group_size, g.bits, tab_box, pl)) return cudaErrorInvalidValue;
    const WideWorkspace w = wide_carve(workspace, pl);
    WideMaps maps;
    memset(&maps, 0, sizeof(maps));
    if (!encode_2d(&maps.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.q, (uint64_t)g.q_stride, (uint64_t)g.M,
                   (uint64_t)g.q_stride, (uint32_t)pl.RB, kWideRows, CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    if (tab_box) {
        const uint64_t row_bytes = (uint64_t)g.groups * 4;
        if (!encode_2d(&maps.s, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.scales, (uint64_t)g.groups, (uint64_t)g.M,
                       row_bytes, kWideTabGroups, kWideRows, CU_TENSOR_MAP_SWIZZLE_NONE) ||
            !encode_2d(&maps.z, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.zeros, (uint64_t)g.groups, (uint64_t)g.M,
                       row_bytes, kWideTabGroups, kWideRows, CU_TENSOR_MAP_SWIZZLE_NONE))
            return cudaErrorInvalidValue;
    }
    WideParams p;
    p.rec = w.rec;
    p.scales = g.scales;
    p.zeros = g.zeros;
    p.bias = g.bias;
    p.y = g.y;
    for (int d = 0; d < 7; ++d) p.y_extra[d] = g.y_extra[d];
    p.n_extra = g.n_extra;
    p.y_all = g.y_all;
    p.part = w.part;
    p.counters = w.counters;
    p.fault = fault_word();
    if (p.fault == nullptr) return cudaErrorInvalidDevicePointer;
    p.M = (int)g.M;
    p.B = (int)g.B;
    p.nfb = pl.nfb;
    p.nrb = pl.nrb;
    p.groups = g.groups;
    p.fold_per_group = g.groups > 1 ? g.group_size / pl.F : 0;
    p.scale_rows = g.scale_rows;
    p.ldy = g.ldy;
    p.units = pl.units;
    p.rec_bytes = pl.rec_bytes;
    p.stage_bytes = pl.stage_bytes;
    p.ns = pl.ns;
    p.tab_off = pl.tab_off;
    p.tab_box = pl.tab_box;
    if (g.bits == 8) return launch_fb<64, 8>(g, pl, w, p, maps, s);
    return pl.F == 128 ? launch_fb<128, 4>(g, pl, w, p, maps, s) : launch_fb<64, 4>(g, pl, w, p, maps, s);
}

}  // namespace wq

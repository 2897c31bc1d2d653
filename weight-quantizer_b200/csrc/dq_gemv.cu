// K1 — streaming decode dequant-GEMM for small batches (B <= 4).
//
// Replaces the per-row dequant + dot of ptqkit's CPU kernel
// (src/ptqkit/csrc/dequant_gemm.cpp:57-218: run_gemm / dequant_row / dots_into)
// for decode-shaped batches, where the packed weight stream from HBM is the
// bound. Same math, y[b,m] = sum_g scale[m,g] * sum_{k in g} (q[m,k]-zero[m,g]) *
// channel[k] * x[b,k], evaluated as
//
//     y[b,m] = sum_chunks scale[m,g] * ( sum_k q[m,k]*x'[b,k]  -  zero[m,g] * sum_k x'[b,k] )
//
// with x' = x * channel and a chunk = the codes of 16 bytes of a row (32 int4 or
// 16 int8 codes, always inside one group).
//
// Mapping ("activation-stationary"). A row slot of WPR warps covers the whole
// K extent of a row: lane l of warp w owns chunks c = (w*32 + l) + j*WPR*32,
// j < NCPL, and keeps x' for those chunks in registers for the entire launch.
// Rows stream past: every iteration a slot takes R consecutive rows, each lane
// multiplies its chunks against its register-resident x', and the row sums are
// reduced over lanes with shuffles and over the slot's warps through shared
// memory, in a fixed order (deterministic, no atomics, no workspace). CTAs are
// persistent, so x is read from L2 once per slot.
//
// Weight stream. One elected thread per slot moves the R rows of codes (and,
// for per-row tables whose row length is a multiple of 16 bytes, their scales
// and zeros) into an NS-deep ring of shared-memory stages with bulk
// asynchronous copies (cp.async.bulk, the TMA unit's linear mode), completing
// on one mbarrier per stage. Lanes then read their 16-byte chunk with one
// shared load: no per-lane address arithmetic or copy instructions. The
// slot barrier that ends every iteration (for the cross-warp reduction) also
// tells the producer that the stage it is about to refill has been consumed.
// Every mbarrier wait is bounded; on expiry the kernel records a fault in the
// library's fault word and runs to completion without waiting again.
//
// Code -> fp32 without conversion instructions. For a 32-bit word of packed
// codes, masking one code in place (w & 0xF << 4p for int4, w & 0xFF << 8p for
// int8) leaves a bit pattern P < 2^24. Read as an IEEE-754 binary32, any such
// pattern has the value P * 2^-149 exactly (exponent field 0 is subnormal,
// field 1 continues the same linear scale). So code * 2^(4p) * 2^-149 is a
// valid FMA operand after one LOP3, and the matching activation is stored
// pre-multiplied by 2^(-4p) * S_b, with S_b = 2^(124 - e_b) a per-batch-row
// power of two chosen from max|x'_b| so that every product lands in the normal
// range. All scalings are exact powers of two; the top byte of a word is
// shifted down once so its codes also sit below bit 24. Products accumulate in
// pairs with the packed fp32 FMA of sm_100 (__ffma2_rn). Subnormal operands
// are handled by FMA at full rate as long as flush-to-zero is off, which is
// the compiler default used for this library.
#include <atomic>
#include <cfloat>

#include "common.cuh"
#include "kernels.h"

namespace wq {
namespace {

template <int BITS>
struct Fmt;
template <>
struct Fmt<4> {
    static constexpr int CH = 32;         // codes per 16-byte chunk
    static constexpr int PER_WORD = 8;    // codes per 32-bit word
};
template <>
struct Fmt<8> {
    static constexpr int CH = 16;
    static constexpr int PER_WORD = 4;
};

// Exponent shift carried by the activation paired with code position i of a
// word (see the extraction in accumulate_word).
template <int BITS>
__device__ __forceinline__ int code_shift(int i) {
    if (BITS == 4) {
        const int p = (i < 6) ? i : i - 6;
        return 4 * p;
    } else {
        const int p = (i < 3) ? i : 0;
        return 8 * p;
    }
}

// One 32-bit word of codes against its activations, held as float2 register
// pairs (the operand form of the packed FMA).
template <int BITS, int NB, int NCPL, int CH2>
__device__ __forceinline__ void accumulate_word(uint32_t w, const float2 (&x2)[NCPL][NB][CH2], int j, int base,
                                                float2 (&acc)[NB]) {
    if (BITS == 4) {
        const uint32_t t = __umulhi(w, 256u);  // w >> 24 on the FMA pipe
        const float2 f01 = make_float2(__uint_as_float(w & 0x0000000Fu), __uint_as_float(w & 0x000000F0u));
        const float2 f23 = make_float2(__uint_as_float(w & 0x00000F00u), __uint_as_float(w & 0x0000F000u));
        const float2 f45 = make_float2(__uint_as_float(w & 0x000F0000u), __uint_as_float(w & 0x00F00000u));
        const float2 f67 = make_float2(__uint_as_float(t & 0x0000000Fu), __uint_as_float(t & 0x000000F0u));
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            acc[b] = __ffma2_rn(f01, x2[j][b][base + 0], acc[b]);
            acc[b] = __ffma2_rn(f23, x2[j][b][base + 1], acc[b]);
            acc[b] = __ffma2_rn(f45, x2[j][b][base + 2], acc[b]);
            acc[b] = __ffma2_rn(f67, x2[j][b][base + 3], acc[b]);
        }
    } else {
        const float2 f01 = make_float2(__uint_as_float(w & 0x000000FFu), __uint_as_float(w & 0x0000FF00u));
        const float2 f23 = make_float2(__uint_as_float(w & 0x00FF0000u), __uint_as_float(__umulhi(w, 256u)));
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            acc[b] = __ffma2_rn(f01, x2[j][b][base + 0], acc[b]);
            acc[b] = __ffma2_rn(f23, x2[j][b][base + 1], acc[b]);
        }
    }
}

struct GemvParams {
    const float* x;
    const uint8_t* q;
    const float* scales;
    const float* zeros;
    const float* channel;
    float* y;
    float* y_extra[7];   // further outputs with y's layout (peer-mapped on other GPUs)
    int n_extra;
    float* y_all;        // NVLink-switch address reaching every rank's y, or nullptr
    const float* bias;   // [M] or nullptr
    unsigned int* fault;
    int M, K, NCH;
    int64_t q_stride, ldy;
    int scale_rows, groups, group_size;
    int wpr;          // warps per row slot
    int slots;        // row slots per CTA
    int ns;           // pipeline stages per slot
    int x_vec4;       // x rows and channel are 16-byte aligned and K % 4 == 0
    int bulk_tables;  // per-row scale/zero tables travel with the codes
    uint32_t stage_bytes;  // bytes of one stage (128-byte multiple)
};

constexpr int kMaxSlots = 8;   // named barriers 1..8 (CTA <= 256 threads)
constexpr int kMaxStages = 8;

// LEAN: per-row scale/zero tables travel with the codes (bulk_tables) and every
// lane's chunks lie inside the row, so the inner loop carries no table-source
// or validity selects.
template <int BITS, int NB, int NCPL, int R, bool LEAN>
__global__ void __launch_bounds__(256) gemv_kernel(const GemvParams p) {
    constexpr int CH = Fmt<BITS>::CH;
    constexpr int PW = Fmt<BITS>::PER_WORD;
    // dynamic smem: stages[slots][ns] (stage_bytes each: codes R*q_stride, then
    // scales R*groups and zeros R*groups fp32 when bulk_tables), then
    // full mbarriers[slots][ns], consumed mbarriers[slots][ns] (8 B each),
    // red[slots][ns][wpr][VPAD], emax[slots][wpr][NB], fills[slots][ns] (u32)
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int slot = warp / p.wpr;
    const int wslot = warp - slot * p.wpr;
    const int slot_threads = p.wpr * 32;
    const int bar_id = slot + 1;
    const bool producer = (wslot == 0 && lane == 0);
    unsigned char* stage_base = smem_raw + (size_t)slot * p.ns * p.stage_bytes;
    uint64_t* mbar_all = reinterpret_cast<uint64_t*>(smem_raw + (size_t)p.slots * p.ns * p.stage_bytes);
    uint64_t* mbar = mbar_all + slot * p.ns;
    uint64_t* cbar = mbar_all + p.slots * p.ns + slot * p.ns;
    constexpr int VPAD = (R * NB) <= 1 ? 1 : ((R * NB) <= 2 ? 2 : ((R * NB) <= 4 ? 4 : 8));
    static_assert(R * NB <= 8, "at most 8 row sums per iteration");
    float* red = reinterpret_cast<float*>(mbar_all + 2 * p.slots * p.ns) + (size_t)slot * p.ns * p.wpr * VPAD;
    float* emax = reinterpret_cast<float*>(mbar_all + 2 * p.slots * p.ns) + (size_t)p.slots * p.ns * p.wpr * VPAD;
    uint32_t* fills = reinterpret_cast<uint32_t*>(emax + p.slots * p.wpr * NB) + slot * p.ns;

    // Programmatic dependent launch: the next kernel on the stream may be
    // scheduled now, and this one reads nothing in global memory before every
    // earlier kernel on the stream has completed (no-ops without the launch
    // attribute).
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int total_slots = (int)gridDim.x * p.slots;
    const int gslot = (int)blockIdx.x * p.slots + slot;
    const int n_iters_total = (p.M + R - 1) / R;
    const uint32_t qs = (uint32_t)p.q_stride;
    const uint32_t codes_bytes = (uint32_t)R * qs;
    const uint32_t table_bytes = (uint32_t)(R * p.groups * 4);
    const uint32_t stage0 = smem_addr(stage_base);
    const uint32_t mbar0 = smem_addr(mbar);
    const uint32_t cbar0 = smem_addr(cbar);

    // producer: bulk-copy iteration `it` into stage `s`
    auto issue = [&](int it, int s) {
        if (it >= n_iters_total) return;
        const int row0 = it * R;
        const int rows = (p.M - row0) < R ? (p.M - row0) : R;
        const uint32_t cb = (uint32_t)rows * qs;
        const uint32_t tb = p.bulk_tables ? (uint32_t)(rows * p.groups * 4) : 0u;
        const uint32_t bar = mbar0 + 8u * (uint32_t)s;
        const uint32_t dst = stage0 + (uint32_t)s * p.stage_bytes;
        mbar_arrive_expect_tx(bar, cb + 2u * tb);
        bulk_copy_g2s(dst, p.q + (int64_t)row0 * p.q_stride, cb, bar);
        ++fills[s];   // only the thread issuing for this slot touches it between barriers
        if (p.bulk_tables) {
            bulk_copy_g2s(dst + codes_bytes, p.scales + (int64_t)row0 * p.groups, tb, bar);
            bulk_copy_g2s(dst + codes_bytes + table_bytes, p.zeros + (int64_t)row0 * p.groups, tb, bar);
        }
    };

    // The weight stream starts before x' is staged: the first NS stages are in
    // flight while the slot loads x, finds max|x'| and scales it.
    if (producer) {
        for (int s = 0; s < p.ns; ++s) {
            mbar_init(smem_addr(mbar + s), 1);
            mbar_init(smem_addr(cbar + s), (uint32_t)p.wpr);   // one arrival per warp of the slot
            fills[s] = 0;
        }
        fence_mbarrier_init();
        for (int s = 0; s < p.ns; ++s) issue(gslot + s * total_slots, s);
    }

    // ---- stage x' = x * channel for this lane's chunks in registers ----------
    float xr[NCPL][NB][CH];
    int cidx[NCPL];
    float mx[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) mx[b] = 0.0f;
#pragma unroll
    for (int j = 0; j < NCPL; ++j) {
        cidx[j] = wslot * 32 + lane + j * p.wpr * 32;
        const int k0 = cidx[j] * CH;
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const float* xb = p.x + (int64_t)b * p.K;
            if (p.x_vec4 && k0 + CH <= p.K) {
#pragma unroll
                for (int i = 0; i < CH; i += 4) {
                    float4 v = __ldg(reinterpret_cast<const float4*>(xb + k0 + i));
                    if (p.channel != nullptr) {
                        const float4 c = __ldg(reinterpret_cast<const float4*>(p.channel + k0 + i));
                        v.x = v.x * c.x; v.y = v.y * c.y; v.z = v.z * c.z; v.w = v.w * c.w;
                    }
                    xr[j][b][i] = v.x; xr[j][b][i + 1] = v.y; xr[j][b][i + 2] = v.z; xr[j][b][i + 3] = v.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < CH; ++i) {
                    const int k = k0 + i;
                    float v = 0.0f;
                    if (k < p.K) {
                        v = __ldg(xb + k);
                        if (p.channel != nullptr) v = v * __ldg(p.channel + k);
                    }
                    xr[j][b][i] = v;
                }
            }
#pragma unroll
            for (int i = 0; i < CH; ++i) mx[b] = fmaxf(mx[b], fabsf(xr[j][b][i]));
        }
    }
    // ---- per batch row exponent e_b from max|x'_b| over the whole row -------
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        float v = mx[b];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) emax[(slot * p.wpr + wslot) * NB + b] = v;
    }
    named_barrier(bar_id, slot_threads);  // also publishes the initialized mbarriers
    int eb[NB];
    float sx[NCPL][NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        float v = 0.0f;
        for (int w = 0; w < p.wpr; ++w) v = fmaxf(v, emax[(slot * p.wpr + w) * NB + b]);
        int e = 0;
        if (v > 0.0f && v <= FLT_MAX) frexpf(v, &e);
        e = e < -120 ? -120 : (e > 128 ? 128 : e);
        eb[b] = e;
        // x'_b * S_b with S_b = 2^(124 - e) <= 2^244 applied as two exact factors.
        const int st = 124 - e;
        const int s1e = st < 120 ? st : 120;
        const float s1 = pow2i(s1e), s2 = pow2i(st - s1e);
#pragma unroll
        for (int j = 0; j < NCPL; ++j) {
            float sum = 0.0f;
#pragma unroll
            for (int i = 0; i < CH; ++i) {
                const float v2 = (xr[j][b][i] * s1) * s2;                // x' * S_b, exact
                sum += (v2 * 0x1p-100f) * 0x1p-49f;                      // x' * S_b * 2^-149
                xr[j][b][i] = v2 * pow2i(-code_shift<BITS>(i % PW));     // paired-code scaling
            }
            sx[j][b] = sum;
        }
    }
    float2 x2[NCPL][NB][CH / 2];
#pragma unroll
    for (int j = 0; j < NCPL; ++j)
#pragma unroll
        for (int b = 0; b < NB; ++b)
#pragma unroll
            for (int i = 0; i < CH / 2; ++i) x2[j][b][i] = make_float2(xr[j][b][2 * i], xr[j][b][2 * i + 1]);

    // ---- loop invariants -------------------------------------------------------
    const bool multi = p.groups > 1;
    int goff[NCPL];
    uint32_t coff[NCPL];
    bool cvalid[NCPL];
    float csc_const[NCPL], czr_const[NCPL];
#pragma unroll
    for (int j = 0; j < NCPL; ++j) {
        cvalid[j] = cidx[j] < p.NCH;
        coff[j] = (uint32_t)cidx[j] * 16u;
        goff[j] = (multi && cvalid[j]) ? (cidx[j] * CH) / p.group_size : 0;
        csc_const[j] = 0.0f;
        czr_const[j] = 0.0f;
        if (p.scale_rows == 1 && cvalid[j]) {  // one table shared by all rows
            csc_const[j] = __ldg(p.scales + goff[j]);
            czr_const[j] = __ldg(p.zeros + goff[j]);
        }
    }

    constexpr int V = R * NB;                         // row sums one iteration produces
    constexpr int VP = V <= 1 ? 1 : (V <= 2 ? 2 : (V <= 4 ? 4 : 8));
    bool faulted = false;
    int s = 0, fin = 0, n_local = 0;
    uint32_t phase = 0;
    for (int it = gslot; it < n_iters_total; it += total_slots) {
        if (!faulted && !mbar_wait_bounded(mbar0 + 8u * (uint32_t)s, phase)) {
            faulted = true;
            atomicOr(p.fault, 1u);
        }
        const unsigned char* stg = stage_base + (size_t)s * p.stage_bytes;
        const float* tsc = reinterpret_cast<const float*>(stg + codes_bytes);
        const float* tzr = reinterpret_cast<const float*>(stg + codes_bytes + table_bytes);

        float yv[VP];
#pragma unroll
        for (int v = 0; v < VP; ++v) yv[v] = 0.0f;
#pragma unroll
        for (int r = 0; r < R; ++r) {
#pragma unroll
            for (int j = 0; j < NCPL; ++j) {
                const uint4 cq = *reinterpret_cast<const uint4*>(stg + (uint32_t)r * qs + coff[j]);
                float sc, zr;
                if constexpr (LEAN) {
                    sc = tsc[r * p.groups + goff[j]];
                    zr = tzr[r * p.groups + goff[j]];
                } else if (p.scale_rows == 1) {
                    sc = csc_const[j];
                    zr = czr_const[j];
                } else if (p.bulk_tables) {
                    sc = tsc[r * p.groups + goff[j]];
                    zr = tzr[r * p.groups + goff[j]];
                } else {
                    const int row = it * R + r;
                    const int rr = row < p.M ? row : p.M - 1;
                    sc = __ldg(p.scales + (int64_t)rr * p.groups + goff[j]);
                    zr = __ldg(p.zeros + (int64_t)rr * p.groups + goff[j]);
                }
                // lanes past the row's last chunk read stale stage bytes (finite
                // once masked, times x' = 0); their scale and zero are forced to 0
                if (!LEAN && !cvalid[j]) {
                    sc = 0.0f;
                    zr = 0.0f;
                }
                // two independent accumulation chains per chunk (words x,z and y,w)
                float2 acc[NB], acc2[NB];
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    acc[b] = make_float2(0.0f, 0.0f);
                    acc2[b] = make_float2(0.0f, 0.0f);
                }
                accumulate_word<BITS, NB, NCPL, CH / 2>(cq.x, x2, j, 0 * (PW / 2), acc);
                accumulate_word<BITS, NB, NCPL, CH / 2>(cq.y, x2, j, 1 * (PW / 2), acc2);
                accumulate_word<BITS, NB, NCPL, CH / 2>(cq.z, x2, j, 2 * (PW / 2), acc);
                accumulate_word<BITS, NB, NCPL, CH / 2>(cq.w, x2, j, 3 * (PW / 2), acc2);
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    const float a = (acc[b].x + acc2[b].x) + (acc[b].y + acc2[b].y);
                    const float t = fmaf(-zr, sx[j][b], a);
                    yv[r * NB + b] = fmaf(sc, t, yv[r * NB + b]);
                }
            }
        }

        // lanes -> one row sum per representative lane (reduce-scatter), then
        // the slot's warps in a fixed order
        int idx = 0;
        const float z = warp_reduce_scatter<VP>(yv, lane, idx);
        float* rb = red + (size_t)s * p.wpr * VPAD;
        if ((lane & (32 / VP - 1)) == 0) rb[wslot * VPAD + idx] = z;
        // This warp is done with stage s and has published its partial sums.
        // No slot-wide barrier: one warp per iteration (rotating) waits for the
        // others, finishes the rows and refills the stage; the rest move on.
        __syncwarp();
        if (lane == 0) mbar_arrive(cbar0 + 8u * (uint32_t)s);
        if (wslot == fin) {
            if (lane == 0 && !faulted && !mbar_wait_bounded(cbar0 + 8u * (uint32_t)s, phase)) {
                faulted = true;
                atomicOr(p.fault, 1u);
            }
            faulted = __shfl_sync(0xffffffffu, faulted ? 1 : 0, 0) != 0;
            __syncwarp();
            if (lane < V) {
                const int r = lane / NB, b = lane - (lane / NB) * NB;
                const int row = it * R + r;
                float v = 0.0f;
                for (int w = 0; w < p.wpr; ++w) v += rb[w * VPAD + lane];
                if (row < p.M) {
                    int e = 0;
#pragma unroll
                    for (int bb = 0; bb < NB; ++bb)
                        if (bb == b) e = eb[bb];
                    const int h = 25 + e, h1 = h / 2;
                    float out = (v * pow2i(h1)) * pow2i(h - h1);
                    if (p.bias != nullptr) out = __fadd_rn(out, p.bias[row]);   // linear.py:99-100
                    const int64_t off = (int64_t)b * p.ldy + row;
                    if (p.y_all != nullptr) {
                        asm volatile("multimem.st.global.f32 [%0], %1;" ::"l"(p.y_all + off), "f"(out) : "memory");
                    } else {
                        p.y[off] = out;
                        for (int d = 0; d < p.n_extra; ++d) p.y_extra[d][off] = out;
                    }
                }
            }
            __syncwarp();
            if (lane == 0 && !faulted) {
                fence_proxy_async_smem();   // the slot's reads of stage s before the bulk copy refills it
                issue(it + p.ns * total_slots, s);
            }
        }
        if (++fin == p.wpr) fin = 0;
        if (++s == p.ns) {
            s = 0;
            phase ^= 1u;
        }
        ++n_local;
    }
    // Copies issued before a fault may still be in flight into this CTA's
    // shared memory: once the whole slot is past its loop, the first warp
    // waits (bounded) for the last fill of every stage. In a fault-free run
    // those phases have completed already.
    named_barrier(bar_id, slot_threads);
    if (wslot == 0 && lane == 0) {
        for (int t = 0; t < p.ns; ++t) {
            const uint32_t n = fills[t];
            if (n > 0 && !mbar_wait_bounded(mbar0 + 8u * (uint32_t)t, (n - 1u) & 1u)) atomicOr(p.fault, 1u);
        }
    }
}

struct Choice {
    int ncpl, wpr, slots;
};

template <int BITS>
bool choose(int NB, int NCH, Choice& c) {
    // chunk slots one lane holds; int4 with 3-4 batch rows keeps one chunk per
    // lane to bound registers (x' for NB*NCPL*CH values lives in registers)
    const int max_ncpl = (BITS == 4 && NB > 2) ? 1 : 2;
    int best_waste = 1 << 30;
    bool found = false;
    for (int ncpl = 1; ncpl <= max_ncpl; ++ncpl) {
        const int wpr = (NCH + 32 * ncpl - 1) / (32 * ncpl);
        if (wpr > 8) continue;
        const int waste = wpr * 32 * ncpl - NCH;
        if (waste < best_waste) {
            best_waste = waste;
            c.ncpl = ncpl;
            c.wpr = wpr;
            found = true;
        }
    }
    if (!found) return false;
    int slots = 256 / (32 * c.wpr);
    if (slots < 1) slots = 1;
    if (slots > kMaxSlots) slots = kMaxSlots;
    c.slots = slots;
    return true;
}

// Shared memory of one SM available to resident CTAs (B200: 228 KB, less a
// 1 KB per-CTA reservation), and the most stages worth keeping in flight.
constexpr size_t kSmemPerSm = 227 * 1024;

template <int BITS, int NB, int NCPL, int R, bool LEAN>
cudaError_t launch_t(GemvParams p, cudaStream_t s) {
    auto kern = gemv_kernel<BITS, NB, NCPL, R, LEAN>;
    const int threads = p.wpr * p.slots * 32;
    const size_t codes_b = (size_t)R * p.q_stride;
    const size_t table_b = p.bulk_tables ? (size_t)R * p.groups * 4 : 0;
    p.stage_bytes = (uint32_t)(((codes_b + 2 * table_b) + 127) / 128 * 128);
    // per stage: a consumed mbarrier and the warps' partial sums; then emax
    const size_t red_b = sizeof(float) * (size_t)p.slots * p.wpr * 8;   // one stage's partial sums
    const size_t tail = sizeof(float) * (size_t)p.slots * p.wpr * NB + sizeof(uint32_t) * (size_t)p.slots * kMaxStages;
    // Host setup cached per device: the kernel's register count, the
    // shared-memory opt-in (set once to the largest size a launch may ask for)
    // and the occupancy of the last (threads, shared memory) pair.
    constexpr int kDevs = 32;
    static std::atomic<int> regs_c[kDevs], optin_c[kDevs];
    static std::atomic<uint64_t> occ_c[kDevs];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const bool cached = dev >= 0 && dev < kDevs;
    int num_regs = cached ? regs_c[dev].load(std::memory_order_relaxed) : 0;
    if (num_regs == 0) {
        cudaFuncAttributes attr;
        e = cudaFuncGetAttributes(&attr, kern);
        if (e != cudaSuccess) return e;
        num_regs = attr.numRegs > 0 ? attr.numRegs : 1;
        if (cached) regs_c[dev].store(num_regs, std::memory_order_relaxed);
    }
    // stages: as many as fit while keeping every CTA the registers allow resident
    int occ_regs = 65536 / (num_regs * threads);
    if (occ_regs < 1) occ_regs = 1;
    if (occ_regs > 4) occ_regs = 4;
    int ns = 0;
    for (int want = occ_regs; want >= 1 && ns < 3; --want) {
        const size_t per_cta = kSmemPerSm / want - 1024;
        ns = (int)((per_cta - tail) / ((size_t)p.slots * (p.stage_bytes + 16) + red_b));
    }
    if (ns > kMaxStages) ns = kMaxStages;
    if (ns < 2) ns = 2;
    p.ns = ns;
    const size_t smem = (size_t)p.slots * ns * p.stage_bytes + 16 * (size_t)p.slots * ns + red_b * ns + tail;
    constexpr int kOptIn = 220 * 1024;
    if (smem > (size_t)kOptIn) return cudaErrorInvalidValue;
    if (!cached || optin_c[dev].load(std::memory_order_relaxed) == 0) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kOptIn);
        if (e != cudaSuccess) return e;
        if (cached) optin_c[dev].store(1, std::memory_order_relaxed);
    }
    const uint64_t key = ((uint64_t)smem << 16) | (uint64_t)threads;   // occupancy in the low byte
    const uint64_t hit = cached ? occ_c[dev].load(std::memory_order_relaxed) : 0;
    int occ = 0;
    if (hit != 0 && (hit >> 8) == key) {
        occ = (int)(hit & 0xFF);
    } else {
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem);
        if (e != cudaSuccess) return e;
        if (occ < 1) return cudaErrorInvalidConfiguration;
        if (cached) occ_c[dev].store((key << 8) | (uint64_t)(occ & 0xFF), std::memory_order_relaxed);
    }
    const int64_t iters = ((int64_t)p.M + R - 1) / R;
    int64_t grid = (int64_t)sm_count() * occ;
    const int64_t need = (iters + p.slots - 1) / p.slots;
    if (grid > need) grid = need;
    if (grid < 1) grid = 1;
    // launched with programmatic stream serialization (see the kernel's first lines)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr_pdl[1];
    attr_pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr_pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr_pdl;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int BITS, bool LEAN>
cudaError_t dispatch_nb(const GemvParams& p, int NB, int ncpl, cudaStream_t s) {
    switch (NB) {
        case 1: return ncpl == 2 ? launch_t<BITS, 1, 2, 4, LEAN>(p, s) : launch_t<BITS, 1, 1, 8, LEAN>(p, s);
        case 2: return ncpl == 2 ? launch_t<BITS, 2, 2, 4, LEAN>(p, s) : launch_t<BITS, 2, 1, 4, LEAN>(p, s);
        case 3:
            if constexpr (BITS == 8) {
                if (ncpl == 2) return launch_t<BITS, 3, 2, 2, LEAN>(p, s);
            }
            return launch_t<BITS, 3, 1, 2, LEAN>(p, s);
        default:
            if constexpr (BITS == 8) {
                if (ncpl == 2) return launch_t<BITS, 4, 2, 2, LEAN>(p, s);
            }
            return launch_t<BITS, 4, 1, 2, LEAN>(p, s);
    }
}

template <int BITS>
cudaError_t dispatch(const GemvParams& p, int NB, int ncpl, bool lean, cudaStream_t s) {
    return lean ? dispatch_nb<BITS, true>(p, NB, ncpl, s) : dispatch_nb<BITS, false>(p, NB, ncpl, s);
}

}  // namespace

size_t gemv_workspace_bytes(int64_t, int64_t, int) { return 0; }

// Batch rows [r0, r0 + nb) of a problem: the same layer, x and every output
// advanced by r0 rows.
static GemmProblem batch_rows(const GemmProblem& g, int64_t r0, int64_t nb) {
    GemmProblem h = g;
    h.B = nb;
    h.x = g.x + r0 * g.K;
    h.y = g.y + r0 * g.ldy;
    for (int d = 0; d < g.n_extra; ++d) h.y_extra[d] = g.y_extra[d] + r0 * g.ldy;
    if (g.y_all != nullptr) h.y_all = g.y_all + r0 * g.ldy;
    return h;
}

// Batches 3-4 that the tensor-core decode kernel takes as two launches.
static bool imma_split(const GemmProblem& p) {
    return (p.B == 3 || p.B == 4) && gemv_imma_supported(batch_rows(p, 0, 2)) &&
           gemv_imma_supported(batch_rows(p, 2, p.B - 2));
}

bool gemv_supported(const GemmProblem& p) {
    if (p.B < 1 || p.B > kGemvMaxBatch || p.K < 1 || p.M < 1) return false;
    if (gemv_imma_supported(p) || imma_split(p)) return true;
    if (p.q_stride % 16 != 0 || (reinterpret_cast<uintptr_t>(p.q) & 15) != 0) return false;
    const int CH = p.bits == 4 ? 32 : 16;
    if (p.groups > 1 && (p.group_size % CH) != 0) return false;
    const int64_t nch = p.q_stride / 16;
    if (nch > (int64_t)8 * 32 * 2) return false;
    if (p.M > ((int64_t)1 << 31) - 64) return false;
    // a stage holds R (<= 4) rows of codes and tables and must fit twice
    if (4 * (p.q_stride + 8 * (int64_t)p.groups) > 48 * 1024) return false;
    Choice c{0, 0, 0};
    const int NB = (int)p.B;
    return p.bits == 4 ? choose<4>(NB, (int)nch, c) : choose<8>(NB, (int)nch, c);
}

cudaError_t launch_gemv(const GemmProblem& g, void* /*workspace*/, cudaStream_t s) {
    if (gemv_imma_supported(g)) return launch_gemv_imma(g, s);
    // Batches 3-4 of an int4 layer the tensor-core decode kernel takes: two
    // passes over the weights (rows 0-1, then the rest) stream less time than
    // one pass of the SIMT kernel, whose activations for 3-4 rows crowd its
    // registers.
    if (imma_split(g)) {
        cudaError_t e = launch_gemv_imma(batch_rows(g, 0, 2), s);
        if (e != cudaSuccess) return e;
        return launch_gemv_imma(batch_rows(g, 2, g.B - 2), s);
    }
    GemvParams p;
    p.x = g.x;
    p.q = g.q;
    p.scales = g.scales;
    p.zeros = g.zeros;
    p.channel = g.channel;
    p.y = g.y;
    p.n_extra = g.n_extra;
    p.y_all = g.y_all;
    p.bias = g.bias;
    for (int d = 0; d < 7; ++d) p.y_extra[d] = g.y_extra[d];
    p.fault = fault_word();
    if (p.fault == nullptr) return cudaErrorInvalidDevicePointer;
    p.M = (int)g.M;
    p.K = (int)g.K;
    p.NCH = (int)(g.q_stride / 16);
    p.q_stride = g.q_stride;
    p.ldy = g.ldy;
    p.scale_rows = g.scale_rows;
    p.groups = g.groups;
    p.group_size = g.group_size;
    p.x_vec4 = (g.K % 4 == 0) && ((reinterpret_cast<uintptr_t>(g.x) & 15) == 0) &&
               (g.channel == nullptr || (reinterpret_cast<uintptr_t>(g.channel) & 15) == 0);
    // per-row tables whose rows are whole 16-byte multiples ride with the codes
    p.bulk_tables = (g.scale_rows != 1) && (g.groups % 4 == 0) &&
                    ((reinterpret_cast<uintptr_t>(g.scales) & 15) == 0) &&
                    ((reinterpret_cast<uintptr_t>(g.zeros) & 15) == 0);
    p.ns = 2;
    p.stage_bytes = 0;
    Choice c{0, 0, 0};
    const int NB = (int)g.B;
    const bool ok = g.bits == 4 ? choose<4>(NB, p.NCH, c) : choose<8>(NB, p.NCH, c);
    if (!ok) return cudaErrorInvalidValue;
    p.wpr = c.wpr;
    p.slots = c.slots;
    const bool lean = p.bulk_tables && c.wpr * 32 * c.ncpl == p.NCH;
    return g.bits == 4 ? dispatch<4>(p, NB, c.ncpl, lean, s) : dispatch<8>(p, NB, c.ncpl, lean, s);
}

}  // namespace wq

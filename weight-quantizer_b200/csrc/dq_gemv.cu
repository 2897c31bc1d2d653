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
// with x' = x * channel and a chunk = the codes of one 16-byte load (32 int4 or
// 16 int8 codes, always inside one group).
//
// Mapping ("activation-stationary"). A row slot of WPR warps covers the whole
// K extent of a row: lane l of warp w owns chunks c = (w*32 + l) + j*WPR*32,
// j < NCPL, and keeps x' for those chunks in registers for the entire launch.
// Rows then stream past: every iteration a slot loads R rows' 16-byte chunks
// (fully coalesced: a warp reads 512 contiguous bytes per row), multiplies
// them against its register-resident x', reduces over lanes with shuffles and
// over the slot's warps through shared memory in a fixed order. CTAs are
// persistent; x is read from L2 once per slot. There is no workspace and no
// atomics: the output is deterministic.
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

template <int BITS, int NB>
__device__ __forceinline__ void accumulate_word(uint32_t w, const float* xw /* [NB][PER_WORD] */,
                                                float2 (&acc)[NB]) {
    if (BITS == 4) {
        const uint32_t t = w >> 24;
        const float2 f01 = make_float2(__uint_as_float(w & 0x0000000Fu), __uint_as_float(w & 0x000000F0u));
        const float2 f23 = make_float2(__uint_as_float(w & 0x00000F00u), __uint_as_float(w & 0x0000F000u));
        const float2 f45 = make_float2(__uint_as_float(w & 0x000F0000u), __uint_as_float(w & 0x00F00000u));
        const float2 f67 = make_float2(__uint_as_float(t & 0x0000000Fu), __uint_as_float(t & 0x000000F0u));
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const float* xb = xw + b * 8;
            acc[b] = __ffma2_rn(f01, make_float2(xb[0], xb[1]), acc[b]);
            acc[b] = __ffma2_rn(f23, make_float2(xb[2], xb[3]), acc[b]);
            acc[b] = __ffma2_rn(f45, make_float2(xb[4], xb[5]), acc[b]);
            acc[b] = __ffma2_rn(f67, make_float2(xb[6], xb[7]), acc[b]);
        }
    } else {
        const float2 f01 = make_float2(__uint_as_float(w & 0x000000FFu), __uint_as_float(w & 0x0000FF00u));
        const float2 f23 = make_float2(__uint_as_float(w & 0x00FF0000u), __uint_as_float(w >> 24));
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const float* xb = xw + b * 4;
            acc[b] = __ffma2_rn(f01, make_float2(xb[0], xb[1]), acc[b]);
            acc[b] = __ffma2_rn(f23, make_float2(xb[2], xb[3]), acc[b]);
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
    int M, K, NCH;
    int64_t q_stride, ldy;
    int scale_rows, groups, group_size;
    int wpr;        // warps per row slot
    int slots;      // row slots per CTA
    int x_vec4;     // x rows and channel are 16-byte aligned and K % 4 == 0
};

constexpr int kMaxSlots = 8;  // named barriers 1..8 (CTA <= 256 threads)

template <int BITS, int NB, int NCPL, int R>
__global__ void __launch_bounds__(256) gemv_kernel(const GemvParams p) {
    constexpr int CH = Fmt<BITS>::CH;
    constexpr int PW = Fmt<BITS>::PER_WORD;
    extern __shared__ float smem[];
    // smem: red[2][slots][wpr][R*NB] partials, then emax[slots][wpr][NB]
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int slot = warp / p.wpr;
    const int wslot = warp - slot * p.wpr;
    const int slot_threads = p.wpr * 32;
    float* red = smem;
    float* emax = smem + 2 * p.slots * p.wpr * R * NB;

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
    asm volatile("bar.sync %0, %1;" ::"r"(slot + 1), "r"(slot_threads));
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

    // ---- stream rows -----------------------------------------------------------
    const int64_t total_slots = (int64_t)gridDim.x * p.slots;
    const int64_t gslot = (int64_t)blockIdx.x * p.slots + slot;
    const int64_t n_iters_total = ((int64_t)p.M + R - 1) / R;
    const bool multi = p.groups > 1;

    uint4 cur[R][NCPL];
    float csc[R][NCPL], czr[R][NCPL];
    auto load = [&](int64_t it, uint4 (&cq)[R][NCPL], float (&sc)[R][NCPL], float (&zr)[R][NCPL]) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int64_t row = it * R + r;
#pragma unroll
            for (int j = 0; j < NCPL; ++j) {
                const int c = cidx[j];
                if (row < p.M && c < p.NCH) {
                    cq[r][j] = ld_stream_v4(p.q + row * p.q_stride + (int64_t)c * 16);
                    const int g = multi ? (c * CH) / p.group_size : 0;
                    const int64_t srow = p.scale_rows == 1 ? 0 : row;
                    sc[r][j] = __ldg(p.scales + srow * p.groups + g);
                    zr[r][j] = __ldg(p.zeros + srow * p.groups + g);
                } else {
                    cq[r][j] = make_uint4(0u, 0u, 0u, 0u);
                    sc[r][j] = 0.0f;
                    zr[r][j] = 0.0f;
                }
            }
        }
    };

    int64_t it = gslot;
    if (it < n_iters_total) load(it, cur, csc, czr);
    int parity = 0;
    for (; it < n_iters_total; it += total_slots) {
        uint4 nxt[R][NCPL];
        float nsc[R][NCPL], nzr[R][NCPL];
        const int64_t nit = it + total_slots;
        if (nit < n_iters_total) load(nit, nxt, nsc, nzr);

        float yacc[R][NB];
#pragma unroll
        for (int r = 0; r < R; ++r) {
#pragma unroll
            for (int b = 0; b < NB; ++b) yacc[r][b] = 0.0f;
#pragma unroll
            for (int j = 0; j < NCPL; ++j) {
                float2 acc[NB];
#pragma unroll
                for (int b = 0; b < NB; ++b) acc[b] = make_float2(0.0f, 0.0f);
                const uint32_t words[4] = {cur[r][j].x, cur[r][j].y, cur[r][j].z, cur[r][j].w};
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) {
                    float xw[NB * PW];
#pragma unroll
                    for (int b = 0; b < NB; ++b)
#pragma unroll
                        for (int i = 0; i < PW; ++i) xw[b * PW + i] = xr[j][b][wi * PW + i];
                    accumulate_word<BITS, NB>(words[wi], xw, acc);
                }
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    const float a = acc[b].x + acc[b].y;
                    const float t = fmaf(-czr[r][j], sx[j][b], a);
                    yacc[r][b] = fmaf(csc[r][j], t, yacc[r][b]);
                }
            }
        }
        // reduce over lanes, then over the slot's warps in a fixed order
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < NB; ++b) yacc[r][b] = warp_sum(yacc[r][b]);
        if (p.wpr == 1) {
            if (lane == 0) {
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int64_t row = it * R + r;
                    if (row < p.M) {
#pragma unroll
                        for (int b = 0; b < NB; ++b) {
                            const int h = 25 + eb[b], h1 = h / 2;
                            p.y[(int64_t)b * p.ldy + row] = (yacc[r][b] * pow2i(h1)) * pow2i(h - h1);
                        }
                    }
                }
            }
        } else {
            float* rb = red + ((parity * p.slots + slot) * p.wpr) * R * NB;
            if (lane == 0) {
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int b = 0; b < NB; ++b) rb[wslot * R * NB + r * NB + b] = yacc[r][b];
            }
            asm volatile("bar.sync %0, %1;" ::"r"(slot + 1), "r"(slot_threads));
            if (wslot == 0 && lane < R * NB) {
                const int r = lane / NB, b = lane - (lane / NB) * NB;
                const int64_t row = it * R + r;
                float v = 0.0f;
                for (int w = 0; w < p.wpr; ++w) v += rb[w * R * NB + lane];
                if (row < p.M) {
                    int e = 0;
#pragma unroll
                    for (int bb = 0; bb < NB; ++bb)
                        if (bb == b) e = eb[bb];
                    const int h = 25 + e, h1 = h / 2;
                    p.y[(int64_t)b * p.ldy + row] = (v * pow2i(h1)) * pow2i(h - h1);
                }
            }
            parity ^= 1;
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int j = 0; j < NCPL; ++j) {
                cur[r][j] = nxt[r][j];
                csc[r][j] = nsc[r][j];
                czr[r][j] = nzr[r][j];
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
        if (waste < best_waste || (waste == best_waste && ncpl > c.ncpl)) {
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

template <int BITS, int NB, int NCPL, int R>
cudaError_t launch_t(const GemvParams& p, cudaStream_t s) {
    auto kern = gemv_kernel<BITS, NB, NCPL, R>;
    const int threads = p.wpr * p.slots * 32;
    const size_t smem = sizeof(float) * (size_t)(2 * p.slots * p.wpr * R * NB + p.slots * p.wpr * NB);
    int occ = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem);
    if (e != cudaSuccess) return e;
    if (occ < 1) occ = 1;
    const int64_t iters = ((int64_t)p.M + R - 1) / R;
    int64_t grid = (int64_t)sm_count() * occ;
    const int64_t need = (iters + p.slots - 1) / p.slots;
    if (grid > need) grid = need;
    if (grid < 1) grid = 1;
    kern<<<(unsigned)grid, threads, smem, s>>>(p);
    return cudaGetLastError();
}

template <int BITS>
cudaError_t dispatch(const GemvParams& p, int NB, int ncpl, cudaStream_t s) {
    switch (NB) {
        case 1: return ncpl == 2 ? launch_t<BITS, 1, 2, 2>(p, s) : launch_t<BITS, 1, 1, 4>(p, s);
        case 2: return ncpl == 2 ? launch_t<BITS, 2, 2, 2>(p, s) : launch_t<BITS, 2, 1, 2>(p, s);
        case 3:
            if constexpr (BITS == 8) {
                if (ncpl == 2) return launch_t<BITS, 3, 2, 1>(p, s);
            }
            return launch_t<BITS, 3, 1, 2>(p, s);
        default:
            if constexpr (BITS == 8) {
                if (ncpl == 2) return launch_t<BITS, 4, 2, 1>(p, s);
            }
            return launch_t<BITS, 4, 1, 2>(p, s);
    }
}

}  // namespace

size_t gemv_workspace_bytes(int64_t, int64_t, int) { return 0; }

bool gemv_supported(const GemmProblem& p) {
    if (p.B < 1 || p.B > kGemvMaxBatch || p.K < 1 || p.M < 1) return false;
    if (p.q_stride % 16 != 0 || (reinterpret_cast<uintptr_t>(p.q) & 15) != 0) return false;
    const int CH = p.bits == 4 ? 32 : 16;
    if (p.groups > 1 && (p.group_size % CH) != 0) return false;
    const int64_t nch = p.q_stride / 16;
    if (nch > (int64_t)8 * 32 * 2) return false;
    if (p.M > ((int64_t)1 << 31) - 64) return false;
    Choice c{0, 0, 0};
    const int NB = (int)p.B;
    return p.bits == 4 ? choose<4>(NB, (int)nch, c) : choose<8>(NB, (int)nch, c);
}

cudaError_t launch_gemv(const GemmProblem& g, void* /*workspace*/, cudaStream_t s) {
    GemvParams p;
    p.x = g.x;
    p.q = g.q;
    p.scales = g.scales;
    p.zeros = g.zeros;
    p.channel = g.channel;
    p.y = g.y;
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
    Choice c{0, 0, 0};
    const int NB = (int)g.B;
    const bool ok = g.bits == 4 ? choose<4>(NB, p.NCH, c) : choose<8>(NB, p.NCH, c);
    if (!ok) return cudaErrorInvalidValue;
    p.wpr = c.wpr;
    p.slots = c.slots;
    return g.bits == 4 ? dispatch<4>(p, NB, c.ncpl, s) : dispatch<8>(p, NB, c.ncpl, s);
}

}  // namespace wq

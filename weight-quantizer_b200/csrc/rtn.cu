// K3 — RTN quantize + int4 pack on the GPU, bit-exact with ptqkit.
//
// Restates src/ptqkit/quant.py:146-184 (qparams, integer_codes), :225-289
// (quantize_weight: finite check, pre_scale fold, granularity dispatch) and
// src/ptqkit/pack.py:17-33 (pack_int4) as device code. Bit-exactness rests on:
//   - every fp32 operation is a correctly rounded __f*_rn intrinsic, so nothing
//     is contracted into an FMA, in the reference's operation order;
//   - round-half-to-even is rintf (cvt.rni), as torch.round;
//   - block min/max are exact reductions; when a block's smallest value is a
//     zero, its sign is the sign of the first zero in row-major block order,
//     found with a (position, sign) min-reduction. torch.minimum(xmin, 0) then
//     keeps a -0.0 and turns a positive minimum into +0.0, which makes the
//     stored zero point -0.0 (quant.py:163-170).
// One warp quantizes one row (all of its groups); codes are gathered in shared
// memory and packed with coalesced stores. Per-tensor granularity first reduces
// the whole matrix (two deterministic passes through a small workspace).
#include <cfloat>
#include <climits>

#include "common.cuh"
#include "kernels.h"

namespace wq {
namespace {

constexpr int kRtnWarps = 8;
constexpr int kEpl = 8;                 // elements a lane caches per group
constexpr int kTensorBlocks = 1184;     // partial blocks of the per-tensor pass
constexpr unsigned long long kNoZero = ~0ull;

struct Stats {
    float amax;                 // symmetric
    float vmin, vmax;           // asymmetric
    unsigned long long zkey;    // 2 * (position of first zero) + signbit, or kNoZero
};

__device__ __forceinline__ void stats_init(Stats& s) {
    s.amax = 0.0f;
    s.vmin = FLT_MAX;
    s.vmax = -FLT_MAX;
    s.zkey = kNoZero;
}

__device__ __forceinline__ void stats_add(Stats& s, float v, unsigned long long pos) {
    s.amax = fmaxf(s.amax, fabsf(v));
    s.vmin = fminf(s.vmin, v);
    s.vmax = fmaxf(s.vmax, v);
    if (v == 0.0f) {
        const unsigned long long key = 2ull * pos + (__float_as_uint(v) >> 31);
        if (key < s.zkey) s.zkey = key;
    }
}

__device__ __forceinline__ void stats_merge(Stats& a, const Stats& b) {
    a.amax = fmaxf(a.amax, b.amax);
    a.vmin = fminf(a.vmin, b.vmin);
    a.vmax = fmaxf(a.vmax, b.vmax);
    if (b.zkey < a.zkey) a.zkey = b.zkey;
}

__device__ __forceinline__ Stats stats_warp(Stats s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Stats t;
        t.amax = __shfl_xor_sync(0xffffffffu, s.amax, o);
        t.vmin = __shfl_xor_sync(0xffffffffu, s.vmin, o);
        t.vmax = __shfl_xor_sync(0xffffffffu, s.vmax, o);
        t.zkey = __shfl_xor_sync(0xffffffffu, s.zkey, o);
        stats_merge(s, t);
    }
    return s;
}

// qparams (quant.py:146-172) from the exact block statistics.
__device__ __forceinline__ void qparams(const Stats& s, int symmetric, int qmax, float& scale,
                                        float& zero) {
    if (symmetric) {
        // torch.where(amax > 0, (2 * amax) / qmax, 1); zero = (qmax + 1) / 2
        scale = s.amax > 0.0f ? __fdiv_rn(__fmul_rn(2.0f, s.amax), (float)qmax) : 1.0f;
        zero = (float)(qmax + 1) / 2.0f;
        return;
    }
    // xmin = minimum(amin, 0): a positive minimum becomes +0.0; a zero minimum
    // keeps the sign of the first zero of the block.
    float xmin = s.vmin;
    if (xmin > 0.0f) {
        xmin = 0.0f;
    } else if (xmin == 0.0f) {
        xmin = (s.zkey != kNoZero && (s.zkey & 1ull)) ? -0.0f : 0.0f;
    }
    float xmax = s.vmax < 0.0f ? 0.0f : s.vmax;
    if (xmin == 0.0f && xmax == 0.0f) {
        xmin = -1.0f;
        xmax = 1.0f;
    }
    float sc = __fdiv_rn(__fsub_rn(xmax, xmin), (float)qmax);
    if (!(sc > 0.0f)) sc = 1.0f;
    float z = rintf(__fdiv_rn(-xmin, sc));
    if (z < 0.0f) z = 0.0f;
    if (z > (float)qmax) z = (float)qmax;
    scale = sc;
    zero = z;
}

// integer_codes (quant.py:175-184)
__device__ __forceinline__ uint8_t code_of(float v, float scale, float zero, int qmax) {
    float q = __fadd_rn(rintf(__fdiv_rn(v, scale)), zero);
    if (q < 0.0f) q = 0.0f;
    if (q > (float)qmax) q = (float)qmax;
    return (uint8_t)(int)rintf(q);
}

__device__ __forceinline__ float load_w(const RtnProblem& p, int64_t row, int64_t k, bool& bad) {
    float v = p.w[row * p.K + k];
    if (!isfinite(v)) bad = true;
    if (p.pre_scale != nullptr) v = __fmul_rn(v, p.pre_scale[k]);
    return v;
}

// pre_scale validation and channel_out = 1 / s (quant.py:242-250).
__global__ void prescale_kernel(const float* s, int64_t K, float* channel_out, int32_t* flags) {
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < K;
         k += (int64_t)gridDim.x * blockDim.x) {
        const float v = s[k];
        if (!isfinite(v) || !(v > 0.0f)) atomicOr(flags, 2);
        channel_out[k] = __fdiv_rn(1.0f, v);
    }
}

__global__ void clear_flags_kernel(int32_t* flags) { *flags = 0; }

// Per-tensor pass 1: partial statistics of the flattened matrix.
__global__ void __launch_bounds__(256) tensor_stats_kernel(const RtnProblem p, Stats* partial) {
    __shared__ Stats sh[8];
    Stats s;
    stats_init(s);
    bool bad = false;
    const int64_t n = p.M * p.K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / p.K, k = i - row * p.K;
        stats_add(s, load_w(p, row, k, bad), (unsigned long long)i);
    }
    if (bad) atomicOr(p.flags, 1);
    s = stats_warp(s);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        Stats t = sh[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) stats_merge(t, sh[w]);
        partial[blockIdx.x] = t;
    }
}

// Row kernel: one warp per row, all groups of the row, then pack.
// mode: group_mode > 0 (group), -1 (channel: one group of K), 0 (tensor:
// statistics come from `partial`).
__global__ void __launch_bounds__(kRtnWarps * 32) rtn_rows_kernel(const RtnProblem p, const Stats* partial,
                                                                  int n_partial) {
    extern __shared__ uint8_t codes_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    uint8_t* codes = codes_smem + (int64_t)warp * p.K;
    const int qmax = (1 << p.bits) - 1;
    const int64_t G = p.group_mode > 0 ? p.group_mode : p.K;
    const int64_t groups = p.group_mode > 0 ? (p.K + G - 1) / G : 1;
    const int64_t row_bytes = p.bits == 4 ? (p.K + 1) / 2 : p.K;

    float t_scale = 1.0f, t_zero = 0.0f;
    if (p.group_mode == 0) {
        Stats s;
        stats_init(s);
        for (int i = lane; i < n_partial; i += 32) stats_merge(s, partial[i]);
        s = stats_warp(s);
        qparams(s, p.symmetric, qmax, t_scale, t_zero);
        if (blockIdx.x == 0 && warp == 0 && lane == 0) {
            p.scales_out[0] = t_scale;
            p.zeros_out[0] = t_zero;
        }
    }

    for (int64_t row = (int64_t)blockIdx.x * warps + warp; row < p.M; row += (int64_t)gridDim.x * warps) {
        bool bad = false;
        for (int64_t g = 0; g < groups; ++g) {
            const int64_t k0 = g * G;
            const int64_t k1 = (k0 + G < p.K) ? k0 + G : p.K;
            float scale = t_scale, zero = t_zero;
            if (p.group_mode != 0) {
                Stats s;
                stats_init(s);
                float cache[kEpl];
#pragma unroll
                for (int i = 0; i < kEpl; ++i) {
                    const int64_t k = k0 + lane + 32 * i;
                    cache[i] = 0.0f;
                    if (k < k1) {
                        cache[i] = load_w(p, row, k, bad);
                        stats_add(s, cache[i], (unsigned long long)(k - k0));
                    }
                }
                for (int64_t k = k0 + lane + 32 * kEpl; k < k1; k += 32)
                    stats_add(s, load_w(p, row, k, bad), (unsigned long long)(k - k0));
                s = stats_warp(s);
                qparams(s, p.symmetric, qmax, scale, zero);
                if (lane == 0) {
                    p.scales_out[row * groups + g] = scale;
                    p.zeros_out[row * groups + g] = zero;
                }
#pragma unroll
                for (int i = 0; i < kEpl; ++i) {
                    const int64_t k = k0 + lane + 32 * i;
                    if (k < k1) codes[k] = code_of(cache[i], scale, zero, qmax);
                }
                for (int64_t k = k0 + lane + 32 * kEpl; k < k1; k += 32)
                    codes[k] = code_of(load_w(p, row, k, bad), scale, zero, qmax);
            } else {
                for (int64_t k = k0 + lane; k < k1; k += 32) {
                    bool unused = false;
                    codes[k] = code_of(load_w(p, row, k, unused), scale, zero, qmax);
                }
            }
        }
        if (bad) atomicOr(p.flags, 1);
        __syncwarp();
        uint8_t* out = p.q_out + row * row_bytes;
        if (p.bits == 4) {
            for (int64_t j = lane; j < row_bytes; j += 32) {
                const uint8_t lo = codes[2 * j] & 0x0F;
                const uint8_t hi = (2 * j + 1 < p.K) ? (codes[2 * j + 1] & 0x0F) : 0;
                out[j] = (uint8_t)(lo | (hi << 4));
            }
        } else {
            for (int64_t j = lane; j < row_bytes; j += 32) out[j] = codes[j];
        }
        __syncwarp();
    }
}

// Group kernel for the common layout: K % G == 0, G in {8, ..., 256} (a power
// of two), K % 8 == 0. The matrix is walked as a flat sequence of 8-element
// chunks in row-major order; LPG = G / 8 consecutive lanes hold one group, a
// warp step covers 256 elements (whole groups, possibly of two rows). Each
// lane loads its chunk with two 16-byte loads, the group's statistics are
// exact shuffle reductions over its LPG lanes, and each lane packs its 8 codes
// into one 32-bit (int4) or 64-bit (int8) store. Same operations per element
// as rtn_rows_kernel, so the outputs are identical.
template <int LPG>
__global__ void __launch_bounds__(256) rtn_groups_kernel(const RtnProblem p) {
    const int lane = threadIdx.x & 31;
    const int qmax = (1 << p.bits) - 1;
    const int64_t G = (int64_t)LPG * 8;
    const int64_t groups = p.K / G;
    const int64_t chunks_per_row = p.K / 8;
    const int64_t total = p.M * chunks_per_row;
    const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    bool bad = false;
    for (int64_t base = warp0 * 32; base < total; base += nwarps * 32) {
        const int64_t c = base + lane;
        const bool live = c < total;
        const int64_t row = live ? c / chunks_per_row : 0;
        const int64_t k = live ? (c - row * chunks_per_row) * 8 : 0;
        float v[8];
        Stats st;
        stats_init(st);
        if (live) {
            const float4 a = *reinterpret_cast<const float4*>(p.w + row * p.K + k);
            const float4 b = *reinterpret_cast<const float4*>(p.w + row * p.K + k + 4);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (!isfinite(v[i])) bad = true;
            if (p.pre_scale != nullptr) {
                const float4 sa = *reinterpret_cast<const float4*>(p.pre_scale + k);
                const float4 sb = *reinterpret_cast<const float4*>(p.pre_scale + k + 4);
                const float sc[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(v[i], sc[i]);
            }
            const unsigned long long pos0 = (unsigned long long)(k % G);
#pragma unroll
            for (int i = 0; i < 8; ++i) stats_add(st, v[i], pos0 + i);
        }
        // exact statistics of the group held by LPG consecutive lanes
#pragma unroll
        for (int o = LPG / 2; o > 0; o >>= 1) {
            Stats t;
            t.amax = __shfl_xor_sync(0xffffffffu, st.amax, o);
            t.vmin = __shfl_xor_sync(0xffffffffu, st.vmin, o);
            t.vmax = __shfl_xor_sync(0xffffffffu, st.vmax, o);
            t.zkey = __shfl_xor_sync(0xffffffffu, st.zkey, o);
            stats_merge(st, t);
        }
        if (!live) continue;
        float scale, zero;
        qparams(st, p.symmetric, qmax, scale, zero);
        if ((lane & (LPG - 1)) == 0) {
            p.scales_out[row * groups + k / G] = scale;
            p.zeros_out[row * groups + k / G] = zero;
        }
        uint32_t cd[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) cd[i] = code_of(v[i], scale, zero, qmax);
        if (p.bits == 4) {
            uint32_t word = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) word |= (cd[i] & 0xFu) << (4 * i);
            *reinterpret_cast<uint32_t*>(p.q_out + row * (p.K / 2) + k / 2) = word;
        } else {
            const uint2 w2 = make_uint2(cd[0] | (cd[1] << 8) | (cd[2] << 16) | (cd[3] << 24),
                                        cd[4] | (cd[5] << 8) | (cd[6] << 16) | (cd[7] << 24));
            *reinterpret_cast<uint2*>(p.q_out + row * p.K + k) = w2;
        }
    }
    if (bad) atomicOr(p.flags, 1);
}

__global__ void minmax_init_kernel(int32_t* mm) {
    mm[0] = INT_MAX;
    mm[1] = INT_MIN;
}

__global__ void pack_int4_kernel(const int32_t* codes, int64_t M, int64_t K, uint8_t* packed, int32_t* mm) {
    const int64_t cols = (K + 1) / 2;
    const int64_t n = M * cols;
    int lo_v = INT_MAX, hi_v = INT_MIN;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / cols, j = i - m * cols;
        const int32_t a = codes[m * K + 2 * j];
        lo_v = min(lo_v, a);
        hi_v = max(hi_v, a);
        int32_t b = 0;
        if (2 * j + 1 < K) {
            b = codes[m * K + 2 * j + 1];
            lo_v = min(lo_v, b);
            hi_v = max(hi_v, b);
        }
        packed[i] = (uint8_t)((a & 0x0F) | ((b & 0x0F) << 4));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        lo_v = min(lo_v, __shfl_xor_sync(0xffffffffu, lo_v, o));
        hi_v = max(hi_v, __shfl_xor_sync(0xffffffffu, hi_v, o));
    }
    if ((threadIdx.x & 31) == 0) {
        if (lo_v != INT_MAX) atomicMin(mm, lo_v);
        if (hi_v != INT_MIN) atomicMax(mm + 1, hi_v);
    }
}

__global__ void unpack_int4_kernel(const uint8_t* packed, int64_t M, int64_t cols, int64_t K, uint8_t* codes) {
    const int64_t n = M * K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / K, k = i - m * K;
        const uint8_t byte = packed[m * cols + (k >> 1)];
        codes[i] = (k & 1) == 0 ? (uint8_t)(byte & 0x0F) : (uint8_t)(byte >> 4);
    }
}

// dequantize_weight (quant.py:292-308): ((code - zero) * scale) [* channel]
__global__ void dequantize_kernel(const uint8_t* q, int64_t M, int64_t K, int64_t q_stride,
                                  const float* scales, int scale_rows, int groups, const float* zeros,
                                  const float* channel, int group_size, int bits, float* w_out) {
    const int64_t n = M * K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / K, k = i - m * K;
        int code;
        if (bits == 8) {
            code = q[m * q_stride + k];
        } else {
            const uint8_t byte = q[m * q_stride + (k >> 1)];
            code = (k & 1) == 0 ? (byte & 0x0F) : (byte >> 4);
        }
        const int64_t srow = scale_rows == 1 ? 0 : m;
        const int64_t g = groups == 1 ? 0 : k / group_size;
        float w = __fmul_rn(__fsub_rn((float)code, zeros[srow * groups + g]), scales[srow * groups + g]);
        if (channel != nullptr) w = __fmul_rn(w, channel[k]);
        w_out[i] = w;
    }
}

__global__ void gather_permute_kernel(const float* src, int64_t P, int64_t B, int64_t Mp, float* dst) {
    const int64_t n = P * B * Mp;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        // i indexes dst [B, P*Mp] row-major
        const int64_t b = i / (P * Mp), r = i - b * P * Mp;
        const int64_t pp = r / Mp, j = r - pp * Mp;
        dst[i] = src[(pp * B + b) * Mp + j];
    }
}

unsigned grid_for(int64_t n, int threads) {
    int64_t blocks = (n + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (unsigned)blocks;
}

}  // namespace

size_t rtn_workspace_bytes(int64_t, int64_t, int group_mode) {
    return group_mode == 0 ? sizeof(Stats) * kTensorBlocks : 0;
}

cudaError_t launch_rtn(const RtnProblem& p, void* workspace, cudaStream_t s) {
    clear_flags_kernel<<<1, 1, 0, s>>>(p.flags);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (p.pre_scale != nullptr && p.K > 0) {
        prescale_kernel<<<grid_for(p.K, 256), 256, 0, s>>>(p.pre_scale, p.K, p.channel_out, p.flags);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    if (p.M == 0 || p.K == 0) return cudaSuccess;
    Stats* partial = nullptr;
    int n_partial = 0;
    if (p.group_mode == 0) {
        partial = static_cast<Stats*>(workspace);
        n_partial = kTensorBlocks;
        tensor_stats_kernel<<<kTensorBlocks, 256, 0, s>>>(p, partial);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    const int64_t G = p.group_mode;
    const bool aligned = (reinterpret_cast<uintptr_t>(p.w) & 15) == 0 && (reinterpret_cast<uintptr_t>(p.q_out) & 7) == 0 &&
                         (p.pre_scale == nullptr || (reinterpret_cast<uintptr_t>(p.pre_scale) & 15) == 0);
    if (G >= 8 && G <= 256 && (G & (G - 1)) == 0 && p.K % G == 0 && aligned) {
        const int64_t warps_needed = (p.M * (p.K / 8) + 31) / 32;
        int64_t blocks = (warps_needed + 7) / 8;
        const int64_t cap = (int64_t)sm_count() * 8;
        if (blocks > cap) blocks = cap;
        switch (G) {
            case 8: rtn_groups_kernel<1><<<(unsigned)blocks, 256, 0, s>>>(p); break;
            case 16: rtn_groups_kernel<2><<<(unsigned)blocks, 256, 0, s>>>(p); break;
            case 32: rtn_groups_kernel<4><<<(unsigned)blocks, 256, 0, s>>>(p); break;
            case 64: rtn_groups_kernel<8><<<(unsigned)blocks, 256, 0, s>>>(p); break;
            case 128: rtn_groups_kernel<16><<<(unsigned)blocks, 256, 0, s>>>(p); break;
            default: rtn_groups_kernel<32><<<(unsigned)blocks, 256, 0, s>>>(p); break;
        }
        return cudaGetLastError();
    }
    int warps = kRtnWarps;
    const int64_t smem_cap = 200 * 1024;
    while (warps > 1 && (int64_t)warps * p.K > smem_cap) warps >>= 1;
    const size_t smem = (size_t)warps * (size_t)p.K;
    if ((int64_t)smem > smem_cap) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        e = cudaFuncSetAttribute(rtn_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    int64_t blocks = (p.M + warps - 1) / warps;
    const int64_t cap = (int64_t)sm_count() * 16;
    if (blocks > cap) blocks = cap;
    rtn_rows_kernel<<<(unsigned)blocks, warps * 32, smem, s>>>(p, partial, n_partial);
    return cudaGetLastError();
}

cudaError_t launch_pack_int4(const int32_t* codes, int64_t M, int64_t K, uint8_t* packed, int32_t* mm,
                             cudaStream_t s) {
    minmax_init_kernel<<<1, 1, 0, s>>>(mm);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || M == 0 || K == 0) return e;
    pack_int4_kernel<<<grid_for(M * ((K + 1) / 2), 256), 256, 0, s>>>(codes, M, K, packed, mm);
    return cudaGetLastError();
}

cudaError_t launch_unpack_int4(const uint8_t* packed, int64_t M, int64_t cols, int64_t K, uint8_t* codes,
                               cudaStream_t s) {
    if (M == 0 || K == 0) return cudaSuccess;
    unpack_int4_kernel<<<grid_for(M * K, 256), 256, 0, s>>>(packed, M, cols, K, codes);
    return cudaGetLastError();
}

cudaError_t launch_dequantize(const uint8_t* q, int64_t M, int64_t K, int64_t q_stride, const float* scales,
                              int scale_rows, int groups, const float* zeros, const float* channel,
                              int group_size, int bits, float* w_out, cudaStream_t s) {
    if (M == 0 || K == 0) return cudaSuccess;
    dequantize_kernel<<<grid_for(M * K, 256), 256, 0, s>>>(q, M, K, q_stride, scales, scale_rows, groups,
                                                          zeros, channel, group_size, bits, w_out);
    return cudaGetLastError();
}

cudaError_t launch_gather_permute(const float* src, int64_t P, int64_t B, int64_t Mp, float* dst,
                                  cudaStream_t s) {
    const int64_t n = P * B * Mp;
    if (n == 0) return cudaSuccess;
    gather_permute_kernel<<<grid_for(n, 256), 256, 0, s>>>(src, P, B, Mp, dst);
    return cudaGetLastError();
}

}  // namespace wq

// K2 — tcgen05 / TMEM dequant-GEMM for batches >= 5 (prefill and wide decode).
//
// Replaces ptqkit's CPU kernel (src/ptqkit/csrc/dequant_gemm.cpp:57-218) for
// batched inputs. The contraction runs on the 5th-generation tensor cores with
// fp32 accuracy from fp16 operands:
//
//   * A = (q - zero) for one 128-row weight tile and a 64-wide K tile. Every
//     code minus an integral zero point is an integer of magnitude <= 255, exact
//     in fp16. Four dequant warps build A from TMA-loaded packed codes
//     (int4: LOP3 with the fp16 exponent 0x6400 gives 1024 + code, HSUB2 of
//     1024 + zero gives the exact difference) and store it in the 128-byte
//     swizzled K-major layout the MMA reads.
//   * B = x' * S_b split into fp16 hi + lo planes by a prep kernel (x' = x *
//     channel, S_b a per-batch-row power of two putting max|x'_b * S_b| in
//     [2^13, 2^14)), so hi + lo carries ~22 significant bits of x'.
//   * D[m, n] = sum_{k in group} A * (hi + lo) accumulates in fp32 in tensor
//     memory: one accumulator per quantization group, double-buffered, so the
//     per-row group scale can be applied outside the MMA. Four epilogue warps
//     read each finished group accumulator with tcgen05.ld, add
//     scale[m, g] * D into register accumulators, and at the end write
//     y[n, m] = acc * 2^-S_b.
//
// Roles (one CTA = one 128 x BN output tile): warp 0 issues the TMA loads of
// the packed codes and the two x' planes into an NS-deep stage ring; warp 1
// allocates tensor memory and one elected lane issues tcgen05.mma (M = 128,
// N = BN, K = 16) and tcgen05.commit; warps 2-5 dequantize; warps 6-9 run the
// epilogue. All hand-offs are mbarriers; every wait is bounded and, on expiry,
// records bit 0 in the library's fault word and stops waiting. Every TMA
// load targets this CTA's own shared memory only.
//
// Output tiles are rasterized in bands of 16 batch tiles so the x' planes of a
// band stay resident in L2 while the weights stream about twice.
#include <cuda.h>
#include <cuda_fp16.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace wq {
namespace {

constexpr int BM = 128;          // weight rows per tile (MMA M)
constexpr int BK = 64;           // K per stage: 64 fp16 = one 128-byte swizzle row
constexpr int kThreads = 320;    // 10 warps
constexpr int kBand = 16;        // batch tiles per rasterization band
constexpr int kWarpTma = 0, kWarpMma = 1, kWarpDq0 = 2, kWarpEpi0 = 6;

struct TcParams {
    const float* scales;
    const float* zeros;
    const float* inv_s;   // [B] 2^-S_b
    float* y;
    unsigned int* fault;
    int M, B, KT, groups, ktg, ngroups, scale_rows, bits;
    int tiles_m, tiles_n;
    int64_t ldy;
};

// ---- PTX helpers specific to this kernel ------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row core
// groups 1024 bytes apart (SBO), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    uint64_t d = (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;              // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024u >> 4) << 32;    // stride byte offset
    d |= (uint64_t)1u << 46;              // version
    d |= (uint64_t)2u << 61;              // SWIZZLE_128B
    return d;
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));  // (a & b) | c
    return d;
}
__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}

// 8 int4 codes (one 32-bit word, k ascending) -> 8 fp16 values (code - zero),
// packed as 16 bytes in k order; zz = half2(1024 + zero) twice.
__device__ __forceinline__ uint4 dq8_int4(uint32_t w, uint32_t zz) {
    const uint32_t t0 = hsub2_u32(lop3_and_or(w, 0x000F000Fu, 0x64006400u), zz);          // k0, k4
    const uint32_t t1 = hsub2_u32(lop3_and_or(w >> 4, 0x000F000Fu, 0x64006400u), zz);     // k1, k5
    const uint32_t t2 = hsub2_u32(lop3_and_or(w >> 8, 0x000F000Fu, 0x64006400u), zz);     // k2, k6
    const uint32_t t3 = hsub2_u32(lop3_and_or(w >> 12, 0x000F000Fu, 0x64006400u), zz);    // k3, k7
    return make_uint4(__byte_perm(t0, t1, 0x5410), __byte_perm(t2, t3, 0x5410), __byte_perm(t0, t1, 0x7632),
                      __byte_perm(t2, t3, 0x7632));
}
// 8 int8 codes (two words) -> 8 fp16 (code - zero)
__device__ __forceinline__ uint4 dq8_int8(uint32_t a, uint32_t b, uint32_t zz) {
    const uint32_t e = 0x64646464u;
    return make_uint4(hsub2_u32(__byte_perm(a, e, 0x4140), zz), hsub2_u32(__byte_perm(a, e, 0x4342), zz),
                      hsub2_u32(__byte_perm(b, e, 0x4140), zz), hsub2_u32(__byte_perm(b, e, 0x4342), zz));
}

template <int BN, int NS>
struct Smem {
    static constexpr int A_BYTES = BM * 128;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int C_MAX = BM * 64;           // packed codes of one stage (int8 worst case)
    static constexpr int STAGE = A_BYTES + 2 * B_BYTES + C_MAX;
    static constexpr int BAR_OFF = NS * STAGE;
    // barriers: full_b, full_c, full_a, empty per stage; acc_full[2], acc_empty[2]
    static constexpr int NBAR = 4 * NS + 4;
    static constexpr int TMEM_SLOT = BAR_OFF + 8 * NBAR;
    static constexpr int TOTAL = TMEM_SLOT + 16;
};

template <int BN, int NS>
__global__ void __launch_bounds__(kThreads, 1)
    dq_gemm_tc_kernel(const TcParams p, const __grid_constant__ CUtensorMap map_q,
                      const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo) {
    using L = Smem<BN, NS>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // the swizzled tiles need 1024-byte alignment of the dynamic window
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_addr(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    auto bar = [&](int i) -> uint32_t { return sbase + L::BAR_OFF + 8u * (uint32_t)i; };
    auto full_b = [&](int s) { return bar(s); };
    auto full_c = [&](int s) { return bar(NS + s); };
    auto full_a = [&](int s) { return bar(2 * NS + s); };
    auto empty = [&](int s) { return bar(3 * NS + s); };
    auto acc_full = [&](int b) { return bar(4 * NS + b); };
    auto acc_empty = [&](int b) { return bar(4 * NS + 2 + b); };
    auto stage_a = [&](int s) { return sbase + (uint32_t)(s * L::STAGE); };
    auto stage_bhi = [&](int s) { return sbase + (uint32_t)(s * L::STAGE + L::A_BYTES); };
    auto stage_blo = [&](int s) { return sbase + (uint32_t)(s * L::STAGE + L::A_BYTES + L::B_BYTES); };
    auto stage_c = [&](int s) { return sbase + (uint32_t)(s * L::STAGE + L::A_BYTES + 2 * L::B_BYTES); };
    const int cbytes = p.bits == 4 ? 32 : 64;  // packed codes per row per stage

    // tile coordinates (bands of kBand batch tiles, weight tiles inside a band)
    const int band = blockIdx.x / (p.tiles_m * kBand);
    const int inner = blockIdx.x - band * p.tiles_m * kBand;
    const int bw = min(kBand, p.tiles_n - band * kBand);
    const int m_tile = inner / bw;
    const int n_tile = band * kBand + (inner - m_tile * bw);
    const int m0 = m_tile * BM, n0 = n_tile * BN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full_b(s), 1);
            mbar_init(full_c(s), 1);
            mbar_init(full_a(s), 128);
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full(b), 1);
            mbar_init(acc_empty(b), 128);
        }
        fence_mbarrier_init();
    }
    constexpr uint32_t kTmemCols = (2 * BN) < 32 ? 32 : 2 * BN;
    if (warp == kWarpMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + L::TMEM_SLOT),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + L::TMEM_SLOT);
    bool faulted = false;
    auto wait = [&](uint32_t b, uint32_t parity) {
        if (faulted) return;
        if (!mbar_wait_bounded(b, parity)) {
            faulted = true;
            atomicOr(p.fault, 1u);
        }
    };

    if (warp == kWarpTma) {
        if (lane == 0) {
            for (int t = 0; t < p.KT; ++t) {
                const int s = t % NS, round = t / NS;
                if (round > 0) wait(empty(s), (uint32_t)((round - 1) & 1));
                mbar_arrive_expect_tx(full_b(s), 2u * L::B_BYTES);
                tma_load_2d(stage_bhi(s), &map_hi, t * BK, n0, full_b(s));
                tma_load_2d(stage_blo(s), &map_lo, t * BK, n0, full_b(s));
                mbar_arrive_expect_tx(full_c(s), (uint32_t)(BM * cbytes));
                tma_load_2d(stage_c(s), &map_q, t * cbytes, m0, full_c(s));
            }
        }
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            // kind::f16 instruction descriptor: D fp32, A/B fp16, both K-major, N = BN, M = 128
            const uint32_t idesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
            for (int t = 0; t < p.KT; ++t) {
                const int s = t % NS, round = t / NS;
                const int g = t / p.ktg;
                const bool first = (t % p.ktg) == 0;
                const bool last = ((t % p.ktg) == p.ktg - 1) || (t == p.KT - 1);
                const int buf = g & 1, use = g >> 1;
                if (first && use > 0) wait(acc_empty(buf), (uint32_t)((use - 1) & 1));
                wait(full_b(s), (uint32_t)(round & 1));
                wait(full_a(s), (uint32_t)(round & 1));
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * BN);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t ad = sw128_desc(stage_a(s) + 32u * kk);
                    mma_f16(d, ad, sw128_desc(stage_bhi(s) + 32u * kk), idesc, (first && kk == 0) ? 0u : 1u);
                    mma_f16(d, ad, sw128_desc(stage_blo(s) + 32u * kk), idesc, 1u);
                }
                mma_commit(empty(s));
                if (last) mma_commit(acc_full(buf));
            }
        }
    } else if (warp < kWarpEpi0) {
        // ---- dequant: thread r builds row r of A for every stage --------------
        const int r = threadIdx.x - kWarpDq0 * 32;
        const int64_t m = min(m0 + r, p.M - 1);
        const int64_t srow = p.scale_rows == 1 ? 0 : m;
        const uint32_t a_row = (uint32_t)r * 128u;
        const uint32_t swz = (uint32_t)(r & 7);
        bool inexact = false;
        for (int t = 0; t < p.KT; ++t) {
            const int s = t % NS, round = t / NS;
            const int g = p.groups == 1 ? 0 : t / p.ktg;
            const float z = __ldg(p.zeros + srow * p.groups + g);
            const float zb = 1024.0f + z;
            const __half zh = __float2half_rn(zb);
            if (__half2float(zh) != zb || !(z >= 0.0f && z <= 1023.0f)) inexact = true;
            const uint32_t zz = (uint32_t)__half_as_ushort(zh) * 0x10001u;
            wait(full_c(s), (uint32_t)(round & 1));
            if (round > 0) wait(empty(s), (uint32_t)((round - 1) & 1));
            const unsigned char* crow = smem + (s * L::STAGE + L::A_BYTES + 2 * L::B_BYTES) + r * cbytes;
            unsigned char* arow = smem + s * L::STAGE;
            if (p.bits == 4) {
                const uint4 c0 = *reinterpret_cast<const uint4*>(crow);
                const uint4 c1 = *reinterpret_cast<const uint4*>(crow + 16);
                const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    *reinterpret_cast<uint4*>(arow + a_row + (((uint32_t)c ^ swz) << 4)) = dq8_int4(w[c], zz);
            } else {
                uint32_t w[16];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint4 v = *reinterpret_cast<const uint4*>(crow + 16 * i);
                    w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
                }
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    *reinterpret_cast<uint4*>(arow + a_row + (((uint32_t)c ^ swz) << 4)) =
                        dq8_int8(w[2 * c], w[2 * c + 1], zz);
            }
            fence_proxy_async_smem();
            mbar_arrive(full_a(s));
        }
        if (inexact) atomicOr(p.fault, 2u);
    } else {
        // ---- epilogue: thread owns row r of the tile, all BN columns -----------
        const int q = warp & 3;                 // TMEM lane quarter this warp may access
        const int r = q * 32 + lane;
        const int64_t m = m0 + r;
        const int64_t srow = p.scale_rows == 1 ? 0 : min(m, (int64_t)p.M - 1);
        float acc[BN];
#pragma unroll
        for (int i = 0; i < BN; ++i) acc[i] = 0.0f;
        for (int g = 0; g < p.ngroups; ++g) {
            const int buf = g & 1, use = g >> 1;
            const float sc = __ldg(p.scales + srow * p.groups + (p.groups == 1 ? 0 : g));
            wait(acc_full(buf), (uint32_t)(use & 1));
            tc_fence_after();
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
#pragma unroll
            for (int c = 0; c < BN / 32; ++c) {
                float v[32];
                tmem_ld32(taddr + 32u * c, v);
#pragma unroll
                for (int i = 0; i < 32; ++i) acc[c * 32 + i] = fmaf(sc, v[i], acc[c * 32 + i]);
            }
            tc_fence_before();
            mbar_arrive(acc_empty(buf));
        }
        if (m < p.M) {
#pragma unroll
            for (int i = 0; i < BN; ++i) {
                const int n = n0 + i;
                if (n < p.B) p.y[(int64_t)n * p.ldy + m] = acc[i] * __ldg(p.inv_s + n);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kWarpMma) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// x' = x * channel, S_b from max|x'_b|, hi/lo fp16 planes [B][Kpad], inv_s[b] = 1/S_b.
__global__ void __launch_bounds__(256) prep_x_kernel(const float* x, const float* channel, int B, int K, int Kpad,
                                                     __half* hi, __half* lo, float* inv_s) {
    __shared__ float red[8];
    const int b = blockIdx.x;
    const float* xb = x + (int64_t)b * K;
    float mx = 0.0f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        float v = xb[k];
        if (channel != nullptr) v = v * channel[k];
        mx = fmaxf(mx, fabsf(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    float v = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v = fmaxf(v, red[w]);
    int e = 0;
    if (v > 0.0f && v <= 3.4028234e38f) frexpf(v, &e);   // v < 2^e
    e = e < -100 ? -100 : (e > 114 ? 114 : e);
    const float S = pow2i(14 - e);                       // max|x' S| < 2^14
    if (threadIdx.x == 0) inv_s[b] = pow2i(e - 14);
    __half* hb = hi + (int64_t)b * Kpad;
    __half* lb = lo + (int64_t)b * Kpad;
    for (int k = threadIdx.x; k < Kpad; k += blockDim.x) {
        float u = 0.0f;
        if (k < K) {
            u = xb[k];
            if (channel != nullptr) u = u * channel[k];
            u = u * S;
        }
        const __half h = __float2half_rn(u);
        hb[k] = h;
        lb[k] = __float2half_rn(u - __half2float(h));
    }
}

// ---- host side ----------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int64_t kpad_of(int64_t K) { return (K + BK - 1) / BK * BK; }

struct TcWorkspace {
    __half* hi;
    __half* lo;
    float* inv_s;
};

TcWorkspace carve(void* ws, int64_t B, int64_t K) {
    const int64_t kp = kpad_of(K);
    unsigned char* p = static_cast<unsigned char*>(ws);
    TcWorkspace w;
    w.hi = reinterpret_cast<__half*>(p);
    w.lo = reinterpret_cast<__half*>(p + B * kp * 2);
    w.inv_s = reinterpret_cast<float*>(p + 2 * B * kp * 2);
    return w;
}

template <int BN, int NS>
cudaError_t launch_bn(const GemmProblem& g, const TcWorkspace& w, cudaStream_t s) {
    using L = Smem<BN, NS>;
    const int64_t kp = kpad_of(g.K);
    CUtensorMap mq, mhi, mlo;
    const uint32_t cbytes = g.bits == 4 ? 32 : 64;
    if (!encode_2d(&mq, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.q, (uint64_t)g.q_stride, (uint64_t)g.M,
                   (uint64_t)g.q_stride, cbytes, BM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_2d(&mhi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w.hi, (uint64_t)kp, (uint64_t)g.B, (uint64_t)kp * 2, BK,
                   BN, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_2d(&mlo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w.lo, (uint64_t)kp, (uint64_t)g.B, (uint64_t)kp * 2, BK,
                   BN, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    TcParams p;
    p.scales = g.scales;
    p.zeros = g.zeros;
    p.inv_s = w.inv_s;
    p.y = g.y;
    p.fault = fault_word();
    if (p.fault == nullptr) return cudaErrorInvalidDevicePointer;
    p.M = (int)g.M;
    p.B = (int)g.B;
    p.KT = (int)(kp / BK);
    p.groups = g.groups;
    p.ktg = g.groups == 1 ? p.KT : g.group_size / BK;
    p.ngroups = (p.KT + p.ktg - 1) / p.ktg;
    p.scale_rows = g.scale_rows;
    p.bits = g.bits;
    p.tiles_m = (int)((g.M + BM - 1) / BM);
    p.tiles_n = (int)((g.B + BN - 1) / BN);
    p.ldy = g.ldy;
    const size_t smem = (size_t)L::TOTAL + 1024;
    auto kern = dq_gemm_tc_kernel<BN, NS>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int64_t grid = (int64_t)p.tiles_m * p.tiles_n;
    if (grid > 0x7fffffff) return cudaErrorInvalidValue;
    kern<<<(unsigned)grid, kThreads, smem, s>>>(p, mq, mhi, mlo);
    return cudaGetLastError();
}

}  // namespace

bool tc_supported(const GemmProblem& p) {
    if (p.B < 5 || p.M < 1 || p.K < 1) return false;
    if (p.q_stride % 16 != 0 || (reinterpret_cast<uintptr_t>(p.q) & 15) != 0) return false;
    if (p.groups > 1 && p.group_size % BK != 0) return false;
    if (p.M > 0x7fffff00 || p.B > 0x7fffff00) return false;
    if (kpad_of(p.K) / BK > 0x7fffffff) return false;
    return encode_fn() != nullptr;
}

size_t tc_workspace_bytes(int64_t B, int64_t K) {
    return (size_t)(2 * B * kpad_of(K) * 2 + B * 4 + 256);
}

cudaError_t launch_tc(const GemmProblem& g, void* workspace, cudaStream_t s) {
    const TcWorkspace w = carve(workspace, g.B, g.K);
    const int64_t kp = kpad_of(g.K);
    prep_x_kernel<<<(unsigned)g.B, 256, 0, s>>>(g.x, g.channel, (int)g.B, (int)g.K, (int)kp, w.hi, w.lo, w.inv_s);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (g.B <= 32) return launch_bn<32, 4>(g, w, s);
    if (g.B <= 64) return launch_bn<64, 4>(g, w, s);
    return launch_bn<128, 3>(g, w, s);
}

}  // namespace wq

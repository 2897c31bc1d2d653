// K2 — tcgen05 / TMEM dequant-GEMM for batches >= 5 (prefill and wide decode).
//
// Replaces ptqkit's CPU kernel (src/ptqkit/csrc/dequant_gemm.cpp:57-218) for
// batched inputs. The contraction runs on the 5th-generation tensor cores with
// fp32 accuracy from fp16 operands:
//
//   * A = (q - zi) for one 128-row weight tile, zi = clamp(rint(zero), 0,
//     1023): a code minus an integer in [0, 1023] is an integer of magnitude
//     <= 1023, exact in fp16. Dequant warps build A from TMA-loaded packed
//     codes (int4: LOP3 with the fp16 exponent 0x6400 gives 1024 + code,
//     HSUB2 of 1024 + zi gives the exact difference) and write it straight
//     into tensor memory with tcgen05.st (lane = weight row, two fp16 per
//     column), two 64-wide K tiles per A stage; the MMA reads A from tensor
//     memory. A zero point that is not such an integer (ptqkit's quantizers
//     never produce one, but the operator accepts any fp32 zero) leaves
//     dz = zero - zi, and the epilogue subtracts dz * sum_{k in g} x'_k * S_b
//     (per batch row and group, summed by the prep kernel), so
//     (q - zero) x' = (q - zi) x' - dz x' holds for every zero point. Warps
//     whose 32 rows all have integer zero points skip that term, which keeps
//     their results bit for bit what they were without it.
//   * B = x' * S_b split into fp16 hi + lo planes by a prep kernel (x' = x *
//     channel, S_b a per-batch-row power of two putting max|x'_b * S_b| in
//     [2^13, 2^14)), so hi + lo carries ~22 significant bits of x'. The prep
//     kernel writes the planes already tiled and 128-byte swizzled exactly as
//     the MMA reads them from shared memory, so one K tile of both planes for
//     one batch tile is a single contiguous bulk copy.
//   * D[m, n] = sum_{k in group} A * (hi + lo) accumulates in fp32 in tensor
//     memory: one accumulator per quantization group, double-buffered, so the
//     per-row group scale can be applied outside the MMA. The epilogue warps
//     read each finished group accumulator with tcgen05.ld, add
//     scale[m, g] * D into register accumulators, and at the end write
//     y[n, m] = acc * 2^-S_b (into every output buffer, or once through an
//     NVLink-switch address, for the row-sharded multi-GPU layer).
//
// Roles (one CTA = one 128 x BN output tile). Warpgroup 0: warp 0 bulk-copies
// the x' planes into an NS-deep shared-memory ring; warp 2 loads packed codes
// (several K tiles per 2D TMA box, 128 bytes per row, 128-byte swizzle) into a
// separate ring that the dequant warps release as soon as they have read it;
// warp 1 allocates tensor memory and one thread issues tcgen05.mma (M = 128,
// N = BN, K = 16, A from tensor memory) and tcgen05.commit, learning which
// tiles are ready from one shared word that warp 3 publishes after waiting on
// their barriers. Then one or two dequant warpgroups and one or two epilogue
// warpgroups (see Cfg). All hand-offs are mbarriers; every wait is bounded and,
// on expiry, records bit 0 in the library's fault word and stops waiting.
// Every TMA and bulk load targets this CTA's own shared memory only.
//
// Output tiles are rasterized in bands of batch tiles sized so that the x'
// planes of a band (at most 40 MB) stay resident in L2 while the weights
// stream past once per band.
#include <cuda.h>
#include <cuda_fp16.h>

#include <atomic>
#include <mutex>

#include "common.cuh"
#include "fp16_codes.cuh"
#include "kernels.h"

namespace wq {

// ---- 2D tensor maps (shared with the wide decode kernel) ---------------------
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

// A map is a pure function of its arguments, and a layer's weights are
// encoded with the same arguments on every call: the last few encodings are
// kept per host thread (no locking) and copied out on a repeat.
namespace {
struct MapKey {
    const void* base;
    uint64_t inner, outer, row_bytes;
    uint32_t box_inner, box_outer;
    int dt, swz;
    bool operator==(const MapKey& o) const {
        return base == o.base && inner == o.inner && outer == o.outer && row_bytes == o.row_bytes &&
               box_inner == o.box_inner && box_outer == o.box_outer && dt == o.dt && swz == o.swz;
    }
};
constexpr int kMapCache = 16;
struct MapCache {
    MapKey key[kMapCache];
    CUtensorMap map[kMapCache];
    int used = 0, next = 0;
};
thread_local MapCache t_maps;
}  // namespace

bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
    const MapKey k{base, inner, outer, row_bytes, box_inner, box_outer, (int)dt, (int)swz};
    MapCache& c = t_maps;
    for (int i = 0; i < c.used; ++i) {
        if (c.key[i] == k) {
            *map = c.map[i];
            return true;
        }
    }
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    if (fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
           CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    const int slot = c.used < kMapCache ? c.used++ : c.next;
    if (slot == c.next) c.next = (c.next + 1) % kMapCache;
    c.key[slot] = k;
    c.map[slot] = *map;
    return true;
}


namespace {

constexpr int BM = 128;          // weight rows per tile (MMA M)
constexpr int BK = 64;           // K per stage: 64 fp16 = one 128-byte swizzle row
// Output tiles are ordered in bands of batch tiles (weight tiles inside a
// band): the x' planes of one band (KT * 256 * BN bytes per batch tile) are
// kept under this size so that they stay in L2 while the weights stream past
// once per band.
constexpr int64_t kBandBytes = (int64_t)40 << 20;
// warpgroup 0: producers, MMA issuer, scheduler; then the dequant warpgroups;
// the last warpgroup runs the epilogue
constexpr int kWarpB = 0, kWarpMma = 1, kWarpCodes = 2, kWarpSched = 3, kWarpDq0 = 4;

// setmaxnreg toward N registers per thread: .dec only lowers and .inc only
// raises the count (the other direction is an illegal instruction), so the
// direction follows from the launch's count.
template <int N, int LAUNCH>
__device__ __forceinline__ void set_regs() {
    if constexpr (N < LAUNCH) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
    } else if constexpr (N > LAUNCH) {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
    }
}

// Launch shape per batch tile. Wide tiles (BN >= 128): one CTA per SM with
// all 512 columns of tensor memory and four warpgroups: N = 128 runs two
// dequant warpgroups (each writes one K tile of every A stage) and one
// epilogue warpgroup; N = 192 one dequant and two epilogue warpgroups (each
// reads 96 columns of every group accumulator: with one, the accumulator
// drain took longer than the next group's MMAs and held the MMA back).
// Narrow tiles: one dequant and one epilogue warpgroup, two CTAs per SM (half
// the tensor memory each) so that one CTA's hand-off latency overlaps the
// other's work. After entering their roles the
// warpgroups re-split the launch's registers with setmaxnreg; the split must
// not exceed the launch's registers (checked here and, for the per-thread
// count ptxas chose, again before the launch).
template <int BN>
struct Cfg {
    // The 192-wide tile drains its accumulators with two epilogue warpgroups
    // (96 columns each: a group's accumulator is read in half the time) and
    // dequantizes with one; the 128-wide tile the other way round.
    static constexpr int EPG = BN > 128 ? 2 : 1;            // epilogue warpgroups
    static constexpr int DQG = BN == 128 ? 2 : 1;           // dequant warpgroups
    static constexpr int EW = BN / EPG;                     // accumulator columns per epilogue thread
    static constexpr int THREADS = (1 + DQG + EPG) * 128;
    static constexpr int WARP_EPI0 = kWarpDq0 + 4 * DQG;
    static constexpr int DQ_WARPS = 4 * DQG;
    static constexpr int MINB = BN >= 128 ? 1 : 2;        // CTAs per SM
    static constexpr uint32_t TMEM_COLS = BN >= 128 ? 512 : 256;
    static constexpr int LAUNCH_REGS = (65536 / (THREADS * MINB)) / 8 * 8;
    static constexpr int REGS_CTL = 40;
    static constexpr int REGS_DQ = BN >= 128 ? 112 : 88;
    static constexpr int REGS_EPI = BN > 128 ? 176 : (BN >= 128 ? 232 : 112);
    // Batch tiles of 32 (batches 5-32) stack the hi and lo planes into one
    // MMA of N = 2 BN (the lo rows follow the hi rows in every K tile of the
    // planes), halving the MMA instructions, which bound this narrow tile;
    // the accumulator then holds sum A hi and sum A lo side by side.
    static constexpr bool STACK = BN <= 32;
    static constexpr int ACCW = STACK ? 2 * BN : BN;      // tensor-memory columns per accumulator
    static_assert(REGS_CTL + DQG * REGS_DQ + EPG * REGS_EPI <= (1 + DQG + EPG) * LAUNCH_REGS,
                  "register split exceeds the launch's registers");
};
constexpr int kCodeRowBytes = 128;  // packed code bytes per row per codes stage
constexpr int kNC = 2;              // codes stages

struct TcParams {
    const unsigned char* planes;  // tiled x' planes [tiles_n][KT][2][BN][128 B]
    const float* scales;
    const float* zeros;
    const float* inv_s;   // [B] 2^-S_b
    const float* xsum;    // [ngroups][bpad] sum over each group of x' * S_b
    int bpad;             // batch rows of the padded planes (row stride of xsum)
    float* y;
    float* y_extra[7];    // further outputs with y's layout (peer-mapped on other GPUs)
    int n_extra;
    float* y_all;         // NVLink-switch address reaching every rank's y, or nullptr
    const float* bias;    // [M] or nullptr
    float* part;          // split-K partial tiles [splits][tiles_m * tiles_n][BN][BM]
    int* counters;        // split-K arrivals per output tile (zeroed by the prep kernel)
    int splits, gran;     // K splits (grid.y) and the K tiles a split boundary is a multiple of
    unsigned int* fault;
    int M, B, KT, groups, ktg, ngroups, scale_rows;
    int tiles_m, tiles_n;
    int band;             // batch tiles per rasterization band
    int64_t ldy;
};

// ---- PTX helpers specific to this kernel ------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
// Store through an NVLink-switch (NVLS) address: the switch writes the value
// into the same position of every rank's buffer bound to that address.
__device__ __forceinline__ void st_all_ranks(float* addr, float v) {
    asm volatile("multimem.st.global.f32 [%0], %1;" ::"l"(addr), "f"(v) : "memory");
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

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

// Tensor memory: 512 columns (256 for the narrow tiles, two CTAs per SM).
// Columns [0, 2 ACCW) hold the two group accumulators; the rest is a ring of
// A stages, each two K tiles wide (2 x 32 columns of packed fp16 pairs, one
// row per lane).
constexpr int kTilesPerA = 2;
constexpr int kAStageCols = kTilesPerA * BK / 2;

template <int BN, int NS, int BITS>
struct Smem {
    static constexpr int CB = BITS == 4 ? 32 : 64;        // packed code bytes per row per K tile
    static constexpr int KC = kCodeRowBytes / CB;          // K tiles per codes stage
    static constexpr int NA = (int)(Cfg<BN>::TMEM_COLS - 2 * Cfg<BN>::ACCW) / kAStageCols;   // A stages in tensor memory
    static constexpr int B_BYTES = BN * 128;               // one plane of one K tile
    static constexpr int STAGE = 2 * B_BYTES;              // hi + lo planes
    static constexpr int C_STAGE = BM * kCodeRowBytes;
    static constexpr int C_OFF = NS * STAGE;
    static constexpr int BAR_OFF = C_OFF + kNC * C_STAGE;
    // barriers: full_b, empty_b per B stage; full_a, empty_a per A stage;
    // c_full, c_empty per codes stage; acc_full[2], acc_empty[2]
    static constexpr int NBAR = 2 * NS + 2 * NA + 2 * kNC + 4;
    static constexpr int TMEM_SLOT = BAR_OFF + 8 * NBAR;
    static constexpr int READY = TMEM_SLOT + 8;   // u32: tiles whose operands are ready
    static constexpr int FLAG = TMEM_SLOT + 12;   // u32: this CTA adds the split-K partials
    static constexpr int TOTAL = TMEM_SLOT + 16;
    static_assert(STAGE % 1024 == 0 && C_STAGE % 1024 == 0, "tiles must stay 1024-byte aligned for the 128-byte swizzle");
    static_assert(TOTAL + 1024 <= 227 * 1024, "stage rings exceed the shared memory of one CTA");
    static_assert(NA >= 2, "tensor memory holds fewer than two A stages");
    static_assert(KC % kTilesPerA == 0, "a codes stage must hold whole A stages");
};

template <int BN, int NS, int BITS, bool SPLIT>
__global__ void __launch_bounds__(Cfg<BN>::THREADS, Cfg<BN>::MINB)
    dq_gemm_tc_kernel(const TcParams p, const __grid_constant__ CUtensorMap map_q) {
    using L = Smem<BN, NS, BITS>;
    using C = Cfg<BN>;
    constexpr int NA = L::NA;
    constexpr int kWarpEpi0 = C::WARP_EPI0;
    constexpr uint32_t kTmemCols = C::TMEM_COLS;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // the swizzled tiles need 1024-byte alignment of the dynamic window
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_addr(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    auto bar = [&](int i) -> uint32_t { return sbase + L::BAR_OFF + 8u * (uint32_t)i; };
    auto full_b = [&](int s) { return bar(s); };
    auto empty_b = [&](int s) { return bar(NS + s); };
    auto full_a = [&](int s) { return bar(2 * NS + s); };
    auto empty_a = [&](int s) { return bar(2 * NS + NA + s); };
    auto c_full = [&](int c) { return bar(2 * NS + 2 * NA + c); };
    auto c_empty = [&](int c) { return bar(2 * NS + 2 * NA + kNC + c); };
    auto acc_full = [&](int b) { return bar(2 * NS + 2 * NA + 2 * kNC + b); };
    auto acc_empty = [&](int b) { return bar(2 * NS + 2 * NA + 2 * kNC + 2 + b); };
    auto stage_b = [&](int s) { return sbase + (uint32_t)(s * L::STAGE); };
    auto stage_c = [&](int c) { return sbase + (uint32_t)(L::C_OFF + c * L::C_STAGE); };

    // tile coordinates (bands of p.band batch tiles, weight tiles inside a band)
    const int band = blockIdx.x / (p.tiles_m * p.band);
    const int inner = blockIdx.x - band * p.tiles_m * p.band;
    const int bw = min(p.band, p.tiles_n - band * p.band);
    const int m_tile = inner / bw;
    const int n_tile = band * p.band + (inner - m_tile * bw);
    const int m0 = m_tile * BM, n0 = n_tile * BN;
    // split-K: this CTA's K tiles [t0, t0 + KTL) and groups [g0, g0 + NGL);
    // split boundaries fall on group and code-box boundaries (p.gran tiles)
    // (the unsplit instantiation reads the kernel parameters as they are)
    int s_t0 = 0, s_ktl = 0, s_g0 = 0, s_ngl = 0;
    if constexpr (SPLIT) {
        const int nu = (p.KT + p.gran - 1) / p.gran;
        const int su0 = (int)blockIdx.y * nu / p.splits, su1 = ((int)blockIdx.y + 1) * nu / p.splits;
        s_t0 = su0 * p.gran;
        s_ktl = min(su1 * p.gran, p.KT) - s_t0;
        s_g0 = s_t0 / p.ktg;
        s_ngl = (s_ktl + p.ktg - 1) / p.ktg;
    }
    auto T0 = [&]() -> int { if constexpr (SPLIT) return s_t0; else return 0; };
    auto KTL = [&]() -> int { if constexpr (SPLIT) return s_ktl; else return p.KT; };
    auto G0 = [&]() -> int { if constexpr (SPLIT) return s_g0; else return 0; };
    auto NGL = [&]() -> int { if constexpr (SPLIT) return s_ngl; else return p.ngroups; };
    const int n_astages = (KTL() + kTilesPerA - 1) / kTilesPerA;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full_b(s), 1);
            mbar_init(empty_b(s), 1);
        }
        for (int s = 0; s < NA; ++s) {
            mbar_init(full_a(s), C::DQ_WARPS);   // one arrival per dequant warp
            mbar_init(empty_a(s), 1);
        }
        for (int c = 0; c < kNC; ++c) {
            mbar_init(c_full(c), 1);
            mbar_init(c_empty(c), C::DQ_WARPS);  // one arrival per dequant warp
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full(b), 1);
            mbar_init(acc_empty(b), 4 * C::EPG);   // one arrival per epilogue warp
        }
        *reinterpret_cast<volatile uint32_t*>(smem + L::READY) = 0u;
        fence_mbarrier_init();
    }
    if (warp == kWarpMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + L::TMEM_SLOT),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Launched with programmatic stream serialization: the setup above
    // overlaps the prep kernel's tail; nothing below reads global memory
    // before that kernel (and every earlier one on the stream) has completed.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + L::TMEM_SLOT);
    const uint32_t tmem_a0 = tmem + (uint32_t)(2 * C::ACCW);
    bool faulted = false;
    auto wait = [&](uint32_t b, uint32_t parity) {
        if (faulted) return;
        if (!mbar_wait_bounded(b, parity)) {
            faulted = true;
            atomicOr(p.fault, 1u);
        }
    };
    // warp-wide wait: lane 0 polls the barrier (acquire), __syncwarp then
    // orders the other lanes after it; the fault flag is shared by the warp
    auto wait_warp = [&](uint32_t b, uint32_t parity) {
        if (lane == 0) wait(b, parity);
        faulted = __shfl_sync(0xffffffffu, faulted ? 1 : 0, 0) != 0;
        __syncwarp();
    };
    // Before the CTA exits, an issuing thread waits (bounded, even after a
    // fault) for the last phase of every ring slot it filled, so no copy or MMA
    // that it started is still writing shared or tensor memory. In a
    // fault-free run these phases have completed already.
    auto drain = [&](int nslots, int nitems, auto barrier_of) {
        for (int s = 0; s < nslots && s < nitems; ++s) {
            const int last_round = (nitems - 1 - s) / nslots;
            if (!mbar_wait_bounded(barrier_of(s), (uint32_t)(last_round & 1))) atomicOr(p.fault, 1u);
        }
    };

    // Each warpgroup re-splits the registers on entering its role: the
    // control warps need few, the epilogue holds BN fp32 accumulators per
    // thread. setmaxnreg is warpgroup-wide, so warpgroup 0 issues it before
    // its warps branch into their roles.
    if (warp < kWarpDq0) {
      set_regs<C::REGS_CTL, C::LAUNCH_REGS>();
      if (warp == kWarpB) {
        // x' planes: one bulk copy of both planes of a K tile per stage. The
        // planes of a band are read by every weight tile of the band, the codes
        // by the band's few concurrent CTAs: the planes are marked to stay in
        // L2 past the code stream.
        if (lane == 0) {
            const uint64_t keep = l2_policy_evict_last();
            const uint32_t tile_bytes = (uint32_t)L::STAGE;
            const unsigned char* src = p.planes + ((size_t)n_tile * p.KT + T0()) * tile_bytes;
            int s = 0;
            uint32_t ph = 0;
            for (int t = 0; t < KTL(); ++t) {
                if (t >= NS) wait(empty_b(s), ph ^ 1u);
                mbar_arrive_expect_tx(full_b(s), tile_bytes);
                bulk_copy_g2s_hint(stage_b(s), src, tile_bytes, full_b(s), keep);
                src += tile_bytes;
                if (++s == NS) {
                    s = 0;
                    ph ^= 1u;
                }
            }
            drain(NS, KTL(), full_b);
        }
      } else if (warp == kWarpCodes) {
        // packed codes: KC K tiles per 2D box (128 rows x 128 bytes, 128-byte
        // swizzle so that the dequant threads read them without bank conflicts)
        if (lane == 0) {
            const int nct = (KTL() + L::KC - 1) / L::KC;
            int c = 0;
            uint32_t ph = 0;
            for (int ct = 0; ct < nct; ++ct) {
                if (ct >= kNC) wait(c_empty(c), ph ^ 1u);
                mbar_arrive_expect_tx(c_full(c), (uint32_t)L::C_STAGE);
                tma_load_2d(stage_c(c), &map_q, (T0() / L::KC + ct) * kCodeRowBytes, m0, c_full(c));
                if (++c == kNC) {
                    c = 0;
                    ph ^= 1u;
                }
            }
            drain(kNC, nct, c_full);
        }
      } else if (warp == kWarpSched) {
        // Scheduler: walks the tiles in order, waits for each tile's x' stage,
        // A stage (first tile of a stage) and accumulator (first tile of a
        // group), and publishes how many tiles are ready. The MMA thread reads
        // that one word instead of the barriers: any shared-memory or barrier
        // operation it issues waits behind its own queued MMAs, so it should
        // touch as few as possible.
        if (lane == 0) {
            int sb = 0, sa = 0, h = 0, gin = 0, g = 0;
            uint32_t phb = 0, pha = 0;
            for (int t = 0; t < KTL(); ++t) {
                const int use = g >> 1;
                if (gin == 0 && use > 0) wait(acc_empty(g & 1), (uint32_t)((use - 1) & 1));
                wait(full_b(sb), phb);
                if (h == 0) wait(full_a(sa), pha);
                asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(sbase + L::READY), "r"((uint32_t)(t + 1))
                             : "memory");
                if ((gin == p.ktg - 1) || (t == KTL() - 1)) {
                    gin = 0;
                    ++g;
                } else {
                    ++gin;
                }
                if (++sb == NS) {
                    sb = 0;
                    phb ^= 1u;
                }
                if (++h == kTilesPerA) {
                    h = 0;
                    if (++sa == NA) {
                        sa = 0;
                        pha ^= 1u;
                    }
                }
            }
        }
      } else {
        // One thread issues every MMA: it reads the scheduler's ready count,
        // then issues every ready tile (up to kIssueBatch) back to back.
        // A comes from tensor memory; B descriptors are built once and a
        // stage, a plane or a 16-wide K step only moves the start-address
        // field (address / 16 in bits 0-13).
        if (lane == 0) {
            constexpr int kIssueBatch = 8;
            // kind::f16 instruction descriptor: D fp32, A/B fp16, both K-major, N = BN, M = 128
            constexpr int MMA_N = C::STACK ? 2 * BN : BN;
            const uint32_t idesc = (1u << 4) | ((uint32_t)(MMA_N >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
            const uint64_t b_desc0 = sw128_desc(stage_b(0));
            constexpr uint64_t kPlaneStep = (uint64_t)(L::B_BYTES >> 4);
            int t = 0, sb = 0, sa = 0, h = 0, gin = 0, g = 0;
            while (t < KTL()) {
                uint32_t ready = 0;
                uint32_t polls = 0;
                for (;;) {
                    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(ready) : "r"(sbase + L::READY)
                                 : "memory");
                    if ((int)ready > t) break;
                    if (++polls == kMaxPolls) break;
                }
                if ((int)ready <= t) {   // the scheduler stalled: give up on the rest of the tile
                    atomicOr(p.fault, 1u);
                    faulted = true;
                    break;
                }
                const int n = min((int)ready - t, kIssueBatch);
                tc_fence_after();
                for (int i = 0; i < n; ++i, ++t) {
                    const bool first = gin == 0;
                    const bool last = (gin == p.ktg - 1) || (t == KTL() - 1);
                    const int buf = g & 1;
                    const uint32_t d = tmem + (uint32_t)(buf * C::ACCW);
                    const uint32_t a_tile = tmem_a0 + (uint32_t)(sa * kAStageCols + h * (BK / 2));
                    const uint64_t b_desc = b_desc0 + (uint64_t)(sb * (L::STAGE >> 4));
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t bd = b_desc + 2u * kk;
                        mma_f16_ts(d, a_tile + 8u * kk, bd, idesc, (first && kk == 0) ? 0u : 1u);
                        if constexpr (!C::STACK) mma_f16_ts(d, a_tile + 8u * kk, bd + kPlaneStep, idesc, 1u);
                    }
                    mma_commit(empty_b(sb));
                    if (last) {
                        mma_commit(acc_full(buf));
                        gin = 0;
                        ++g;
                    } else {
                        ++gin;
                    }
                    if (h == kTilesPerA - 1 || t == KTL() - 1) mma_commit(empty_a(sa));
                    if (++sb == NS) sb = 0;
                    if (++h == kTilesPerA) {
                        h = 0;
                        if (++sa == NA) sa = 0;
                    }
                }
            }
            drain(NS, KTL(), empty_b);
            drain(NA, n_astages, empty_a);
        }
      }
    } else if (warp < kWarpEpi0) {
        set_regs<C::REGS_DQ, C::LAUNCH_REGS>();
        // ---- dequant: warp w writes TMEM lanes 32 (w % 4) .. + 31 (thread =
        // one weight row) for its K tiles of every A stage --------------------
        const int q = warp & 3;
        // with two dequant warpgroups each writes one K tile of an A stage,
        // with one it writes both
        const int h_begin = C::DQG == 2 ? (warp - kWarpDq0) >> 2 : 0;
        const int h_end = C::DQG == 2 ? h_begin + 1 : kTilesPerA;
        const int r = q * 32 + lane;
        const int64_t m = min(m0 + r, p.M - 1);
        const int64_t srow = p.scale_rows == 1 ? 0 : m;
        const uint32_t swz = (uint32_t)(r & 7);
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        // Zero points of groups g + 1 .. g + 4 are in flight while group g is
        // processed: every thread reads its own row, so these loads are not
        // coalesced and take longer than a few K tiles under load.
        const float* zrow = p.zeros + srow * p.groups + G0();
        float z_cur = __ldg(zrow);
        float z_n1 = NGL() > 1 ? __ldg(zrow + 1) : 0.0f;
        float z_n2 = NGL() > 2 ? __ldg(zrow + 2) : 0.0f;
        float z_n3 = NGL() > 3 ? __ldg(zrow + 3) : 0.0f;
        float z_n4 = NGL() > 4 ? __ldg(zrow + 4) : 0.0f;
        int g = 0, gin = h_begin;   // this warp's next tile t = 2 ja + h is tile gin of group g
        auto next_group = [&]() {
            gin -= p.ktg;
            ++g;
            z_cur = z_n1;
            z_n1 = z_n2;
            z_n2 = z_n3;
            z_n3 = z_n4;
            if (g + 4 < NGL()) z_n4 = __ldg(zrow + g + 4);
        };
        while (gin >= p.ktg) next_group();
        const int nct = (KTL() + L::KC - 1) / L::KC;
        int sa = 0, c = 0, ja = 0;
        uint32_t pha = 0, cph = 0;
        for (int ct = 0; ct < nct; ++ct) {
            wait_warp(c_full(c), cph);
            const unsigned char* crow = smem + L::C_OFF + c * L::C_STAGE + r * kCodeRowBytes;
            for (int js = 0; js < L::KC / kTilesPerA && ja < n_astages; ++js, ++ja) {
                if (ja >= NA) wait_warp(empty_a(sa), pha ^ 1u);
                tc_fence_after();
                for (int h = h_begin; h < h_end; ++h) {
                  const int t = kTilesPerA * ja + h;
                  if (t < KTL()) {
                    const int kin = kTilesPerA * js + h;   // K tile inside the codes stage
                    const __half zh = __float2half_rn(1024.0f + zero_int(z_cur));   // exact
                    const uint32_t zz = (uint32_t)__half_as_ushort(zh) * 0x10001u;
                    uint32_t a[32];
                    if constexpr (BITS == 4) {
                        // K tile = 16-byte chunks 2 kin, 2 kin + 1 of the row (swizzled)
                        const uint4 c0 = *reinterpret_cast<const uint4*>(crow + (((uint32_t)(2 * kin) ^ swz) << 4));
                        const uint4 c1 = *reinterpret_cast<const uint4*>(crow + (((uint32_t)(2 * kin + 1) ^ swz) << 4));
                        const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
                        for (int cc = 0; cc < 8; ++cc) {
                            const uint4 v = dq8_int4(w[cc], zz);
                            a[4 * cc] = v.x; a[4 * cc + 1] = v.y; a[4 * cc + 2] = v.z; a[4 * cc + 3] = v.w;
                        }
                    } else {
                        uint32_t w[16];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint4 v = *reinterpret_cast<const uint4*>(crow + (((uint32_t)(4 * kin + i) ^ swz) << 4));
                            w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
                        }
#pragma unroll
                        for (int cc = 0; cc < 8; ++cc) {
                            const uint4 v = dq8_int8(w[2 * cc], w[2 * cc + 1], zz);
                            a[4 * cc] = v.x; a[4 * cc + 1] = v.y; a[4 * cc + 2] = v.z; a[4 * cc + 3] = v.w;
                        }
                    }
                    tmem_st32(tmem_a0 + lane_base + (uint32_t)(sa * kAStageCols + h * (BK / 2)), a);
                  }
                  if (h + 1 < h_end) {   // the next tile of the same A stage
                    ++gin;
                    while (gin >= p.ktg) next_group();
                  }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(full_a(sa));
                gin += kTilesPerA - (h_end - 1 - h_begin);   // on to this warp's first tile of the next stage
                while (gin >= p.ktg) next_group();
                if (++sa == NA) {
                    sa = 0;
                    pha ^= 1u;
                }
            }
            // every code this warp read from the stage has reached tcgen05.st;
            // the proxy fence orders the reads before the TMA unit refills it
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(c_empty(c));
            if (++c == kNC) {
                c = 0;
                cph ^= 1u;
            }
        }
    } else {
        set_regs<C::REGS_EPI, C::LAUNCH_REGS>();
        // ---- epilogue: thread owns row r of the tile, EW of the BN columns
        // (epilogue warpgroup e: columns c0 .. c0 + EW - 1) ------------------------
        const int q = warp & 3;                 // TMEM lane quarter this warp may access
        const int r = q * 32 + lane;
        constexpr int EW = C::EW;
        const int64_t m = m0 + r;
        const int64_t srow = p.scale_rows == 1 ? 0 : min(m, (int64_t)p.M - 1);
        const int c0 = C::EPG == 1 ? 0 : ((warp - kWarpEpi0) >> 2) * EW;
        float acc[EW];
#pragma unroll
        for (int i = 0; i < EW; ++i) acc[i] = 0.0f;
        // scales of groups g + 1 .. g + 4 are in flight while group g is read
        const float* srow_p = p.scales + srow * p.groups + G0();
        float sc_n1 = NGL() > 1 ? __ldg(srow_p + 1) : 0.0f;
        float sc_n2 = NGL() > 2 ? __ldg(srow_p + 2) : 0.0f;
        float sc_n3 = NGL() > 3 ? __ldg(srow_p + 3) : 0.0f;
        float sc_n4 = NGL() > 4 ? __ldg(srow_p + 4) : 0.0f;
        float sc = __ldg(srow_p);
        // zero points of groups g + 1, g + 2 in flight, for the dz term
        const float* zrow_p = p.zeros + srow * p.groups + G0();
        float zc = __ldg(zrow_p);
        float z_n1 = NGL() > 1 ? __ldg(zrow_p + 1) : 0.0f;
        float z_n2 = NGL() > 2 ? __ldg(zrow_p + 2) : 0.0f;
        for (int g = 0; g < NGL(); ++g) {
            const int buf = g & 1, use = g >> 1;
            wait_warp(acc_full(buf), (uint32_t)(use & 1));
            tc_fence_after();
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * C::ACCW);
            if constexpr (BN > 128) {
                // 32 columns per load (each load waits for its data: fewer,
                // wider loads drain the accumulator in fewer round trips)
#pragma unroll
                for (int cc = 0; cc < EW / 32; ++cc) {
                    float v[32];
                    tmem_ld32(taddr + (uint32_t)c0 + 32u * cc, v);
#pragma unroll
                    for (int i = 0; i < 32; ++i) acc[cc * 32 + i] = fmaf(sc, v[i], acc[cc * 32 + i]);
                }
            } else {
                // stacked planes: the hi sums, then the lo sums BN columns further
#pragma unroll
                for (int pl = 0; pl < (C::STACK ? 2 : 1); ++pl) {
#pragma unroll
                    for (int cc = 0; cc < BN / 32; ++cc) {
                        float v[32];
                        tmem_ld32(taddr + (uint32_t)(pl * BN) + 32u * cc, v);
#pragma unroll
                        for (int i = 0; i < 32; ++i) acc[cc * 32 + i] = fmaf(sc, v[i], acc[cc * 32 + i]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty(buf));
            // fractional zero points: acc -= scale * dz * sum_{k in g} x' S_b
            // (rows with dz = 0 add 0 * sum, which leaves acc unchanged)
            const float dz = zc - zero_int(zc);
            if (__any_sync(0xffffffffu, dz != 0.0f)) {
                const float cz = -(sc * dz);
                const float4* xs = reinterpret_cast<const float4*>(p.xsum + (int64_t)(G0() + g) * p.bpad + n0 + c0);
#pragma unroll
                for (int i = 0; i < EW / 4; ++i) {
                    const float4 v = __ldg(xs + i);
                    acc[4 * i] = fmaf(cz, v.x, acc[4 * i]);
                    acc[4 * i + 1] = fmaf(cz, v.y, acc[4 * i + 1]);
                    acc[4 * i + 2] = fmaf(cz, v.z, acc[4 * i + 2]);
                    acc[4 * i + 3] = fmaf(cz, v.w, acc[4 * i + 3]);
                }
            }
            zc = z_n1;
            z_n1 = z_n2;
            if (g + 3 < NGL()) z_n2 = __ldg(zrow_p + g + 3);
            sc = sc_n1;
            sc_n1 = sc_n2;
            sc_n2 = sc_n3;
            sc_n3 = sc_n4;
            if (g + 5 < NGL()) sc_n4 = __ldg(srow_p + g + 5);
        }
        bool write = true;
        if constexpr (SPLIT) {
            // Split-K: the CTA's sums go to its partial slot; the last of the
            // tile's splits to arrive adds all slots in split order (a fixed
            // order, whichever CTA is last) and writes y.
            const int tile = m_tile * p.tiles_n + n_tile;
            const size_t tile_stride = (size_t)p.tiles_m * p.tiles_n * BN * BM;
            float* mine = p.part + (size_t)blockIdx.y * tile_stride + (size_t)tile * BN * BM;
#pragma unroll
            for (int i = 0; i < EW; ++i) mine[(c0 + i) * BM + r] = acc[i];
            __threadfence();
            named_barrier(1, 128 * C::EPG);   // the epilogue warpgroups
            volatile uint32_t* flag = reinterpret_cast<volatile uint32_t*>(smem + L::FLAG);
            if (warp == kWarpEpi0 && lane == 0) {
                const int prev = atomicAdd(p.counters + tile, 1);
                const bool last = prev == p.splits - 1;
                if (last) p.counters[tile] = 0;
                *flag = last ? 1u : 0u;
            }
            named_barrier(1, 128 * C::EPG);
            write = *flag != 0u;
            if (write) {
                __threadfence();
#pragma unroll
                for (int i = 0; i < EW; ++i) acc[i] = 0.0f;
                for (int sp = 0; sp < p.splits; ++sp) {
                    const float* src = p.part + (size_t)sp * tile_stride + (size_t)tile * BN * BM;
#pragma unroll
                    for (int i = 0; i < EW; ++i) acc[i] += __ldcg(src + (c0 + i) * BM + r);
                }
            }
        }
        if (write && m < p.M) {
            // y = acc * 2^-S_b, then the layer's bias (linear.py:99-100) as one
            // fp32 add after the product, like the reference (the _rn intrinsics
            // keep the two roundings apart). Without a bias the add is of -0.0,
            // which returns every value unchanged.
            const float bm = p.bias != nullptr ? __ldg(p.bias + m) : -0.0f;
            // Every output buffer gets the tile; stores to peer-mapped buffers
            // travel over NVLink while other tiles still compute. No fence:
            // the kernel's completion makes its peer stores visible to work
            // ordered after it, and the caller orders the ranks after the call.
            // columns n0 + c0 + i, i < nv, of rows n of y: one running pointer
            const int nv = min(EW, p.B - (n0 + c0));
            const float* is = p.inv_s + n0 + c0;
            if (p.y_all != nullptr) {
                // one store reaches every rank's y through the NVLink switch
                float* yp = p.y_all + (int64_t)(n0 + c0) * p.ldy + m;
#pragma unroll
                for (int i = 0; i < EW; ++i) {
                    if (i < nv) st_all_ranks(yp, __fadd_rn(__fmul_rn(acc[i], __ldg(is + i)), bm));
                    yp += p.ldy;
                }
            } else {
                for (int d = 0; d <= p.n_extra; ++d) {
                    float* yp = (d == 0 ? p.y : p.y_extra[d - 1]) + (int64_t)(n0 + c0) * p.ldy + m;
#pragma unroll
                    for (int i = 0; i < EW; ++i) {
                        if (i < nv) *yp = __fadd_rn(__fmul_rn(acc[i], __ldg(is + i)), bm);
                        yp += p.ldy;
                    }
                }
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

// x' = x * channel, S_b from max|x'_b|, fp16 hi/lo planes written in the
// tiled, swizzled form the kernel copies verbatim: batch tile nt = b / BN,
// row r = b % BN, K tile kt = k / 64, 16-byte chunk c = (k % 64) / 8 at byte
// ((nt * KT + kt) * 2 + plane) * BN * 128 + r * 128 + ((c ^ (r & 7)) << 4).
// Rows b >= B (padding of the last batch tile) are written as zeros. For
// int4 layers (`nibble_order`) the 8 values of a chunk are stored in the order
// k0 k4 k1 k5 k2 k6 k3 k7, matching the order the dequant warps produce A in.
// Also xsum[g * bpad + b] = sum of x' * S_b over group g (gsz values; warp w
// sums groups w, w + 8, ..., lanes strided then a butterfly: a fixed order).
__global__ void __launch_bounds__(256) prep_x_kernel(const float* x, const float* channel, int B, int K, int KT,
                                                     int BN, bool nibble_order, unsigned char* planes, float* inv_s,
                                                     int gsz, int ngroups, int bpad, float* xsum, int* counters,
                                                     int ncounters) {
    __shared__ float red[8];
    // x may be the previous kernel's output; the tensor-core kernel that
    // follows waits for this one to complete before it reads the planes
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int b = blockIdx.x;
    if (b == 0)   // split-K arrival counters of the tensor-core kernel that follows
        for (int i = threadIdx.x; i < ncounters; i += blockDim.x) counters[i] = 0;
    const bool real = b < B;
    const float* xb = x + (int64_t)(real ? b : 0) * K;
    float mx = 0.0f;
    if (real) {
        for (int k = threadIdx.x; k < K; k += blockDim.x) {
            float v = xb[k];
            if (channel != nullptr) v = v * channel[k];
            mx = fmaxf(mx, fabsf(v));
        }
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
    if (threadIdx.x == 0 && real) inv_s[b] = pow2i(e - 14);
    const int nt = b / BN, r = b - nt * BN;
    const size_t plane_bytes = (size_t)BN * 128;
    for (int ch = threadIdx.x; ch < KT * 8; ch += blockDim.x) {
        const int k0 = ch * 8, kt = ch >> 3, c = ch & 7;
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float u[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int k = k0 + (nibble_order ? i + 4 * j : 2 * i + j);
                float t = 0.0f;
                if (real && k < K) {
                    t = xb[k];
                    if (channel != nullptr) t = t * channel[k];
                    t = t * S;
                }
                u[j] = t;
            }
            const __half h0 = __float2half_rn(u[0]), h1 = __float2half_rn(u[1]);
            const __half l0 = __float2half_rn(u[0] - __half2float(h0)), l1 = __float2half_rn(u[1] - __half2float(h1));
            hw[i] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
            lw[i] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        }
        unsigned char* tile = planes + ((size_t)nt * KT + kt) * 2 * plane_bytes;
        const size_t off = (size_t)r * 128 + ((uint32_t)(c ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(tile + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(tile + plane_bytes + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int g = warp; g < ngroups; g += (int)(blockDim.x >> 5)) {
        float acc = 0.0f;
        if (real) {
            const int k1 = min(K, (g + 1) * gsz);
            for (int k = g * gsz + lane; k < k1; k += 32) {
                float t = xb[k];
                if (channel != nullptr) t = t * channel[k];
                acc += t * S;
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) xsum[(int64_t)g * bpad + b] = acc;
    }
}

// ---- host side ----------------------------------------------------------------
int64_t kt_of(int64_t K) { return (K + BK - 1) / BK; }
// Batch tile: N = 192 for large batches (each MMA then carries 1.5x the work
// of N = 128 for the same issue cost, with the accumulators still
// double-buffered in tensor memory), else the smallest of 32/64/128 that
// covers the batch.
int bn_of(int64_t B) { return B <= 32 ? 32 : (B <= 64 ? 64 : (B < 1024 ? 128 : 192)); }
int64_t bpad_of(int64_t B) { const int bn = bn_of(B); return (B + bn - 1) / bn * bn; }

// Groups as the kernel walks them: one per group_size (a multiple of BK),
// or one for the whole row.
int64_t ngroups_of(int64_t K, int group_size) { return group_size >= K ? 1 : (K + group_size - 1) / group_size; }
int64_t round256(int64_t v) { return (v + 255) / 256 * 256; }

// Split-K plan. When the output tiles fill less than half of the SMs' CTA
// slots (small layers, or few rows per GPU), each tile's K range is cut into
// `splits` parts on boundaries of `gran` K tiles: a multiple of the group (so
// every part holds whole groups) and of the code stage (so every part starts
// a TMA box). Layers of one group are not split.
struct SplitPlan {
    int splits, gran;
};

SplitPlan split_plan(int64_t B, int64_t M, int64_t K, int group_size, int bits) {
    SplitPlan sp{1, 1};
    const int64_t KT = kt_of(K);
    if (ngroups_of(K, group_size) < 2) return sp;
    const int bn = bn_of(B);
    const int64_t tiles = ((M + BM - 1) / BM) * ((B + bn - 1) / bn);
    const int64_t slots = (int64_t)sm_count() * (bn >= 128 ? 1 : 2);
    if (2 * tiles > slots) return sp;
    const int kc = kCodeRowBytes / (bits == 4 ? 32 : 64);   // K tiles per code stage
    const int ktg = group_size / BK;
    int g = ktg;
    while (g % kc != 0) g += ktg;                            // lcm(ktg, kc)
    const int64_t units = (KT + g - 1) / g;
    int64_t n = slots / tiles;
    if (n > units) n = units;
    if (n > 16) n = 16;
    sp.splits = (int)(n < 1 ? 1 : n);
    sp.gran = g;
    return sp;
}

// Workspace: [planes: bpad * KT * BK * 4 B][inv_s: B floats, padded to 256 B]
// [xsum: ngroups * bpad floats][split-K partial tiles][split-K counters]
struct TcWorkspace {
    unsigned char* planes;
    float* inv_s;
    float* xsum;
    float* part;
    int* counters;
    SplitPlan plan;
    int64_t tiles;
};

TcWorkspace carve(void* ws, int64_t B, int64_t M, int64_t K, int group_size, int bits) {
    unsigned char* p = static_cast<unsigned char*>(ws);
    TcWorkspace w;
    const int bn = bn_of(B);
    w.plan = split_plan(B, M, K, group_size, bits);
    w.tiles = ((M + BM - 1) / BM) * ((B + bn - 1) / bn);
    const int64_t planes = bpad_of(B) * kt_of(K) * BK * 4;
    w.planes = p;
    p += planes;
    w.inv_s = reinterpret_cast<float*>(p);
    p += round256(B * 4);
    w.xsum = reinterpret_cast<float*>(p);
    p += round256(ngroups_of(K, group_size) * bpad_of(B) * 4);
    w.part = reinterpret_cast<float*>(p);
    if (w.plan.splits > 1) p += round256((int64_t)w.plan.splits * w.tiles * bn * BM * 4);
    w.counters = reinterpret_cast<int*>(p);
    return w;
}

template <int BN, int NS, int BITS, bool SPLIT>
cudaError_t launch_bn_t(const GemmProblem& g, const TcWorkspace& w, cudaStream_t s) {
    using L = Smem<BN, NS, BITS>;
    CUtensorMap mq;
    if (!encode_2d(&mq, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.q, (uint64_t)g.q_stride, (uint64_t)g.M,
                   (uint64_t)g.q_stride, kCodeRowBytes, BM, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    TcParams p;
    p.planes = w.planes;
    p.scales = g.scales;
    p.zeros = g.zeros;
    p.inv_s = w.inv_s;
    p.xsum = w.xsum;
    p.bpad = (int)bpad_of(g.B);
    p.y = g.y;
    p.n_extra = g.n_extra;
    p.y_all = g.y_all;
    p.bias = g.bias;
    p.part = w.part;
    p.counters = w.counters;
    p.splits = w.plan.splits;
    p.gran = w.plan.gran;
    for (int d = 0; d < 7; ++d) p.y_extra[d] = g.y_extra[d];
    p.fault = fault_word();
    if (p.fault == nullptr) return cudaErrorInvalidDevicePointer;
    p.M = (int)g.M;
    p.B = (int)g.B;
    p.KT = (int)kt_of(g.K);
    p.groups = g.groups;
    p.ktg = g.groups == 1 ? p.KT : g.group_size / BK;
    p.ngroups = (p.KT + p.ktg - 1) / p.ktg;
    p.scale_rows = g.scale_rows;
    p.tiles_m = (int)((g.M + BM - 1) / BM);
    p.tiles_n = (int)((g.B + BN - 1) / BN);
    {
        // the fewest bands whose x' fits kBandBytes, then equal band widths
        const int64_t per_tile = (int64_t)p.KT * 256 * BN;
        int64_t most = kBandBytes / per_tile;
        if (most < 1) most = 1;
        const int64_t bands = (p.tiles_n + most - 1) / most;
        p.band = (int)((p.tiles_n + bands - 1) / bands);
    }
    p.ldy = g.ldy;
    const size_t smem = (size_t)L::TOTAL + 1024;
    auto kern = dq_gemm_tc_kernel<BN, NS, BITS, SPLIT>;
    // Once per device: the shared-memory opt-in, and the register check. The
    // setmaxnreg split assumes the launch gives every thread exactly
    // LAUNCH_REGS registers; refuse to launch otherwise (the increase would
    // wait for registers that do not exist).
    constexpr int kDevs = 32;
    static std::atomic<int> ready[kDevs];   // 0 not yet checked, 1 ready, 2 wrong register count
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const int known = (dev >= 0 && dev < kDevs) ? ready[dev].load(std::memory_order_relaxed) : 0;
    if (known == 2) return cudaErrorInvalidConfiguration;
    if (known == 0) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        cudaFuncAttributes attr;
        e = cudaFuncGetAttributes(&attr, kern);
        if (e != cudaSuccess) return e;
        const bool ok = attr.numRegs == Cfg<BN>::LAUNCH_REGS;
        if (dev >= 0 && dev < kDevs) ready[dev].store(ok ? 1 : 2, std::memory_order_relaxed);
        if (!ok) return cudaErrorInvalidConfiguration;
    }
    const int64_t grid = (int64_t)p.tiles_m * p.tiles_n;
    if (grid > 0x7fffffff) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid, (unsigned)p.splits);
    cfg.blockDim = dim3(Cfg<BN>::THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p, mq);
}

// the split-K epilogue is a separate instantiation, so the unsplit kernel
// (large batches) keeps its register allocation
template <int BN, int NS, int BITS>
cudaError_t launch_bn(const GemmProblem& g, const TcWorkspace& w, cudaStream_t s) {
    return w.plan.splits > 1 ? launch_bn_t<BN, NS, BITS, true>(g, w, s) : launch_bn_t<BN, NS, BITS, false>(g, w, s);
}

}  // namespace

bool tc_supported(const GemmProblem& p) {
    if (p.B < 5 || p.M < 1 || p.K < 1) return false;
    if (p.q_stride % 16 != 0 || (reinterpret_cast<uintptr_t>(p.q) & 15) != 0) return false;
    if (p.groups > 1 && p.group_size % BK != 0) return false;
    if (p.M > 0x7fffff00 || p.B > 0x7fffff00) return false;
    if (kt_of(p.K) > 0x7fffffff / 8) return false;
    return encode_fn() != nullptr;
}

size_t tc_workspace_bytes(int64_t B, int64_t M, int64_t K, int group_size, int bits) {
    // fp16 hi + lo planes of the padded batch, 1/S_b, per-group sums of x' S_b,
    // and for split-K the partial tiles and one counter per output tile
    const SplitPlan sp = split_plan(B, M, K, group_size, bits);
    const int bn = bn_of(B);
    const int64_t tiles = ((M + BM - 1) / BM) * ((B + bn - 1) / bn);
    int64_t bytes = bpad_of(B) * kt_of(K) * BK * 4 + round256(B * 4) + round256(ngroups_of(K, group_size) * bpad_of(B) * 4);
    if (sp.splits > 1) bytes += round256((int64_t)sp.splits * tiles * bn * BM * 4);
    return (size_t)(bytes + round256(tiles * 4) + 256);
}

cudaError_t launch_tc(const GemmProblem& g, void* workspace, cudaStream_t s) {
    const TcWorkspace w = carve(workspace, g.B, g.M, g.K, g.group_size, g.bits);
    const int bn = bn_of(g.B);
    const int64_t bpad = bpad_of(g.B);
    const int64_t ng = ngroups_of(g.K, g.group_size);
    const int gsz = ng == 1 ? (int)g.K : g.group_size;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)bpad);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, prep_x_kernel, g.x, g.channel, (int)g.B, (int)g.K, (int)kt_of(g.K), bn,
                                       g.bits == 4, w.planes, w.inv_s, gsz, (int)ng, (int)bpad, w.xsum, w.counters,
                                       w.plan.splits > 1 ? (int)w.tiles : 0);
    if (e != cudaSuccess) return e;
    // x' stage counts: 192 KB of planes next to two 16 KB codes stages
    if (g.bits == 4) {
        if (bn == 32) return launch_bn<32, 4, 4>(g, w, s);
        if (bn == 64) return launch_bn<64, 4, 4>(g, w, s);
        if (bn == 128) return launch_bn<128, 6, 4>(g, w, s);
        return launch_bn<192, 4, 4>(g, w, s);
    }
    if (bn == 32) return launch_bn<32, 4, 8>(g, w, s);
    if (bn == 64) return launch_bn<64, 4, 8>(g, w, s);
    if (bn == 128) return launch_bn<128, 6, 8>(g, w, s);
    return launch_bn<192, 4, 8>(g, w, s);
}

}  // namespace wq

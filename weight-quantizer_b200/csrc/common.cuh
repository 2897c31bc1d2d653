// Shared device helpers for the wq_b200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "wq_b200 kernels are written for sm_100a (B200) only"
#endif

namespace wq {

constexpr int kWarp = 32;

// 16-byte streaming load that bypasses L1 allocation: the packed weight stream
// is read exactly once per launch, so it should not evict the staged
// activations from L1/shared memory.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float ld_ro(const float* p) { return __ldg(p); }

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Asynchronous global -> shared copies (cp.async). With `valid` false the
// source size is 0: nothing is read and the destination is zero-filled.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_addr(dst)), "l"(src),
                 "r"(valid ? 4 : 0)
                 : "memory");
}
// Same, with the destination given as a shared-window address.
__device__ __forceinline__ void cp_async16_s(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async4_s(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(valid ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- named barriers, mbarriers and bulk (TMA linear) copies ---------------
__device__ __forceinline__ void named_barrier(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Global -> shared bulk copy into this CTA only, completing on `bar`. Both
// addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
// L2 policy that keeps lines past ordinary ones (evict_last) for all of a
// copy's bytes, and the bulk copy above with that policy as its L2 hint.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_copy_g2s_hint(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                                   uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}
// Orders this thread's generic-proxy shared-memory accesses (and those it has
// observed) before later async-proxy accesses (TMA, bulk copies, tcgen05) to
// the same shared memory, and the reverse.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// One non-blocking probe of a phase (never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Every wait on an mbarrier in this library gives up after this many polls
// (each poll may suspend the thread for a short hardware-defined time).
constexpr uint32_t kMaxPolls = 1u << 22;
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    for (uint32_t n = 0; n < kMaxPolls; ++n)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}


__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Warp reduce-scatter of V (power of two, <= 8) values per lane: returns the
// full warp sum of value `idx`, held by the lanes whose index is a multiple of
// 32 / V (lane = idx * 32 / V). log2(V) halving exchanges, then plain rounds;
// the summation order is fixed, so results are deterministic.
template <int V>
__device__ __forceinline__ float warp_reduce_scatter(const float (&v)[V], int lane, int& idx) {
    if constexpr (V == 1) {
        idx = 0;
        return warp_sum(v[0]);
    } else {
        float w[V];
#pragma unroll
        for (int i = 0; i < V; ++i) w[i] = v[i];
        int n = V;
        int off = 16;
        idx = 0;
#pragma unroll
        for (int round = 0; round < 3; ++round) {
            if (n == 1) break;
            const bool hi = (lane & off) != 0;
            const int h = n / 2;
#pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                if (i < h) {
                    const float send = hi ? w[i] : w[i + h];
                    const float keep = hi ? w[i + h] : w[i];
                    w[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                }
            }
            idx = idx * 2 + (hi ? 1 : 0);
            n = h;
            off >>= 1;
        }
        float z = w[0];
        for (; off > 0; off >>= 1) z += __shfl_xor_sync(0xffffffffu, z, off);
        return z;
    }
}

// Exact power of two 2^e for e in [-126, 127] built from its bit pattern.
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

}  // namespace wq

// fp16 operands of the tcgen05 kind::f16 dequant-GEMM kernels (sm_100a):
// packed codes -> exact fp16 (code - zi) in registers.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace wq {

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));  // (a & b) | c
    return d;
}
__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}

// The integer zero point A is built with: rint(zero) clamped to [0, 1023]
// (1024 + zi is then exact in fp16; NaN maps to 0 and reaches y through the
// epilogue's dz term, as it reaches the reference's (code - zero)).
__device__ __forceinline__ float zero_int(float z) { return fminf(fmaxf(rintf(z), 0.0f), 1023.0f); }

// 8 int4 codes (one 32-bit word, k ascending) -> 8 fp16 values (code - zi)
// in the order the nibble masks produce them, k0 k4 k1 k5 k2 k6 k3 k7; the
// prep kernel stores the x' planes of int4 layers in the same order inside
// every group of 8, so the products pair up without a byte shuffle.
// zz = half2(1024 + zi) twice.
__device__ __forceinline__ uint4 dq8_int4(uint32_t w, uint32_t zz) {
    return make_uint4(hsub2_u32(lop3_and_or(w, 0x000F000Fu, 0x64006400u), zz),          // k0, k4
                      hsub2_u32(lop3_and_or(w >> 4, 0x000F000Fu, 0x64006400u), zz),     // k1, k5
                      hsub2_u32(lop3_and_or(w >> 8, 0x000F000Fu, 0x64006400u), zz),     // k2, k6
                      hsub2_u32(lop3_and_or(w >> 12, 0x000F000Fu, 0x64006400u), zz));   // k3, k7
}
// 8 int8 codes (two words) -> 8 fp16 (code - zi)
__device__ __forceinline__ uint4 dq8_int8(uint32_t a, uint32_t b, uint32_t zz) {
    const uint32_t e = 0x64646464u;
    return make_uint4(hsub2_u32(__byte_perm(a, e, 0x4140), zz), hsub2_u32(__byte_perm(a, e, 0x4342), zz),
                      hsub2_u32(__byte_perm(b, e, 0x4140), zz), hsub2_u32(__byte_perm(b, e, 0x4342), zz));
}

}  // namespace wq

// k_gemv_core.cuh -- the decode GEMV's per-fragment primitives (LUT decode of Q4L nibbles with PRMT, the int8 MMA
// whose accumulator starts at the bits of 1.5 * 2^23, fp16 scale pairs), shared by k_gemv.cu and the fused decode
// kernel (k_fused.cu).
#pragma once

#include <cuda_fp16.h>
#include <string.h>

#include "inzg_internal.h"

namespace inzg {

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Pipe balancing: `one` is a kernel argument equal to 1 that the compiler cannot fold, so the integer multiply-adds
// below stay IMADs (FMA pipe) instead of becoming adds, shifts or selects on the ALU pipe, which the PRMT-based LUT
// decode already fills.
// 4 nibble selectors (bits 0..15 of w; wx = w ^ 0x8888) -> 4 LUT bytes. Levels are <= 127, so a selector with bit 3
// set makes PRMT replicate a zero sign bit: each half-table lookup yields 0 where the other half applies, and the two
// halves are added (disjoint bytes, so the sum is the byte-wise merge).
__device__ __forceinline__ uint32_t lut16(uint32_t w, uint32_t wx, uint4 T, uint32_t one) {
    return prmt(T.x, T.y, w) * one + prmt(T.z, T.w, wx);
}

// the high 16 bits of w (bits 16..31 -> 0..15): w * 2^16 >> 32 on the integer multiplier (k16 = one << 16)
__device__ __forceinline__ uint32_t hi16(uint32_t w, uint32_t k16) { return __umulhi(w, k16); }

__device__ __forceinline__ float2 h2f16x2(uint32_t bits) {
    __half2 h;
    memcpy(&h, &bits, 4);
    return __half22float2(h);
}

__device__ __forceinline__ float h2f16(uint32_t bits) { return __half2float(__ushort_as_half((unsigned short)bits)); }

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D = A * B + c (the same c in all four accumulator slots)
__device__ __forceinline__ void mma_u8s8_c(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                           uint32_t b1, int c) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c));
}

}  // namespace inzg

// fp16 fragment helpers shared by the batch-1 decode and the greedy LM head (sm_100a): int4 words
// dequantised into exact fp16 integers for mma.sync, and the Veltkamp split of an activation into
// fp16 high and low parts.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace gtm {

// ---- fp16 fragments ------------------------------------------------------------------------
// Dequantise one 32-bit word (8 int4, low nibble first) into four fp16x2 registers with one LOP3
// each: (1024+n0, 1024+n4), (1024+16n1, 1024+16n5), (1024+n2, 1024+n6), (1024+16n3, 1024+16n7),
// all exact in fp16. The activation table carries x for the even elements and x/16 for the odd
// ones, so each product is 1024*x + n*x or 64*x + n*x; the per-group constant
// C = 1024 * sum(x_even) + 64 * sum(x_odd) is subtracted once per group in fp32.
__device__ __forceinline__ void dq_word(uint32_t w, uint32_t (&r)[4]) {
    const uint32_t m = 0x64006400u;                         // fp16 1024.0 in both halves
    const uint32_t w8 = w >> 8;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r[0]) : "r"(w), "r"(0x000F000Fu), "r"(m));
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r[1]) : "r"(w), "r"(0x00F000F0u), "r"(m));
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r[2]) : "r"(w8), "r"(0x000F000Fu), "r"(m));
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r[3]) : "r"(w8), "r"(0x00F000F0u), "r"(m));
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Builds the fragment table of `groups` 64-element groups of the fp32 vector v (in shared
// memory): for thread column t and part hl (0 = fp16 high part, 1 = low part) the 16 elements
// 16t..16t+15 as (x0,x4)(x1,x5)(x2,x6)(x3,x7)(x8,x12)(x9,x13)(x10,x14)(x11,x15), odd elements
// divided by 16 (exact). Also per-group sums xs (for the bias) and the offset constants cs.
// hi + lo = b with hi = b rounded to 11 significant bits (Veltkamp split, exact in fp32) and lo =
// b - hi; converted in pairs with one packed instruction each. hi is exact in fp16 for
// |b| >= 2^-14; below that the fp16 conversion rounds it again (an absolute error under 2^-25).
__device__ __forceinline__ void split11(float b, float& hi, float& lo) {
    const float c = __fmul_rn(b, 8193.0f);
    hi = __fsub_rn(c, __fsub_rn(c, b));
    lo = __fsub_rn(b, hi);
}
__device__ __forceinline__ uint32_t cvt2(float lo_half, float hi_half) {   // (low 16 bits, high 16 bits)
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi_half), "f"(lo_half));
    return r;
}

}  // namespace gtm

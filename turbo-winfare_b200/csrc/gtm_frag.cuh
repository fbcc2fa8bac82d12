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


// ---- integer products: u8 nibbles x three s8 limbs of the activation -------------------------------
// mma.sync.m16n8k32 (u8 x s8 -> s32): a0/a2 the nibbles 0,2,4,6 / 1,3,5,7 of row g's word (one u8
// each), a1/a3 the same of row g + 8; b0/b1 the activation limbs of those K slots in column g.
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}


// The low bytes of four words, a in the lowest.
__device__ __forceinline__ uint32_t pack_s8(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// Activation limb tables. Per 64-element group: x = 2^(E-6) (L0 + L1 2^-7 + L2 2^-14), |x| < 2^E,
// three signed limbs of at most 64 in magnitude, so every element is carried to 2^-21 of the
// group's largest; integer accumulation is exact. Per group the table also keeps
// (sum of x, 2^(E-6)) for the bias term and the scale.
// The limbs of 16 elements of a 64-element group whose four 16-element parts sit in four adjacent
// lanes (whole warps call it: the lanes share the group's largest magnitude and its sum). L[l][e]
// holds limb l of element e in its low byte (two's complement); sx = sum of the group's x, sE =
// 2^(E-6).
__device__ __forceinline__ void limb_decompose(const float (&x)[16], uint32_t (&L)[3][16], float& sx_out, float& sE) {
    float mx = 0.0f, sx = 0.0f;
#pragma unroll
    for (int e = 0; e < 16; ++e) { mx = fmaxf(mx, fabsf(x[e])); sx += x[e]; }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    sx += __shfl_xor_sync(0xffffffffu, sx, 1);
    sx += __shfl_xor_sync(0xffffffffu, sx, 2);
    // |x| < 2^E for the group (exponent field of the largest magnitude, minus 126), kept >= -120
    const int E = max((int)((__float_as_uint(mx) >> 23) & 0xFFu) - 126, -120);
    const float up = __int_as_float((127 + 6 - E) << 23);     // 2^(6-E): |x up| < 64
    // round to nearest even by adding 1.5 * 2^23 (|v| <= 64): the sum's low mantissa bits are the
    // integer, whose low byte is the limb in two's complement; all steps are exact
    constexpr float kMagic = 12582912.0f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        const float v = x[e] * up;                            // exact (power of two)
        const float f0 = v + kMagic;
        const float v1 = (v - (f0 - kMagic)) * 128.0f;        // exact; |v1| <= 64
        const float f1 = v1 + kMagic;
        const float f2 = (v1 - (f1 - kMagic)) * 128.0f + kMagic;
        L[0][e] = __float_as_uint(f0);
        L[1][e] = __float_as_uint(f1);
        L[2][e] = __float_as_uint(f2);
    }
    sx_out = sx;
    sE = __int_as_float((127 + E - 6) << 23);
}

// Table of a vector, per quad Q (4 groups) and double group h: 12 lane entries of 8 words at (2 Q + h) * 96
// + e * 8, one per lane (g, t) that holds nonzero B values: g = 4 a + limb (limb < 3) with a = t >> 1
// (the lane pair of group 2 h + a), e = 6 a + 2 limb + (t & 1). Words 2 w, 2 w + 1 of the entry are
// the lane's b0, b1 for the MMA of word w: limb `limb` of the elements 128 h + 32 t + 8 w + {0, 2,
// 4, 6} and {1, 3, 5, 7} of the quad, one signed byte each (K slot 4 t + i and 4 t + 16 + i hold
// nibbles 2 i and 2 i + 1 of the lane's word w). The 12 reading lanes of a double group take 384
// consecutive bytes.
// One builder thread per (group j, sub): the 16 elements 16 sub + (0..15) of the group, i.e. words
// 2 (sub & 1) and 2 (sub & 1) + 1 of lane t = 2 (j & 1) + (sub >> 1) of the group's double group;
// the four builder lanes of a group (adjacent) share its largest magnitude and its sum. tbl_q is
// the quad's table, gq = j % 4.
constexpr int kLimbQuadWords = 192;   // words of one quad's table
__device__ __forceinline__ void limb_item(const float (&x)[16], bool on, uint32_t* tbl_q, int gq, int sub,
                                           float2* gs, int j) {
    uint32_t L[3][16];
    float sx, sE;
    limb_decompose(x, L, sx, sE);
    const int h = gq >> 1, a = gq & 1, tl = sub >> 1, wp = sub & 1;
    uint32_t* base = tbl_q + h * 96;
    if (on) {
#pragma unroll
        for (int limb = 0; limb < 3; ++limb) {
            uint32_t* ent = base + (6 * a + 2 * limb + tl) * 8;
#pragma unroll
            for (int ww = 0; ww < 2; ++ww) {
                const int b = 8 * ww;
                ent[2 * (2 * wp + ww)] = pack_s8(L[limb][b], L[limb][b + 2], L[limb][b + 4], L[limb][b + 6]);
                ent[2 * (2 * wp + ww) + 1] = pack_s8(L[limb][b + 1], L[limb][b + 3], L[limb][b + 5], L[limb][b + 7]);
            }
        }
        if (sub == 0) gs[j] = make_float2(sx, sE);
    }
}

}  // namespace gtm

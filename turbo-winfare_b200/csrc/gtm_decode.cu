// Fused batch-1 MoE decode for sm_100a: one persistent cooperative launch runs a token through
// `num_layers` MoE blocks with every expert resident in HBM and no host round trip.
//
// Replaces the per-layer MoE sequence of ForwardRunner::produce_token (src/runner.cpp:549-716):
// MulBF16 -> GemvInt8 -> RouterTopK -> CPU read-back -> shared expert (GemvInt4 x3, GeGLU,
// RMSNormK) -> per expert GemvInt4 gate/up, GeGLU, GemvInt4 down, ScaleAccum -> LayerTail.
//
// Int4 products (gemv_groups): weights are dequantised to fp16 in registers (exact integers
// 0..15, two LOP3 masks per nibble pair) and fed as the A operand of mma.sync.m16n8k16; the
// activation goes in as B split into an fp16 high part (column 0) and low part (column 1), so
// sum_k q_k * x_k comes out in fp32 to ~2^-22 of x. The group's bf16 scale and bias are applied
// in fp32 after each 64-element group: y += s * (d_hi + d_lo) + b * sum(x). A 16-row tile is
// either 8 gate rows on top of the same 8 up rows (so GeGLU happens in registers) or 16 rows of a
// down projection. tcgen05 would need the dequantised tile staged through shared memory for a
// one-column product; mma.sync consumes the register fragments the dequant produces directly.
//
// Per layer (one token), with split arrive/wait grid barriers (bounded waits):
//   P1  every CTA: layer tail of the previous layer from the down partials, optional
//       between-layer RMSNorm, views (dense_x, routed_x, router input); CTAs 0..127: one router
//       logit each in the reference's exact order (bit-identical logits)      -> arrive A1
//       every CTA: its share of the 264 shared gate/up tiles (+GeGLU)
//   P2  wait A1; top-8 (each CTA); L2-prefetch its routed down rows; its share of the 704 routed
//       gate/up tiles (+GeGLU)                                                -> arrive B
//   P3  wait B (every CTA's shared and routed activations); its share of the 1936 down items,
//       the shared down (3 thirds of K x 176 row tiles) and the routed down (8 experts x 176 row
//       tiles, partials x w_k) in one pass; L2-prefetch the next layer's router row, shared
//       gate/up and down                                                      -> arrive C
// The down partials [3 shared + 8 routed][2816] are summed in fixed order by the next tail.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gtm_common.cuh"
#include "gtm_internal.h"

namespace gtm {
namespace dec {

constexpr int D = 2816, FE = 704, FS = 2112, NE = 128, TOPK = 8;
constexpr int NT = 512, NW = NT / 32;
constexpr int GD = D / kGroup;            // 44 groups in a hidden-sized input
constexpr int GFE = FE / kGroup;          // 11
constexpr int GFS = FS / kGroup;          // 33
constexpr int TILES_R = TOPK * FE / 8;    // 704 routed gate/up tiles (8 row pairs each)
constexpr int TILES_S = FS / 8;           // 264 shared gate/up tiles
constexpr int OT = D / 16;                // 176 output row tiles of the down projection
constexpr int NSEG = 3 + TOPK;            // down partials: 3 shared thirds + 8 routed experts
constexpr int ITEMS_DN = OT * NSEG;       // 1936 down items: row tile item / NSEG, segment item % NSEG
constexpr int MAX_ITEMS = 17;             // per CTA and phase (down items over >= 118 CTAs)
constexpr int ROW_GU = D / 2;             // 1408 bytes per gate/up row
constexpr int RIN_PITCH = 65;
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr int ACT_R = TOPK * FE;          // 5632 routed activations, after the 2112 shared ones

enum { BAR_A1 = 0, BAR_B = 2, BAR_C = 3 };

struct Params {
    GtmLayer layers[GTM_MAX_LAYERS];
    GtmDecodeIO io;
    int num_layers;
    float eps;
    float inv_sqrt_d;
    unsigned* flags;   // [4][256]
    uint64_t wait_limit_ns;      // bound of every grid-barrier wait
    unsigned first_wait_extra;   // added to the first wait's epoch (test hook: 1 = never reached)
    int* err;
    int* sticky;
    float* logits;     // [NE]
    float* act;        // [FS + ACT_R]: shared activations, then the 8 routed slots (segment s at s * 704)
    float* part;       // [2 contributors][2: shared, routed][D] down sums (the rest of NSEG x D unused)
};

// B-operand fragment tables: per 64-element group, 8 slots (4 thread columns x hi/lo) of 8
// packed fp16 pairs, stored half-major so the 8 reading lanes hit consecutive 16-byte chunks.
constexpr int TBL_WORDS = 64;   // 32-bit words per group (256 bytes)

// Arrays read or written with 16-byte vector accesses or cp.async carry alignas(16).
struct Smem {
    alignas(16) float hid[D];
    alignas(16) float ab[2 * D];   // scratch: [0, D) and [D, 2D), or one 2D-float vector
    alignas(16) float rin[GD * RIN_PITCH];
    alignas(16) uint32_t tbl_r[GD * TBL_WORDS];        // routed_x
    alignas(16) uint32_t tbl_d[GD * TBL_WORDS];        // dense_x
    alignas(16) uint32_t tbl_dn[NSEG * GFE * TBL_WORDS];  // down inputs: shared act, then routed slots
    float xs_r[GD], xs_d[GD], xs_dn[NSEG * GFE];
    float cs_r[GD], cs_d[GD], cs_dn[NSEG * GFE];
    // bf16 norm vectors, copied ahead of use: this layer's pre_ffn_norm, pre_ffn_norm_2,
    // router.scale and the previous layer's post_ffn_norm_1, post_ffn_norm_2, post_ffn_norm
    alignas(16) uint16_t nw[6][D];
    alignas(16) uint16_t pes[NE];   // per_expert_scale of the layer (copied with the pre-FFN norms)
    float slot[MAX_ITEMS][NW][16];
    float terms[GD];
    double red[40];
    double red2[2][NW][2];   // two-value block reductions, double-buffered
    float topw[TOPK];
    int topi[TOPK];
    int flag;
};

static_assert(offsetof(Smem, nw) % 16 == 0 && offsetof(Smem, ab) % 16 == 0 && offsetof(Smem, tbl_r) % 16 == 0 &&
                  offsetof(Smem, tbl_d) % 16 == 0 && offsetof(Smem, tbl_dn) % 16 == 0 &&
                  offsetof(Smem, hid) % 16 == 0,
              "vector-accessed shared arrays must be 16-byte aligned");

__device__ __forceinline__ const uint8_t* rp(const void* base, uint64_t off) {
    return static_cast<const uint8_t*>(base) + off;
}
__device__ __forceinline__ const uint16_t* rp16(const void* base, uint64_t off) {
    return reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(base) + off);
}

__device__ __forceinline__ uint2 ldg_nc_u2(const void* p) {
    uint2 v;
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint16_t ldg_nc_u16(const void* p) {
    uint16_t v;
    asm("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}
// L2 prefetch hint for [p, p + bytes): one prefetch.global.L2 per 128-byte line, the warp's lanes
// striding over the lines. Per-thread hints cost the issuing warp next to nothing, whereas a bulk
// prefetch is a TMA operation (~64 cycles each, measured) and a warp issuing dozens of small ones
// blocked for microseconds while the other warps waited for it at the phase's first barrier.
__device__ __forceinline__ void prefetch_lines(const void* p, uint32_t bytes, int lane) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    for (uint32_t o = (uint32_t)lane * 128u; o < bytes; o += 32u * 128u)
        asm volatile("prefetch.global.L2 [%0];" :: "l"(b + o));
}

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

// nv (1 or 2) tables in one pass: items [0, 4 groups) build table 0, [4 groups, 8 groups) table 1
// (4 groups is a multiple of 4, so no 4-lane shuffle group straddles the two)
__device__ void build_tables(int nv, int groups, const float* v0, uint32_t* tbl0, float* xs0, float* cs0,
                             const float* v1, uint32_t* tbl1, float* xs1, float* cs1, bool from_global = false) {
    // one thread per (group j, thread column t): both parts of its 16 elements, then the group's
    // sums over the 4 columns (adjacent lanes). Items past the last table read row 0 of table 0.
    for (int i2 = threadIdx.x; i2 < ((nv * groups * 4 + 31) & ~31); i2 += blockDim.x) {
        const bool on = i2 < nv * groups * 4;
        const bool second = on && i2 >= groups * 4;
        const int i = second ? i2 - groups * 4 : i2;
        const float* v = second ? v1 : v0;
        uint32_t* tbl = second ? tbl1 : tbl0;
        float* xs = second ? xs1 : xs0;
        float* cs = second ? cs1 : cs0;
        const int j = on ? i >> 2 : 0, t = i & 3;
        const float4* src = reinterpret_cast<const float4*>(v + j * 64 + t * 16);
        float x[16], hi[16], lo[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            // global sources were written by other CTAs in this launch: read them from L2
            const float4 f = from_global ? __ldcg(src + q) : src[q];
            x[4 * q] = f.x; x[4 * q + 1] = f.y; x[4 * q + 2] = f.z; x[4 * q + 3] = f.w;
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) split11((q & 1) ? x[q] * 0.0625f : x[q], hi[q], lo[q]);
        // pairs (x0,x4)(x1,x5)(x2,x6)(x3,x7) | (x8,x12)(x9,x13)(x10,x14)(x11,x15)
        const uint4 h0 = make_uint4(cvt2(hi[0], hi[4]), cvt2(hi[1], hi[5]), cvt2(hi[2], hi[6]), cvt2(hi[3], hi[7]));
        const uint4 h1 = make_uint4(cvt2(hi[8], hi[12]), cvt2(hi[9], hi[13]), cvt2(hi[10], hi[14]), cvt2(hi[11], hi[15]));
        const uint4 l0 = make_uint4(cvt2(lo[0], lo[4]), cvt2(lo[1], lo[5]), cvt2(lo[2], lo[6]), cvt2(lo[3], lo[7]));
        const uint4 l1 = make_uint4(cvt2(lo[8], lo[12]), cvt2(lo[9], lo[13]), cvt2(lo[10], lo[14]), cvt2(lo[11], lo[15]));
        float sx = 0.0f, c = 0.0f;
        if (on) {
            *reinterpret_cast<uint4*>(tbl + ((j * 2 + 0) * 8 + t * 2 + 0) * 4) = h0;
            *reinterpret_cast<uint4*>(tbl + ((j * 2 + 1) * 8 + t * 2 + 0) * 4) = h1;
            *reinterpret_cast<uint4*>(tbl + ((j * 2 + 0) * 8 + t * 2 + 1) * 4) = l0;
            *reinterpret_cast<uint4*>(tbl + ((j * 2 + 1) * 8 + t * 2 + 1) * 4) = l1;
            // what the MMA adds besides n*x: 1024 * (hi + lo) as the fp16 operands hold them
            const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
            const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float2 fh = __half22float2(*reinterpret_cast<const __half2*>(&hw[q]));
                const float2 fl = __half22float2(*reinterpret_cast<const __half2*>(&lw[q]));
                c += 1024.0f * ((fh.x + fl.x) + (fh.y + fl.y));
            }
#pragma unroll
            for (int q = 0; q < 16; ++q) sx += x[q];
        }
        sx += __shfl_xor_sync(0xffffffffu, sx, 1);
        sx += __shfl_xor_sync(0xffffffffu, sx, 2);
        c += __shfl_xor_sync(0xffffffffu, c, 1);
        c += __shfl_xor_sync(0xffffffffu, c, 2);
        if (on && t == 0) { xs[j] = sx; cs[j] = c; }
    }
}

__device__ void build_table(const float* v, int groups, uint32_t* tbl, float* xs, float* cs) {
    build_tables(1, groups, v, tbl, xs, cs, v, tbl, xs, cs);
}

// One warp: groups [j0, j1) of a 16-row tile. Rows g (pointer set a) and g + 8 (set b); lane
// (g, t = 0) accumulates y_a (row g) and y_b (row g + 8).
struct TileRows {
    const uint8_t* wa;     // row g, byte 0 of group 0
    const uint8_t* wb;     // row g + 8
    const uint16_t* sa;    // scales of row g
    const uint16_t* ba;
    const uint16_t* sb;
    const uint16_t* bb;
};

// Groups are taken four at a time: group q0 + m puts its activation in B columns 2m (fp16 high
// part) and 2m + 1 (low part), so after the quad lane (g, t) holds group q0 + t's products for
// rows g and g + 8 and applies that group's scale, bias and offset constant. The per-lane sums
// cover the groups congruent to t mod 4; the caller adds the four lanes of a row.
// Global loads of one quad: the 4 groups' weight words for rows g and g + 8 (always from a valid
// group of the run) and this lane's group's scales and biases.
struct QuadLoads {
    uint2 wa[4], wb[4];
    uint16_t sa, ba, sb, bb;
};

__device__ __forceinline__ QuadLoads load_quad(const TileRows& R, int q0, int j0, int j1, int t) {
    QuadLoads Q;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int j = q0 + m;
        const int jc = (j >= j0 && j < j1) ? j : j0;
        Q.wa[m] = ldg_nc_u2(R.wa + 32 * jc + 8 * t);
        Q.wb[m] = ldg_nc_u2(R.wb + 32 * jc + 8 * t);
    }
    const int j = q0 + t;
    const int jc = (j >= j0 && j < j1) ? j : j0;
    Q.sa = ldg_nc_u16(R.sa + jc);
    Q.ba = ldg_nc_u16(R.ba + jc);
    Q.sb = ldg_nc_u16(R.sb + jc);
    Q.bb = ldg_nc_u16(R.bb + jc);
    return Q;
}

__device__ __forceinline__ void compute_quad(const QuadLoads& Q, int q0, int j0, int j1, const uint32_t* tbl,
                                             const float* xs, const float* cs, float& ya, float& yb) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int slotn = t * 2 + (g & 1);
    float dE[4] = {0.0f, 0.0f, 0.0f, 0.0f}, dO[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int j = q0 + m;
        const bool on = j >= j0 && j < j1;           // warp-uniform
        uint4 b0 = make_uint4(0u, 0u, 0u, 0u), b1 = make_uint4(0u, 0u, 0u, 0u);
        if (on && (g >> 1) == m) {
            b0 = *reinterpret_cast<const uint4*>(tbl + ((j * 2 + 0) * 8 + slotn) * 4);
            b1 = *reinterpret_cast<const uint4*>(tbl + ((j * 2 + 1) * 8 + slotn) * 4);
        }
        uint32_t qa0[4], qa1[4], qb0[4], qb1[4];
        dq_word(Q.wa[m].x, qa0);
        dq_word(Q.wa[m].y, qa1);
        dq_word(Q.wb[m].x, qb0);
        dq_word(Q.wb[m].y, qb1);
        float (&d)[4] = (m & 1) ? dO : dE;
        mma16816(d, qa0[0], qb0[0], qa0[1], qb0[1], b0.x, b0.y);
        mma16816(d, qa0[2], qb0[2], qa0[3], qb0[3], b0.z, b0.w);
        mma16816(d, qa1[0], qb1[0], qa1[1], qb1[1], b1.x, b1.y);
        mma16816(d, qa1[2], qb1[2], qa1[3], qb1[3], b1.z, b1.w);
    }
    const int j = q0 + t;
    if (j >= j0 && j < j1) {
        const float x = xs[j], c = cs[j];
        ya = fmaf(bf16f(Q.ba), x, fmaf(bf16f(Q.sa), ((dE[0] + dO[0]) + (dE[1] + dO[1])) - c, ya));
        yb = fmaf(bf16f(Q.bb), x, fmaf(bf16f(Q.sb), ((dE[2] + dO[2]) + (dE[3] + dO[3])) - c, yb));
    }
}

// Loads of the next quad are issued before the current one is computed, so each warp keeps two
// quads (4 KB of weights) in flight.
__device__ __forceinline__ void gemv_groups(const TileRows& R, int j0, int j1, const uint32_t* tbl, const float* xs,
                                            const float* cs, float& ya, float& yb) {
    const int t = threadIdx.x & 3;
    int q0 = j0 & ~3;
    QuadLoads cur = load_quad(R, q0, j0, j1, t);
    for (; q0 < j1; q0 += 4) {
        QuadLoads nxt = cur;
        if (q0 + 4 < j1) nxt = load_quad(R, q0 + 4, j0, j1, t);
        compute_quad(cur, q0, j0, j1, tbl, xs, cs, ya, yb);
        cur = nxt;
    }
}

// Splits n_items x L groups evenly over the CTA's warps; each warp walks its contiguous run of
// (item, group) pairs and leaves one partial per item it touched in s.slot[item][warp].
template <class RowsFn>
__device__ __forceinline__ void warp_items(Smem& s, int slot_base, int n_items, int L, int jbase, const uint32_t* tbl,
                                           const float* xs, const float* cs, RowsFn rows_of) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int total = n_items * L;
    int p = warp * total / NW;
    const int p1 = (warp + 1) * total / NW;
    while (p < p1) {
        const int item = p / L, j0 = p - item * L;
        const int j1 = min(L, j0 + (p1 - p));
        const TileRows R = rows_of(item);
        float ya = 0.0f, yb = 0.0f;
        gemv_groups(R, jbase + j0, jbase + j1, tbl, xs, cs, ya, yb);
        ya += __shfl_xor_sync(0xffffffffu, ya, 1);
        ya += __shfl_xor_sync(0xffffffffu, ya, 2);
        yb += __shfl_xor_sync(0xffffffffu, yb, 1);
        yb += __shfl_xor_sync(0xffffffffu, yb, 2);
        if (t == 0) {
            s.slot[slot_base + item][warp][g] = ya;
            s.slot[slot_base + item][warp][8 + g] = yb;
        }
        p += j1 - j0;
    }
}

// As warp_items, with each item's own table and K-group base (the down phase mixes segments).
struct ItemSrc {
    TileRows R;
    const uint32_t* tbl;
    const float* xs;
    const float* cs;
    int jbase;
};
template <class SrcFn>
__device__ __forceinline__ void warp_items_src(Smem& s, int n_items, int L, SrcFn src_of) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int total = n_items * L;
    int p = warp * total / NW;
    const int p1 = (warp + 1) * total / NW;
    while (p < p1) {
        const int item = p / L, j0 = p - item * L;
        const int j1 = min(L, j0 + (p1 - p));
        const ItemSrc S = src_of(item);
        float ya = 0.0f, yb = 0.0f;
        gemv_groups(S.R, S.jbase + j0, S.jbase + j1, S.tbl, S.xs, S.cs, ya, yb);
        ya += __shfl_xor_sync(0xffffffffu, ya, 1);
        ya += __shfl_xor_sync(0xffffffffu, ya, 2);
        yb += __shfl_xor_sync(0xffffffffu, yb, 1);
        yb += __shfl_xor_sync(0xffffffffu, yb, 2);
        if (t == 0) {
            s.slot[item][warp][g] = ya;
            s.slot[item][warp][8 + g] = yb;
        }
        p += j1 - j0;
    }
}

__device__ __forceinline__ void zero_slots(Smem& s, int n_items) {
    float* f = &s.slot[0][0][0];
    for (int i = threadIdx.x; i < n_items * NW * 16; i += blockDim.x) f[i] = 0.0f;
}

__device__ __forceinline__ float slot_sum(const Smem& s, int item, int r) {
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) v += s.slot[item][w][r];
    return v;
}

__device__ __forceinline__ float gelu_tanh_f(float x) {
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

// ---- barriers ------------------------------------------------------------------------------
__device__ __forceinline__ void arrive(const Params& P, int kind, unsigned value) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        st_release(P.flags + kind * 256 + blockIdx.x, value);
    }
}

__device__ bool wait_all(const Params& P, Smem& s, int kind, unsigned value) {
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const unsigned* f = P.flags + kind * 256;
        const uint64_t t0 = globaltimer_ns();
        bool ok = true;
        for (;;) {
            bool mine = true;
            for (unsigned b = lane; b < gridDim.x; b += 32) mine &= (ld_relaxed(f + b) >= value);
            const int e = lane == 0 ? ld_volatile_int(P.err) : 0;
            if (__all_sync(0xffffffffu, mine)) break;
            if (__shfl_sync(0xffffffffu, e, 0) != 0) { ok = false; break; }
            if (globaltimer_ns() - t0 > P.wait_limit_ns) {
                if (lane == 0) { atomicExch(P.err, 1); atomicExch(P.sticky, 1); }
                ok = false;
                break;
            }
        }
        __threadfence();
        if (lane == 0) s.flag = ok ? 0 : 1;
    }
    __syncthreads();
    return s.flag == 0;
}

// ---- P1 pieces ----------------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(sa), "l"(gmem) : "memory");
}

// Starts copying norm vectors into s.nw: the pre-FFN set (pre_ffn_norm, pre_ffn_norm_2,
// router.scale) of layer Lpre into slots 0..2 and the post-FFN set (post_ffn_norm_1, _2, and
// post_ffn_norm) of layer Lpost into slots 3..5; either may be null. Completed by
// tail_and_views.
__device__ void load_norms_async(Smem& s, const GtmLayer* Lpre, const GtmLayer* Lpost) {
    constexpr int per = D * 2 / 16;   // 16-byte chunks per vector
    for (int i = threadIdx.x; i < 6 * per; i += NT) {
        const int v = i / per, c = i - v * per;
        const GtmLayer* L = v < 3 ? Lpre : Lpost;
        if (!L) continue;
        const uint64_t off = v == 0 ? L->pre_ffn_norm : v == 1 ? L->pre_ffn_norm_2 : v == 2 ? L->router_scale
                           : v == 3 ? L->post_ffn_norm_1 : v == 4 ? L->post_ffn_norm_2 : L->post_ffn_norm;
        cp_async16(&s.nw[v][c * 8], rp(L->resident_dev, off) + c * 16);
    }
    if (Lpre && threadIdx.x < NE * 2 / 16)
        cp_async16(&s.pes[threadIdx.x * 8], rp(Lpre->resident_dev, Lpre->per_expert_scale) + threadIdx.x * 16);
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// Sums a and b over the block with one barrier: each thread adds the warp partials itself in
// warp order, so every thread (and every CTA, given the same data) gets the same bits.
// Consecutive calls must alternate `buf`.
__device__ __forceinline__ double2 block_sum2(Smem& s, double a, double b, int buf) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    if (lane == 0) { s.red2[buf][warp][0] = a; s.red2[buf][warp][1] = b; }
    __syncthreads();
    double ra = 0.0, rb = 0.0;
#pragma unroll
    for (int w = 0; w < NW; ++w) { ra += s.red2[buf][w][0]; rb += s.red2[buf][w][1]; }
    return make_double2(ra, rb);
}

// 1 / sqrt(float(sum / D) + eps), the reference's formula (src/cpu_reference.cpp:46); the mean
// is formed with a multiply by 1/D (one extra rounding, far below the float conversion).
constexpr double kInvD = 1.0 / (double)D;
__device__ __forceinline__ float rms_inv_from_sum(double sum, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(__dmul_rn(sum, kInvD)), eps)));
}

// The same with the reference's exact bits when `sum` is a parallel double sum of x*x: see
// exact_rms_inv for the argument; the bound (D + 48) ulps also covers the tree depth (< 30) and
// the multiply by the rounded 1/D. The check is identical on every thread, so the rare fallback
// (a sequential sum by thread 0, then the reference's division) is a uniform branch.
__device__ float certified_rms_inv(Smem& s, const float* x, double sum, float eps) {
    const double q = __dmul_rn(sum, kInvD);
    float f = __double2float_rn(q);
    const double fd = (double)f;
    const double lo = (fd + (double)nextafterf(f, -INFINITY)) * 0.5;
    const double hi = (fd + (double)nextafterf(f, INFINITY)) * 0.5;
    const double bound = q * ((double)D + 48.0) * 1.1102230246251565e-16;
    if (!(q - lo > bound && hi - q > bound)) {
        if (threadIdx.x == 0) {
            double seq = 0.0;
            for (int i = 0; i < D; ++i) seq = __dadd_rn(seq, __dmul_rn((double)x[i], (double)x[i]));
            s.red[32] = seq;
        }
        __syncthreads();
        f = __double2float_rn(__ddiv_rn(s.red[32], (double)D));
    }
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(f, eps)));
}

// Layer tail of the previous layer Lp (src/cpu_reference.cpp:512-520), when there is one, from
// the down partials (shared output = the 3 shared thirds, h2 = the 8 routed experts in router
// order), the optional weightless RMSNorm between layers, then the views of layer L
// (src/cpu_reference.cpp:425-443): dense_x = h*w_pre, routed_x = h*w_pre2 and
// router_in = h*bf16(router.scale)*(1/sqrt(D)) with h = rmsnorm_no_scale(hidden), exactly as the
// reference rounds them; finally the fragment tables of dense_x and routed_x.
__device__ void tail_and_views(Smem& s, const Params& P, const GtmLayer* Lp, bool norm_between, bool do_views,
                               float* h1_out, float* h2_out, float* hid_out) {
    const int tid = threadIdx.x;
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    float* h2 = s.ab;
    float* sh = s.ab + D;
    double a = 0.0;
    int buf = 0;
    if (Lp) {
        const float ls = bf16f(*rp16(Lp->resident_dev, Lp->layer_scalar));
        double b = 0.0;
        for (int i = tid; i < D / 4; i += NT) {
            // part [contributor][shared, routed][D]: shared = p00 + p10, routed h2 = p01 + p11
            const float4* pp = reinterpret_cast<const float4*>(P.part) + i;
            float4 vs = __ldcg(pp), vh = __ldcg(pp + (D / 4));
            const float4 s1 = __ldcg(pp + 2 * (D / 4)), r1 = __ldcg(pp + 3 * (D / 4));
            vs.x += s1.x; vs.y += s1.y; vs.z += s1.z; vs.w += s1.w;
            vh.x += r1.x; vh.y += r1.y; vh.z += r1.z; vh.w += r1.w;
            reinterpret_cast<float4*>(sh)[i] = vs;
            reinterpret_cast<float4*>(h2)[i] = vh;
            a += (double)vs.x * vs.x + (double)vs.y * vs.y + (double)vs.z * vs.z + (double)vs.w * vs.w;
            b += (double)vh.x * vh.x + (double)vh.y * vh.y + (double)vh.z * vh.z + (double)vh.w * vh.w;
        }
        double2 r = block_sum2(s, a, b, buf); buf ^= 1;
        const float inv1 = rms_inv_from_sum(r.x, P.eps), inv2 = rms_inv_from_sum(r.y, P.eps);
        a = 0.0;
        for (int i = tid; i < D; i += NT) {
            const float h1 = __fmul_rn(__fmul_rn(sh[i], inv1), bf16f(s.nw[3][i]));
            if (h1_out) h1_out[i] = h1;
            if (h2_out) h2_out[i] = h2[i];
            const float t = __fadd_rn(__fmul_rn(__fmul_rn(h2[i], inv2), bf16f(s.nw[4][i])), h1);
            h2[i] = t;
            a += (double)t * t;
        }
        r = block_sum2(s, a, 0.0, buf); buf ^= 1;
        const float inv3 = rms_inv_from_sum(r.x, P.eps);
        a = 0.0;
        for (int i = tid; i < D; i += NT) {
            const float hv = __fmul_rn(__fadd_rn(s.hid[i], __fmul_rn(__fmul_rn(h2[i], inv3), bf16f(s.nw[5][i]))), ls);
            s.hid[i] = hv;
            a += (double)hv * hv;
        }
        if (norm_between) {
            r = block_sum2(s, a, 0.0, buf); buf ^= 1;
            const float inv4 = rms_inv_from_sum(r.x, P.eps);
            a = 0.0;
            for (int i = tid; i < D; i += NT) {
                const float hv = __fmul_rn(s.hid[i], inv4);
                s.hid[i] = hv;
                a += (double)hv * hv;
            }
        }
        if (hid_out)
            for (int i = tid; i < D; i += NT) hid_out[i] = s.hid[i];
    } else {
        for (int i = tid; i < D; i += NT) a += (double)s.hid[i] * s.hid[i];
    }
    if (!do_views) {
        __syncthreads();
        return;
    }
    const double2 r = block_sum2(s, a, 0.0, buf);
    const float inv = certified_rms_inv(s, s.hid, r.x, P.eps);
    for (int i = tid; i < D; i += NT) {
        const float h = __fmul_rn(s.hid[i], inv);
        sh[i] = __fmul_rn(h, bf16f(s.nw[0][i]));    // dense_x
        h2[i] = __fmul_rn(h, bf16f(s.nw[1][i]));    // routed_x
        s.rin[(i >> 6) * RIN_PITCH + (i & 63)] = __fmul_rn(__fmul_rn(h, bf16f(s.nw[2][i])), P.inv_sqrt_d);
    }
    __syncthreads();
    build_tables(2, GD, h2, s.tbl_r, s.xs_r, s.cs_r, sh, s.tbl_d, s.xs_d, s.cs_d);
    __syncthreads();
}

// One router logit in src/cpu_reference.cpp:86-106's order (bit-identical).
__device__ float router_row(Smem& s, const GtmLayer& L, int row) {
    const int tid = threadIdx.x;
    const uint8_t* W = rp(L.resident_dev, L.router.weight) + (size_t)row * D;
    const uint16_t* S = rp16(L.resident_dev, L.router.scales) + row * GD;
    const uint16_t* B = rp16(L.resident_dev, L.router.biases) + row * GD;
    if (tid < GD) {
        const uint4* wg = reinterpret_cast<const uint4*>(W + tid * kGroup);
        uint4 q[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] = ldg_stream_u4(wg + i);
        const float sc = bf16f(ldg_u16(S + tid)), bi = bf16f(ldg_u16(B + tid));
        const float* x = s.rin + tid * RIN_PITCH;
        float dot = 0.0f, sum = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t wv[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const float xv = x[i * 16 + c * 4 + b];
                    dot = __fadd_rn(dot, __fmul_rn((float)((wv[c] >> (8 * b)) & 0xFFu), xv));
                    sum = __fadd_rn(sum, xv);
                }
            }
        }
        s.terms[tid] = __fadd_rn(__fmul_rn(sc, dot), __fmul_rn(bi, sum));
    }
    __syncthreads();
    float acc = 0.0f;
    if (tid == 0)
        for (int g = 0; g < GD; ++g) acc = __fadd_rn(acc, s.terms[g]);
    return acc;
}

// Top-8 of the 128 logits by (value desc, index asc), softmax over the 8, times
// per_expert_scale (src/cpu_reference.cpp:447-480). Warp 0; results in s.topi / s.topw.
__device__ void select_topk(Smem& s, const GtmLayer& L, const float* logits, bool writer, uint32_t* idx_out,
                            float* w_out, float* logits_out) {
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    float v[4];
    bool taken[4] = {false, false, false, false};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        v[j] = __ldcg(logits + lane + 32 * j);
        if (writer && logits_out) logits_out[lane + 32 * j] = v[j];
    }
    // Order-preserving unsigned keys (-0 folded onto +0, which compare equal as floats); each
    // round takes the largest key, then the lowest index holding it: (value desc, index asc).
    uint32_t key[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t u = __float_as_uint(v[j] == 0.0f ? 0.0f : v[j]);
        key[j] = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    }
    float my_sel = 0.0f;
    int my_idx = 0;
    float top0 = 0.0f;
#pragma unroll
    for (int k = 0; k < TOPK; ++k) {
        uint32_t ck = 0u, ci = 0xFFFFFFFFu;          // this lane's best untaken (key desc, index asc)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (!taken[j] && (ci == 0xFFFFFFFFu || key[j] > ck)) { ck = key[j]; ci = (uint32_t)(lane + 32 * j); }
        const uint32_t mk = __reduce_max_sync(0xffffffffu, ck);
        const uint32_t bi = __reduce_min_sync(0xffffffffu, ck == mk ? ci : 0xFFFFFFFFu);
        const float bv = __uint_as_float((mk & 0x80000000u) ? (mk & 0x7FFFFFFFu) : ~mk);
        if (k == 0) top0 = bv;
        if (lane == k) { my_sel = bv; my_idx = (int)bi; }
#pragma unroll
        for (int j = 0; j < 4; ++j) if ((uint32_t)(lane + 32 * j) == bi) taken[j] = true;
    }
    // lanes 0..7: exp and per-expert scale in parallel, the sum in order on every lane
    const float e = lane < TOPK ? expf(__fsub_rn(my_sel, top0)) : 0.0f;
    const uint16_t pes_bits = lane < TOPK ? s.pes[my_idx] : 0;
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < TOPK; ++k) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, e, k));
    if (lane < TOPK) {
        const float w = __fmul_rn(__fdiv_rn(e, sum), bf16f(pes_bits));
        s.topi[lane] = my_idx;
        s.topw[lane] = w;
        if (writer && idx_out) idx_out[lane] = (uint32_t)my_idx;
        if (writer && w_out) w_out[lane] = w;
    }
}

// ---- work lists ----------------------------------------------------------------------------------
__device__ __forceinline__ int share(int n, int c, int G) { return (int)((long long)c * n / G); }

// gate/up tile rows: row g = gate row r0 + g, row g + 8 = up row r0 + g (same x)
__device__ __forceinline__ TileRows gu_rows(const uint8_t* base_g, const uint8_t* base_u, const GtmQuant& qg,
                                            const GtmQuant& qu, int r) {
    TileRows R;
    R.wa = base_g + qg.weight + (uint64_t)r * ROW_GU;
    R.wb = base_u + qu.weight + (uint64_t)r * ROW_GU;
    R.sa = reinterpret_cast<const uint16_t*>(base_g + qg.scales) + (uint64_t)r * GD;
    R.ba = reinterpret_cast<const uint16_t*>(base_g + qg.biases) + (uint64_t)r * GD;
    R.sb = reinterpret_cast<const uint16_t*>(base_u + qu.scales) + (uint64_t)r * GD;
    R.bb = reinterpret_cast<const uint16_t*>(base_u + qu.biases) + (uint64_t)r * GD;
    return R;
}

__device__ __forceinline__ TileRows down_rows(const uint8_t* base, const GtmQuant& q, int row, uint32_t row_bytes,
                                              uint32_t groups) {
    TileRows R;
    R.wa = base + q.weight + (uint64_t)row * row_bytes;
    R.wb = base + q.weight + (uint64_t)(row + 8) * row_bytes;
    R.sa = reinterpret_cast<const uint16_t*>(base + q.scales) + (uint64_t)row * groups;
    R.ba = reinterpret_cast<const uint16_t*>(base + q.biases) + (uint64_t)row * groups;
    R.sb = reinterpret_cast<const uint16_t*>(base + q.scales) + (uint64_t)(row + 8) * groups;
    R.bb = reinterpret_cast<const uint16_t*>(base + q.biases) + (uint64_t)(row + 8) * groups;
    return R;
}

// Shared gate/up tiles [t0, t1) -> act[8*T + r]
__device__ void shared_gate_up(Smem& s, const Params& P, const GtmLayer& L, int t0, int t1) {
    const int n = t1 - t0;
    if (n <= 0) return;
    zero_slots(s, n);
    __syncthreads();
    const uint8_t* base = static_cast<const uint8_t*>(L.resident_dev);
    const int lane_g = (threadIdx.x & 31) >> 2;
    warp_items(s, 0, n, GD, 0, s.tbl_d, s.xs_d, s.cs_d, [&](int item) {
        return gu_rows(base, base, L.shared_gate, L.shared_up, (t0 + item) * 8 + lane_g);
    });
    __syncthreads();
    for (int i = threadIdx.x; i < n * 8; i += NT) {
        const int item = i >> 3, r = i & 7;
        const float gt = slot_sum(s, item, r), up = slot_sum(s, item, 8 + r);
        P.act[(t0 + item) * 8 + r] = gelu_tanh_f(gt) * up;
    }
}

// Routed gate/up tiles [t0, t1) (tile T: expert slot T / 88, rows 8 * (T % 88) ..) -> act[FS + 8*T + r]
__device__ void routed_gate_up(Smem& s, const Params& P, const GtmLayer& L, int t0, int t1) {
    const int n = t1 - t0;
    if (n <= 0) return;
    zero_slots(s, n);
    __syncthreads();
    const int lane_g = (threadIdx.x & 31) >> 2;
    warp_items(s, 0, n, GD, 0, s.tbl_r, s.xs_r, s.cs_r, [&](int item) {
        const int T = t0 + item, k = T / (FE / 8), r = (T - k * (FE / 8)) * 8 + lane_g;
        const uint8_t* blk = rp(L.experts_dev, (uint64_t)s.topi[k] * L.expert_stride);
        return gu_rows(blk, blk, L.expert_gate, L.expert_up, r);
    });
    __syncthreads();
    for (int i = threadIdx.x; i < n * 8; i += NT) {
        const int item = i >> 3, r = i & 7;
        const float gt = slot_sum(s, item, r), up = slot_sum(s, item, 8 + r);
        P.act[FS + (t0 + item) * 8 + r] = gelu_tanh_f(gt) * up;
    }
}

// Down items [i0, i1) of the shared expert and the 8 routed experts, one pass, in row-tile-major
// order: item i -> row tile ot = i / NSEG, segment q = i % NSEG. Segments 0..2: K groups
// [11q, 11q + 11) of the shared down rows (33 groups); segments 3..10: expert slot k = q - 3, all 11
// groups of its down rows, times w_k. The table of segment q is tbl_dn + 11 q. The CTA sums its
// segments of each row tile in segment order, shared and routed apart, into contributor slot 0
// (the CTA holding segment 0 of the tile) or 1: a CTA holds >= 13 consecutive items, so a tile of
// 11 has at most two contributors, and the tail reads part[0] + part[1] (4 vectors, not 11).
__device__ void down_items(Smem& s, const Params& P, const GtmLayer& L, int i0, int i1) {
    const int n = i1 - i0;
    if (n <= 0) return;
    zero_slots(s, n);
    __syncthreads();
    const uint8_t* res = static_cast<const uint8_t*>(L.resident_dev);
    const int lane_g = (threadIdx.x & 31) >> 2;
    warp_items_src(s, n, GFE, [&](int item) {
        const int it = i0 + item, ot = it / NSEG, q = it - ot * NSEG;
        ItemSrc S;
        if (q < 3) {
            S.R = down_rows(res, L.shared_down, ot * 16 + lane_g, FS / 2, GFS);
            S.tbl = s.tbl_dn;
            S.xs = s.xs_dn;
            S.cs = s.cs_dn;
            S.jbase = q * GFE;
        } else {
            const uint8_t* blk = rp(L.experts_dev, (uint64_t)s.topi[q - 3] * L.expert_stride);
            S.R = down_rows(blk, L.expert_down, ot * 16 + lane_g, FE / 2, GFE);
            S.tbl = s.tbl_dn + q * GFE * TBL_WORDS;
            S.xs = s.xs_dn + q * GFE;
            S.cs = s.cs_dn + q * GFE;
            S.jbase = 0;
        }
        return S;
    });
    __syncthreads();
    const int ot0 = i0 / NSEG, ot1 = (i1 - 1) / NSEG;
    for (int i = threadIdx.x; i < (ot1 - ot0 + 1) * 16; i += NT) {
        const int ot = ot0 + (i >> 4), r = i & 15;
        const int a = max(i0, ot * NSEG), b = min(i1, ot * NSEG + NSEG);
        float sh = 0.0f, h2 = 0.0f;
        for (int it = a; it < b; ++it) {
            const int q = it - ot * NSEG;
            const float v = slot_sum(s, it - i0, r);
            if (q < 3) sh = __fadd_rn(sh, v);
            else h2 = __fadd_rn(h2, __fmul_rn(s.topw[q - 3], v));   // the product rounded, as the combine had it
        }
        const int c = a == ot * NSEG ? 0 : 1;
        float* pc = P.part + (size_t)c * 2 * D + ot * 16 + r;
        pc[0] = sh;
        pc[D] = h2;
        if (c == 0 && b == ot * NSEG + NSEG) {   // the whole tile here: no second contributor
            pc[2 * D] = 0.0f;
            pc[3 * D] = 0.0f;
        }
    }
}

// L2 prefetch of the weights this CTA reads in the next layer's P1 (router row, shared gate/up
// tiles, norm vectors) and of its shared-down rows.
// Every range below lies inside one tensor; the CTA's warps take the ranges round-robin.
__device__ void prefetch_layer_static(const GtmLayer& L, int cta, int G) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint8_t* base = static_cast<const uint8_t*>(L.resident_dev);
    const int nrow = cta < NE ? (NE - 1 - cta) / G + 1 : 0;          // router rows of this CTA
    const int t0 = share(TILES_S, cta, G), t1 = share(TILES_S, cta + 1, G);
    const int i0 = share(ITEMS_DN, cta, G), i1 = share(ITEMS_DN, cta + 1, G);   // this CTA's down items
    const int n_router = 3 * nrow, n_sgu = t1 > t0 ? 6 : 0, n_sd = 18 * (i1 - i0), n_vec = 6;
    const int total = n_router + n_sgu + n_sd + n_vec;
    for (int i = warp; i < total; i += NW) {
        const uint8_t* p;
        uint32_t n;
        if (i < n_router) {
            const uint64_t row = (uint64_t)(cta + (i / 3) * G);
            const int part = i % 3;
            if (part == 0) { p = base + L.router.weight + row * D; n = D; }
            else { p = base + (part == 1 ? L.router.scales : L.router.biases) + row * GD * 2; n = GD * 2; }
        } else if (i < n_router + n_sgu) {
            const int k = i - n_router, m = k / 3, part = k % 3;
            const GtmQuant& q = m ? L.shared_up : L.shared_gate;
            if (part == 0) { p = base + q.weight + (uint64_t)t0 * 8 * ROW_GU; n = (t1 - t0) * 8 * ROW_GU; }
            else { p = base + (part == 1 ? q.scales : q.biases) + (uint64_t)t0 * 8 * GD * 2; n = (t1 - t0) * 8 * GD * 2; }
        } else if (i < n_router + n_sgu + n_sd) {
            // the shared-down items among them (segments 0..2); routed ones prefetch after the top-8
            const int k = i - n_router - n_sgu, it = i0 + k / 18, part = k % 18;
            const int ot = it / NSEG, q = it - ot * NSEG;
            if (q >= 3) continue;
            if (part < 16) {
                p = base + L.shared_down.weight + ((uint64_t)ot * 16 + part) * (FS / 2) + q * GFE * 32;
                n = GFE * 32;
            } else {
                p = base + (part == 16 ? L.shared_down.scales : L.shared_down.biases) + (uint64_t)ot * 16 * GFS * 2;
                n = 16 * GFS * 2;
            }
        } else {
            const int v = i - n_router - n_sgu - n_sd;
            const uint64_t off = v == 0 ? L.pre_ffn_norm : v == 1 ? L.pre_ffn_norm_2 : v == 2 ? L.router_scale
                               : v == 3 ? L.post_ffn_norm_1 : v == 4 ? L.post_ffn_norm_2 : L.post_ffn_norm;
            p = base + off;
            n = D * 2;
        }
        prefetch_lines(p, n, lane);
    }
}

// L2 prefetch of this CTA's routed gate/up rows (known once the top-8 is): per tile 8 gate rows,
// 8 up rows and their scales and biases, each a contiguous range.
__device__ void prefetch_routed_gate_up(const Smem& s, const GtmLayer& L, int cta, int G) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = share(TILES_R, cta, G), t1 = share(TILES_R, cta + 1, G);
    for (int i = warp; i < 6 * (t1 - t0); i += NW) {
        const int T = t0 + i / 6, part = i % 6, k = T / (FE / 8), r8 = T - k * (FE / 8);
        const uint8_t* blk = rp(L.experts_dev, (uint64_t)s.topi[k] * L.expert_stride);
        const GtmQuant& q = part < 3 ? L.expert_gate : L.expert_up;
        const int pp = part % 3;
        if (pp == 0) prefetch_lines(blk + q.weight + (uint64_t)r8 * 8 * ROW_GU, 8 * ROW_GU, lane);
        else prefetch_lines(blk + (pp == 1 ? q.scales : q.biases) + (uint64_t)r8 * 8 * GD * 2, 8 * GD * 2, lane);
    }
}

// L2 prefetch of this CTA's routed-down rows (known once the top-8 is).
__device__ void prefetch_routed_down(const Smem& s, const GtmLayer& L, int cta, int G) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i0 = share(ITEMS_DN, cta, G), i1 = share(ITEMS_DN, cta + 1, G);
    for (int i = warp; i < 3 * (i1 - i0); i += NW) {
        const int it = i0 + i / 3, part = i % 3, ot = it / NSEG, q = it - ot * NSEG;
        if (q < 3) continue;   // shared-down items were prefetched with the layer's static weights
        const uint8_t* blk = rp(L.experts_dev, (uint64_t)s.topi[q - 3] * L.expert_stride);
        if (part == 0) prefetch_lines(blk + L.expert_down.weight + (uint64_t)ot * 16 * (FE / 2), 16 * (FE / 2), lane);
        else prefetch_lines(blk + (part == 1 ? L.expert_down.scales : L.expert_down.biases) + (uint64_t)ot * 16 * GFE * 2,
                            16 * GFE * 2, lane);
    }
}

__global__ void __launch_bounds__(NT, 1) moe_decode_kernel(const __grid_constant__ Params P) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_raw);
    const int tid = threadIdx.x;
    const int G = gridDim.x, cta = blockIdx.x;
    const GtmDecodeIO& io = P.io;
    const bool writer = cta == 0;

    prefetch_layer_static(P.layers[0], cta, G);
    load_norms_async(s, &P.layers[0], nullptr);
    for (int i = tid; i < D; i += NT) s.hid[i] = io.hidden_in_dev[i];
    __syncthreads();

    for (int l = 0; l < P.num_layers; ++l) {
        const GtmLayer& L = P.layers[l];
        const unsigned ep = (unsigned)(l + 1);
        // ---- P1 ----
        if (l > 0) {
            if (!wait_all(P, s, BAR_C, ep - 1)) return;
            tail_and_views(s, P, &P.layers[l - 1], (io.flags & GTM_DECODE_NORM_BETWEEN_LAYERS) != 0, true,
                           writer && io.h1_dev ? io.h1_dev + (size_t)(l - 1) * D : nullptr,
                           writer && io.h2_dev ? io.h2_dev + (size_t)(l - 1) * D : nullptr,
                           writer && io.hidden_layers_dev ? io.hidden_layers_dev + (size_t)(l - 1) * D : nullptr);
        } else {
            tail_and_views(s, P, nullptr, false, true, nullptr, nullptr, nullptr);
        }
        for (int row = cta; row < NE; row += G) {
            float lg = router_row(s, L, row);
            if (tid == 0) {
                if (io.logit_bias_dev) lg = __fadd_rn(lg, io.logit_bias_dev[(size_t)l * NE + row]);
                P.logits[row] = lg;
            }
            __syncthreads();
        }
        arrive(P, BAR_A1, ep);
        // (its shared activations are published by the B arrival below, which follows in order)
        shared_gate_up(s, P, L, share(TILES_S, cta, G), share(TILES_S, cta + 1, G));

        // ---- P2 ----
        if (!wait_all(P, s, BAR_A1, ep + (l == 0 ? P.first_wait_extra : 0u))) return;
        select_topk(s, L, P.logits, writer, io.topk_idx_dev ? io.topk_idx_dev + (size_t)l * TOPK : nullptr,
                    io.topk_w_dev ? io.topk_w_dev + (size_t)l * TOPK : nullptr,
                    io.logits_dev ? io.logits_dev + (size_t)l * NE : nullptr);
        __syncthreads();
        prefetch_routed_gate_up(s, L, cta, G);
        prefetch_routed_down(s, L, cta, G);
        routed_gate_up(s, P, L, share(TILES_R, cta, G), share(TILES_R, cta + 1, G));
        arrive(P, BAR_B, ep);

        // ---- P3: shared and routed down in one pass (every CTA's B arrival follows its shared
        //      gate/up, so B covers both activation sets) ----
        if (!wait_all(P, s, BAR_B, ep)) return;
        const int d0 = share(ITEMS_DN, cta, G), d1 = share(ITEMS_DN, cta + 1, G);
        if (d1 > d0) {
            // a CTA's >= 11 consecutive row-tile-major items read every segment: the tables of all
            // 11 (the shared activations, then the 8 routed slots), built straight from L2
            build_tables(1, NSEG * GFE, P.act, s.tbl_dn, s.xs_dn, s.cs_dn, P.act, s.tbl_dn, s.xs_dn, s.cs_dn, true);
        }
        __syncthreads();
        if (l + 1 < P.num_layers) prefetch_layer_static(P.layers[l + 1], cta, G);
        load_norms_async(s, l + 1 < P.num_layers ? &P.layers[l + 1] : nullptr, &L);
        down_items(s, P, L, d0, d1);
        arrive(P, BAR_C, ep);
    }

    // final tail by CTA 0
    if (!writer) return;
    const int l = P.num_layers;
    if (!wait_all(P, s, BAR_C, (unsigned)l)) return;
    tail_and_views(s, P, &P.layers[l - 1], false, false, io.h1_dev ? io.h1_dev + (size_t)(l - 1) * D : nullptr,
                   io.h2_dev ? io.h2_dev + (size_t)(l - 1) * D : nullptr,
                   io.hidden_layers_dev ? io.hidden_layers_dev + (size_t)(l - 1) * D : nullptr);
    for (int i = tid; i < D; i += NT) io.hidden_out_dev[i] = s.hid[i];
}

// ================================================================================================
// Tied LM head + greedy argmax (LMHeadGreedy.hlsl:1-73 + ArgmaxReduce.hlsl:1-62, runner.cpp:720-770)
//
// token = argmax_r logits[r], ties to the lower row, where logits = the int4 matvec of the normed
// hidden state in the CPU reference's exact operation order (cpu_reference.cpp:55-83; softcap is
// monotonic and skipped, as in the reference's greedy path). Computing every row in that order
// is issue-bound, so:
//   1. lm_approx: every row by the decode's mma.sync tiles (fp16 integer weights, fp16 high/low
//      activations, fp32 accumulation), HBM-bound, together with a rigorous bound E_r on the
//      distance between that value and the exact CPU-order value:
//        E_r = 2^-14 * sum_g (1100 |s_g| + 2 |b_g|) * sum_{k in g} |x_k|
//      (the MMA path's fp32 accumulation around its 1024 offset errs by < 64 * 2^-23 * 1039 |s| A_g
//      per group, the CPU order's own roundings by < (64 * 15 + 44 * 16) * 2^-24 (|s| + |b|) A_g,
//      and the x-sum orders differ by < 64 * 2^-24 A_g: E_r is 8x or more above each);
//   2. lm_exact: L = max_r (approx_r - E_r); only rows with approx_r + E_r >= L can hold the
//      maximum. Each of them is recomputed in the exact CPU order (one warp per row, a lane per
//      group, the groups summed in order by one lane) and folded into a 64-bit key (orderable
//      value, then the complement of the row) by atomicMax, which keeps (value desc, row asc)
//      independently of the order the rows arrive in;
//   3. lm_finish: the key -> token id and exact logit.
// Degenerate inputs (x = 0: every row ties) only make step 2 longer: every candidate is exact.
// ================================================================================================
constexpr int LM_THREADS = 256;   // 75 registers: three CTAs (24 warps) per SM

struct LmArgs {
    const uint8_t* w;        // [rows][D/2] packed int4, low nibble first
    const uint16_t* s;       // [rows][GD] bf16 scales
    const uint16_t* b;       // [rows][GD] bf16 biases
    const float* x;          // [D] normed hidden state
    int rows;
    float2* ae;              // [rows] (approximate logit, bound)
    float* cta_lb;           // [gridDim of lm_approx] max of approx - bound per CTA
    int n_lb;
    unsigned long long* key; // best (value, row)
    int* n_cand;             // rows recomputed exactly
    uint32_t* token;
    float* logit;            // exact logit of the token (nullable)
};

__device__ __forceinline__ uint32_t orderable(float v) {
    const uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float from_orderable(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__global__ void __launch_bounds__(LM_THREADS) lm_approx(const __grid_constant__ LmArgs A) {
    __shared__ __align__(16) float sx[D];
    __shared__ __align__(16) uint32_t tbl[GD * TBL_WORDS];
    __shared__ float xs[GD], cs[GD], xa[GD];
    __shared__ float wlb[LM_THREADS / 32];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    if (blockIdx.x == 0 && tid == 0) { *A.key = 0ull; *A.n_cand = 0; }
    for (int i = tid; i < D; i += blockDim.x) sx[i] = A.x[i];
    __syncthreads();
    build_table(sx, GD, tbl, xs, cs);
    for (int j = tid; j < GD; j += blockDim.x) {
        float a = 0.0f;
        for (int k = 0; k < kGroup; ++k) a += fabsf(sx[j * kGroup + k]);
        xa[j] = a;
    }
    __syncthreads();
    float lb = -INFINITY;
    const int ntiles = (A.rows + 15) / 16;
    for (int tile = blockIdx.x * (LM_THREADS / 32) + warp; tile < ntiles; tile += gridDim.x * (LM_THREADS / 32)) {
        const int ra = min(tile * 16 + g, A.rows - 1), rb = min(tile * 16 + 8 + g, A.rows - 1);
        TileRows R;
        R.wa = A.w + (size_t)ra * (D / 2);
        R.wb = A.w + (size_t)rb * (D / 2);
        R.sa = A.s + (size_t)ra * GD;
        R.ba = A.b + (size_t)ra * GD;
        R.sb = A.s + (size_t)rb * GD;
        R.bb = A.b + (size_t)rb * GD;
        float ya = 0.0f, yb = 0.0f, ea = 0.0f, eb = 0.0f;
        QuadLoads cur = load_quad(R, 0, 0, GD, t);
        for (int q0 = 0; q0 < GD; q0 += 4) {
            QuadLoads nxt = cur;
            if (q0 + 4 < GD) nxt = load_quad(R, q0 + 4, 0, GD, t);
            compute_quad(cur, q0, 0, GD, tbl, xs, cs, ya, yb);
            const int j = q0 + t;
            if (j < GD) {
                ea = fmaf(fmaf(1100.0f, fabsf(bf16f(cur.sa)), 2.0f * fabsf(bf16f(cur.ba))), xa[j], ea);
                eb = fmaf(fmaf(1100.0f, fabsf(bf16f(cur.sb)), 2.0f * fabsf(bf16f(cur.bb))), xa[j], eb);
            }
            cur = nxt;
        }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
            ya += __shfl_xor_sync(0xffffffffu, ya, o);
            yb += __shfl_xor_sync(0xffffffffu, yb, o);
            ea += __shfl_xor_sync(0xffffffffu, ea, o);
            eb += __shfl_xor_sync(0xffffffffu, eb, o);
        }
        // the bound's own fp32 sums are below 2^-20 of it: round it up by 2^-10
        ea *= 6.103515625e-05f * 1.0009765625f;
        eb *= 6.103515625e-05f * 1.0009765625f;
        if (t == 0) {
            const int r0 = tile * 16 + g, r1 = r0 + 8;
            if (r0 < A.rows) { A.ae[r0] = make_float2(ya, ea); lb = fmaxf(lb, ya - ea); }
            if (r1 < A.rows) { A.ae[r1] = make_float2(yb, eb); lb = fmaxf(lb, yb - eb); }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lb = fmaxf(lb, __shfl_xor_sync(0xffffffffu, lb, o));
    if (lane == 0) wlb[warp] = lb;
    __syncthreads();
    if (tid == 0) {
        float m = wlb[0];
        for (int w = 1; w < LM_THREADS / 32; ++w) m = fmaxf(m, wlb[w]);
        A.cta_lb[blockIdx.x] = m;
    }
}

// Exact CPU-order logit of one row (cpu_reference.cpp:55-83): lane l takes groups l and l + 32;
// per group dot += q_lo * x0, dot += q_hi * x1, sum += x0 + x1 element pair by pair, then
// term = s * dot + b * sum; lane 0 adds the 44 terms in group order.
__device__ float exact_row(const LmArgs& A, const float* sx, float* terms, int row) {
    const int lane = threadIdx.x & 31;
    const uint8_t* wr = A.w + (size_t)row * (D / 2);
    for (int gi = lane; gi < GD; gi += 32) {
        const float s = bf16f(A.s[(size_t)row * GD + gi]), b = bf16f(A.b[(size_t)row * GD + gi]);
        const uint4* wq = reinterpret_cast<const uint4*>(wr + gi * (kGroup / 2));
        const uint4 q0 = wq[0], q1 = wq[1];
        const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const float* xg = sx + gi * kGroup;
        float dot = 0.0f, sum = 0.0f;
#pragma unroll
        for (int wi = 0; wi < 8; ++wi) {
#pragma unroll
            for (int by = 0; by < 4; ++by) {
                const uint32_t byte = (words[wi] >> (8 * by)) & 0xFFu;
                const int e = wi * 8 + by * 2;
                const float x0 = xg[e], x1 = xg[e + 1];
                dot = __fadd_rn(dot, __fmul_rn((float)(byte & 0x0Fu), x0));
                dot = __fadd_rn(dot, __fmul_rn((float)(byte >> 4), x1));
                sum = __fadd_rn(sum, __fadd_rn(x0, x1));
            }
        }
        terms[gi] = __fadd_rn(__fmul_rn(s, dot), __fmul_rn(b, sum));
    }
    __syncwarp();
    float acc = 0.0f;
    if (lane == 0)
        for (int gi = 0; gi < GD; ++gi) acc = __fadd_rn(acc, terms[gi]);
    __syncwarp();
    return acc;
}

__global__ void __launch_bounds__(256) lm_exact(const __grid_constant__ LmArgs A) {
    __shared__ __align__(16) float sx[D];
    __shared__ float terms[256 / 32][GD];
    __shared__ float s_l;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < D; i += blockDim.x) sx[i] = A.x[i];
    if (tid < 32) {
        float m = -INFINITY;
        for (int i = tid; i < A.n_lb; i += 32) m = fmaxf(m, A.cta_lb[i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (tid == 0) s_l = m;
    }
    __syncthreads();
    const float L = s_l;
    const int nw = gridDim.x * (blockDim.x >> 5);
    for (int base = (blockIdx.x * (blockDim.x >> 5) + warp) * 32; base < A.rows; base += nw * 32) {
        const int r = base + lane;
        bool cand = false;
        if (r < A.rows) {
            const float2 v = A.ae[r];
            cand = v.x + v.y >= L;
        }
        unsigned m = __ballot_sync(0xffffffffu, cand);
        while (m) {
            const int k = __ffs(m) - 1;
            m &= m - 1;
            const int row = base + k;
            const float v = exact_row(A, sx, terms[warp], row);
            if (lane == 0) {
                atomicMax(A.key, ((unsigned long long)orderable(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)row));
                atomicAdd(A.n_cand, 1);
            }
        }
    }
}

__global__ void lm_finish(const __grid_constant__ LmArgs A) {
    const unsigned long long k = *A.key;
    *A.token = 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
    if (A.logit) *A.logit = from_orderable((uint32_t)(k >> 32));
}

}  // namespace dec

// Workspace: [0, 4096) barrier flags (4 kinds x 256 CTAs) and [4096] this launch's error word,
// both cleared before every launch; [4100] the sticky error word (zero-initialised once by the
// workspace's owner, read and cleared by gtm_moe_decode_check); from 4352: logits, act, partials.
constexpr size_t kErrOffset = 4096, kStickyOffset = 4100, kDataOffset = 4352;

size_t decode_workspace_bytes() {
    return kDataOffset + sizeof(float) * (dec::NE + dec::ACT_R + dec::FS + (size_t)dec::NSEG * dec::D) + 256;
}
size_t decode_sticky_offset() { return kStickyOffset; }

int launch_decode(const GtmDims& dims, const GtmLayer* layers, int num_layers, const GtmDecodeIO& io,
                  void* ws, size_t ws_bytes, cudaStream_t stream, int num_ctas) {
    using namespace dec;
    (void)ws_bytes;
    Params P;
    memset(&P, 0, sizeof(P));
    for (int l = 0; l < num_layers; ++l) P.layers[l] = layers[l];
    P.io = io;
    P.num_layers = num_layers;
    P.eps = dims.eps;
    P.inv_sqrt_d = 1.0f / sqrtf((float)D);
    const bool test_wait = (io.flags & GTM_DECODE_TEST_WAIT_RUNS_OUT) != 0;
    P.wait_limit_ns = test_wait ? 2000000ull : kTimeoutNs;
    P.first_wait_extra = test_wait ? 1u : 0u;
    unsigned char* w = static_cast<unsigned char*>(ws);
    P.flags = reinterpret_cast<unsigned*>(w);
    P.err = reinterpret_cast<int*>(w + kErrOffset);
    P.sticky = reinterpret_cast<int*>(w + kStickyOffset);
    float* f = reinterpret_cast<float*>(w + kDataOffset);
    P.logits = f;
    P.act = f + NE;
    P.part = P.act + FS + ACT_R;
    cudaError_t e = cudaMemsetAsync(w, 0, kErrOffset + sizeof(int), stream);
    if (e != cudaSuccess) return set_cuda_error("gtm_moe_decode: memset", e);
    const size_t smem = sizeof(Smem);
    static bool attr_done = false;
    if (!attr_done) {
        e = cudaFuncSetAttribute(moe_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return set_cuda_error("gtm_moe_decode: smem attribute", e);
        attr_done = true;
    }
    void* args[] = {(void*)&P};
    e = cudaLaunchCooperativeKernel((const void*)moe_decode_kernel, dim3(num_ctas), dim3(NT), args, smem, stream);
    if (e != cudaSuccess) return set_cuda_error("gtm_moe_decode: cooperative launch", e);
    return GTM_OK;
}

}  // namespace gtm

namespace gtm {

size_t lm_head_workspace_bytes(uint32_t rows) {
    return 256 + (size_t)rows * 8 + 4096 * 4;
}

int launch_lm_head(uint32_t rows, const void* w, const uint16_t* s, const uint16_t* b, const float* x, uint32_t* token,
                   float* logit, void* ws, cudaStream_t st, int num_sms) {
    using namespace dec;
    uint8_t* p = static_cast<uint8_t*>(ws);
    LmArgs A;
    memset(&A, 0, sizeof(A));
    A.w = static_cast<const uint8_t*>(w); A.s = s; A.b = b; A.x = x; A.rows = (int)rows;
    A.key = reinterpret_cast<unsigned long long*>(p);
    A.n_cand = reinterpret_cast<int*>(p + 8);
    A.ae = reinterpret_cast<float2*>(p + 256);
    A.cta_lb = reinterpret_cast<float*>(p + 256 + (size_t)rows * 8);
    A.token = token; A.logit = logit;
    const int g1 = std::min(num_sms * 3, 4096);   // persistent: three CTAs per SM
    A.n_lb = g1;
    lm_approx<<<g1, LM_THREADS, 0, st>>>(A);
    lm_exact<<<num_sms * 4, 256, 0, st>>>(A);
    lm_finish<<<1, 1, 0, st>>>(A);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("gtm_lm_head_greedy", e);
    return GTM_OK;
}

int lm_head_candidates(void* ws, cudaStream_t st, int* n) {
    const cudaError_t e = cudaMemcpyAsync(n, static_cast<uint8_t*>(ws) + 8, sizeof(int), cudaMemcpyDeviceToHost, st);
    const cudaError_t e2 = e == cudaSuccess ? cudaStreamSynchronize(st) : e;
    if (e2 != cudaSuccess) return set_cuda_error("gtm_lm_head_candidates", e2);
    return GTM_OK;
}

}  // namespace gtm

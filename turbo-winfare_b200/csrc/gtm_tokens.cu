// MoE block for T > 1 tokens (batched decode, prefill) on sm_100a.
//
// The reference runs every token through the per-expert GEMV chain one at a time
// (src/runner.cpp:845-854 for prefill, :612-657 per expert). Here the T tokens of a layer are
// grouped by expert and the expert products become dense contractions on the tcgen05 tensor
// cores:
//   1. tok_views_router   per token: views (exact RMS), router logits in the reference's exact
//                         order (or caller-given routing logits), optional logit bias, top-8
//   2. tok_route          counts per expert, token-slot rows grouped by expert, GEMM tile lists
//   3. tok_gather         routed_x rows in expert order, split into fp16 high and low parts
//   4. grouped_gemm<0>    gate/up of the 8 routed experts and the shared expert, GeGLU fused,
//                         activations written as fp16 high/low parts
//   5. grouped_gemm<1>    down projections, routing weight fused (routed rows)
//   6. tok_combine        h2 = sum over the 8 slots in router order, shared output, layer tail
//
// Grouped GEMM (one CTA per SM, persistent over a device-built tile list). A tile is 128 token
// rows x 512 output features (four 128-column fp32 accumulators in TMEM) over K in blocks of 64
// (one quantisation group). Operand A (tokens) is the fp16 high part and the fp16 low part of the
// activations, each loaded by TMA in the 128-byte swizzle layout; both are multiplied against the
// same B tile, so the products carry ~22 bits of the activation. Operand B (features) is the int4
// weight matrix dequantised in the kernel by six producer warps to fp16 w = q * scale + bias
// (exact when the bias is a multiple of the scale that fits fp16, as for the benchmark's
// zero-point 8) and written straight into the swizzled layout. One thread issues the tcgen05.mma
// (M=128, N=128, K=16); mbarriers hand stages between TMA, dequant and MMA; the epilogue warps read
// TMEM with tcgen05.ld. Every wait is bounded; on expiry the CTA unwinds, frees its TMEM and
// reports through the error word.
#include <cstdint>
#include <cstring>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gtm_common.cuh"
#include "gtm_internal.h"
#include "gtm_tcgen05.cuh"

namespace gtm {
namespace tok {

constexpr int D = 2816, FE = 704, FS = 2112, NE = 128, TOPK = 8, GD = D / kGroup;
constexpr int BM = 128, BK = 64, NSUB = 4, BNF = NSUB * 128, STAGES = 2;
constexpr int GEMM_THREADS = 256;
constexpr int DQ_THREADS = 192;          // warps 2..7
constexpr uint32_t A_TILE = BM * BK * 2; // 16 KB per fp16 operand tile
constexpr uint32_t B_TILE = BNF * BK * 2;  // 64 KB
constexpr uint64_t kWaitNs = 1000000000ull;
constexpr int RIN_PITCH = 65;

struct Tile {
    int32_t expert;   // routed expert id, or -1 for the shared expert
    int32_t row0;     // first activation row
    int32_t rows;     // valid rows (<= 128)
    int32_t ftile;    // feature tile (512 features)
};

// ================================================================================================
// 1. views + router + top-8, one CTA per token
// ================================================================================================
struct ViewsArgs {
    int T;
    const float* x_f32;          // [T][D] or null
    const uint16_t* x_bf16;      // [T][D] or null
    const uint8_t* resident;
    GtmLayer L;
    float eps, inv_sqrt_d;
    const float* logit_bias;     // [E] or null
    const float* route_logits;   // [T][E] or null
    __half* dense_hi;            // [T][D]
    __half* dense_lo;
    float* routed;               // [T][D] fp32
    uint32_t* idx;               // [T][8]
    float* w;                    // [T][8]
    float* logits_out;           // [T][E] or null
};

__device__ __forceinline__ const uint16_t* rp16(const void* base, uint64_t off) {
    return reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(base) + off);
}

__global__ void __launch_bounds__(512) tok_views_router(const __grid_constant__ ViewsArgs A) {
    __shared__ __align__(16) float sx[D];
    __shared__ float srin[GD * RIN_PITCH];
    __shared__ float slog[NE];
    __shared__ double red[40];
    const int t = blockIdx.x, tid = threadIdx.x;
    const GtmLayer& L = A.L;
    for (int i = tid; i < D; i += blockDim.x)
        sx[i] = A.x_f32 ? A.x_f32[(size_t)t * D + i] : bf16f(A.x_bf16[(size_t)t * D + i]);
    __syncthreads();
    const float inv = exact_rms_inv(sx, D, A.eps, red);
    const uint16_t* w_pre = rp16(L.resident_dev, L.pre_ffn_norm);
    const uint16_t* w_pre2 = rp16(L.resident_dev, L.pre_ffn_norm_2);
    const uint16_t* rs = rp16(L.resident_dev, L.router_scale);
    for (int i = tid; i < D; i += blockDim.x) {
        const float h = __fmul_rn(sx[i], inv);
        const float dx = __fmul_rn(h, bf16f(w_pre[i]));
        const __half hi = __float2half_rn(dx);
        A.dense_hi[(size_t)t * D + i] = hi;
        A.dense_lo[(size_t)t * D + i] = __float2half_rn(dx - __half2float(hi));
        A.routed[(size_t)t * D + i] = __fmul_rn(h, bf16f(w_pre2[i]));
        srin[(i >> 6) * RIN_PITCH + (i & 63)] = __fmul_rn(__fmul_rn(h, bf16f(rs[i])), A.inv_sqrt_d);
    }
    __syncthreads();
    if (A.route_logits) {
        for (int e = tid; e < NE; e += blockDim.x) slog[e] = A.route_logits[(size_t)t * NE + e];
    } else {
        // logits in src/cpu_reference.cpp:86-106's order: 11 rows at a time, 44 threads a row
        const uint8_t* W = static_cast<const uint8_t*>(L.resident_dev) + L.router.weight;
        const uint16_t* S = rp16(L.resident_dev, L.router.scales);
        const uint16_t* B = rp16(L.resident_dev, L.router.biases);
        __shared__ float terms[11][GD];
        for (int r0 = 0; r0 < NE; r0 += 11) {
            const int rr = tid / GD, g = tid - rr * GD, row = r0 + rr;
            if (rr < 11 && row < NE) {
                const uint4* wg = reinterpret_cast<const uint4*>(W + (size_t)row * D + g * kGroup);
                const float* x = srin + g * RIN_PITCH;
                float dot = 0.0f, sum = 0.0f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint4 q = ldg_stream_u4(wg + i);
                    const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int c = 0; c < 4; ++c)
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const float xv = x[i * 16 + c * 4 + b];
                            dot = __fadd_rn(dot, __fmul_rn((float)((wv[c] >> (8 * b)) & 0xFFu), xv));
                            sum = __fadd_rn(sum, xv);
                        }
                }
                terms[rr][g] = __fadd_rn(__fmul_rn(bf16f(S[row * GD + g]), dot), __fmul_rn(bf16f(B[row * GD + g]), sum));
            }
            __syncthreads();
            if (tid < 11 && r0 + tid < NE) {
                float acc = 0.0f;
                for (int g2 = 0; g2 < GD; ++g2) acc = __fadd_rn(acc, terms[tid][g2]);
                slog[r0 + tid] = acc;
            }
            __syncthreads();
        }
    }
    __syncthreads();
    if (tid < 32) {
        const int lane = tid;
        float v[4];
        uint32_t key[4];
        bool taken[4] = {false, false, false, false};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = lane + 32 * j;
            v[j] = A.logit_bias ? __fadd_rn(slog[e], A.logit_bias[e]) : slog[e];
            if (A.logits_out) A.logits_out[(size_t)t * NE + e] = v[j];
            const uint32_t u = __float_as_uint(v[j] == 0.0f ? 0.0f : v[j]);
            key[j] = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
        }
        float my_sel = 0.0f, top0 = 0.0f;
        int my_idx = 0;
#pragma unroll
        for (int k = 0; k < TOPK; ++k) {
            uint32_t ck = 0u, ci = 0xFFFFFFFFu;
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
        const float e = lane < TOPK ? expf(__fsub_rn(my_sel, top0)) : 0.0f;
        const uint16_t pes = lane < TOPK ? *rp16(L.resident_dev, L.per_expert_scale + 2ull * (uint32_t)my_idx) : 0;
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < TOPK; ++k) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, e, k));
        if (lane < TOPK) {
            A.idx[(size_t)t * TOPK + lane] = (uint32_t)my_idx;
            A.w[(size_t)t * TOPK + lane] = __fmul_rn(__fdiv_rn(e, sum), bf16f(pes));
        }
    }
}

// ================================================================================================
// 2. routing tables and tile lists (one CTA)
// ================================================================================================
struct RouteArgs {
    int T;
    const uint32_t* idx;     // [T][8]
    const float* w;          // [T][8]
    int* counts;             // [E]
    int* offsets;            // [E + 1]
    int* perm_token;         // [8T]
    float* perm_w;           // [8T]
    int* pos;                // [T][8]
    Tile* tiles0;            // gate/up tiles
    Tile* tiles1;            // down tiles
    int* n_tiles;            // [2]
};

constexpr int FT0_R = (2 * FE + BNF - 1) / BNF;   // 3 feature tiles of routed gate/up (1408 features)
constexpr int FT0_S = (2 * FS + BNF - 1) / BNF;   // 9 of shared gate/up (4224)
constexpr int FT1 = (D + BNF - 1) / BNF;          // 6 of the down projections (2816)

__global__ void __launch_bounds__(1024) tok_route(const __grid_constant__ RouteArgs A) {
    __shared__ int cnt[NE], off[NE + 1], t0[NE + 1], t1[NE + 1];
    const int tid = threadIdx.x, n = A.T * TOPK;
    for (int e = tid; e < NE; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
        const int e = (int)A.idx[i];
        A.pos[i] = atomicAdd(&cnt[e], 1);          // slot within the expert, completed below
    }
    __syncthreads();
    if (tid == 0) {
        int o = 0, a = 0, b = 0;
        for (int e = 0; e < NE; ++e) {
            off[e] = o; t0[e] = a; t1[e] = b;
            const int mt = (cnt[e] + BM - 1) / BM;
            o += cnt[e]; a += mt * FT0_R; b += mt * FT1;
        }
        off[NE] = o; t0[NE] = a; t1[NE] = b;
    }
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
        const int e = (int)A.idx[i];
        const int row = off[e] + A.pos[i];
        A.pos[i] = row;
        A.perm_token[row] = i / TOPK;
        A.perm_w[row] = A.w[i];
    }
    for (int e = tid; e < NE; e += blockDim.x) {
        A.counts[e] = cnt[e];
        A.offsets[e] = off[e];
        const int mt = (cnt[e] + BM - 1) / BM;
        for (int m = 0; m < mt; ++m) {
            const int r0 = off[e] + m * BM, rows = min(BM, cnt[e] - m * BM);
            for (int f = 0; f < FT0_R; ++f) A.tiles0[t0[e] + m * FT0_R + f] = Tile{e, r0, rows, f};
            for (int f = 0; f < FT1; ++f) A.tiles1[t1[e] + m * FT1 + f] = Tile{e, r0, rows, f};
        }
    }
    if (tid == 0) A.offsets[NE] = off[NE];
    // shared expert over all T tokens, after the routed tiles
    const int mts = (A.T + BM - 1) / BM;
    for (int i = tid; i < mts * FT0_S; i += blockDim.x) {
        const int m = i / FT0_S, f = i - m * FT0_S;
        A.tiles0[t0[NE] + i] = Tile{-1, m * BM, min(BM, A.T - m * BM), f};
    }
    for (int i = tid; i < mts * FT1; i += blockDim.x) {
        const int m = i / FT1, f = i - m * FT1;
        A.tiles1[t1[NE] + i] = Tile{-1, m * BM, min(BM, A.T - m * BM), f};
    }
    if (tid == 0) {
        A.n_tiles[0] = t0[NE] + mts * FT0_S;
        A.n_tiles[1] = t1[NE] + mts * FT1;
    }
}

// ================================================================================================
// 3. gather routed_x rows in expert order as fp16 high / low parts
// ================================================================================================
__global__ void __launch_bounds__(256) tok_gather(const float* routed, const int* perm_token, __half* xhi, __half* xlo) {
    const int row = blockIdx.x;
    const int t = perm_token[row];
    const float4* src = reinterpret_cast<const float4*>(routed + (size_t)t * D);
    for (int i = threadIdx.x; i < D / 4; i += blockDim.x) {
        const float4 v = src[i];
        const float f[4] = {v.x, v.y, v.z, v.w};
        __half h[4], l[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            h[q] = __float2half_rn(f[q]);
            l[q] = __float2half_rn(f[q] - __half2float(h[q]));
        }
        __half2* dh = reinterpret_cast<__half2*>(xhi + (size_t)row * D) + 2 * i;
        __half2* dl = reinterpret_cast<__half2*>(xlo + (size_t)row * D) + 2 * i;
        dh[0] = __halves2half2(h[0], h[1]); dh[1] = __halves2half2(h[2], h[3]);
        dl[0] = __halves2half2(l[0], l[1]); dl[1] = __halves2half2(l[2], l[3]);
    }
}

// ================================================================================================
// 4/5. grouped GEMM
// ================================================================================================
struct GemmArgs {
    CUtensorMap map_r_hi, map_r_lo, map_s_hi, map_s_lo;   // A operands (routed rows / shared rows)
    const Tile* tiles;
    const int* n_tiles;
    const uint8_t* experts;
    uint64_t expert_stride;
    GtmQuant ex_a, ex_b;        // routed: gate, up (mode 0) or down (mode 1)
    const uint8_t* resident;
    GtmQuant sh_a, sh_b;        // shared: gate, up (mode 0) or down (mode 1)
    int k_r, k_s;               // input width of the routed / shared operand
    int nf_r, nf_s;             // output features (mode 0: 2 x intermediate, gate/up interleaved)
    __half* act_r_hi; __half* act_r_lo;   // mode 0 outputs [rows][k of mode 1]
    __half* act_s_hi; __half* act_s_lo;
    float* out_r; float* out_s;           // mode 1 outputs [rows][D]
    const float* perm_w;                  // mode 1: routing weight per routed row
    int* err;
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// 8 int4 (low nibble first) -> 8 fp16 w = q * s + b in element order, packed in a uint4.
__device__ __forceinline__ uint4 dequant8(uint32_t w, uint32_t s2, uint32_t b2) {
    const uint32_t m = 0x64006400u, w8 = w >> 8;
    uint32_t l0, h0, l1, h1;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(l0) : "r"(w), "r"(0x000F000Fu), "r"(m));
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(h0) : "r"(w), "r"(0x00F000F0u), "r"(m));
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(l1) : "r"(w8), "r"(0x000F000Fu), "r"(m));
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(h1) : "r"(w8), "r"(0x00F000F0u), "r"(m));
    uint32_t q0, q1, q2, q3;   // (n0,n4) (n1,n5) (n2,n6) (n3,n7) as exact fp16
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q0) : "r"(l0), "r"(m));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(q1) : "r"(h0), "r"(0x2C002C00u), "r"(0xD400D400u));
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q2) : "r"(l1), "r"(m));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(q3) : "r"(h1), "r"(0x2C002C00u), "r"(0xD400D400u));
    // element order (n0,n1) (n2,n3) (n4,n5) (n6,n7)
    uint32_t p0 = prmt(q0, q1, 0x5410), p1 = prmt(q2, q3, 0x5410), p2 = prmt(q0, q1, 0x7632), p3 = prmt(q2, q3, 0x7632);
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(p0) : "r"(p0), "r"(s2), "r"(b2));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(p1) : "r"(p1), "r"(s2), "r"(b2));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(p2) : "r"(p2), "r"(s2), "r"(b2));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(p3) : "r"(p3), "r"(s2), "r"(b2));
    return make_uint4(p0, p1, p2, p3);
}

__device__ __forceinline__ uint32_t bf16_to_h2(uint16_t b) {
    const __half h = __float2half_rn(bf16f(b));
    const uint32_t u = __half_as_ushort(h);
    return u | (u << 16);
}

__device__ __forceinline__ float gelu_tanh_f(float x) {
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

struct TileInfo {
    Tile t;
    bool routed;
    int K, nkb, nf, nsub;
};

__device__ __forceinline__ TileInfo tile_info(const GemmArgs& A, int i) {
    TileInfo ti;
    ti.t = A.tiles[i];
    ti.routed = ti.t.expert >= 0;
    ti.K = ti.routed ? A.k_r : A.k_s;
    ti.nkb = ti.K / BK;
    ti.nf = ti.routed ? A.nf_r : A.nf_s;
    ti.nsub = min(NSUB, (ti.nf - ti.t.ftile * BNF + 127) / 128);
    return ti;
}

template <int MODE>
__global__ void __launch_bounds__(GEMM_THREADS, 1) grouped_gemm(const __grid_constant__ GemmArgs A) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sAhi = base;                        // [STAGES][16 KB]
    uint8_t* sAlo = base + STAGES * A_TILE;      // [STAGES][16 KB]
    uint8_t* sB = base + 2 * STAGES * A_TILE;    // [STAGES][64 KB]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * B_TILE);
    uint64_t* a_full = bars;                     // [STAGES]
    uint64_t* b_full = bars + STAGES;
    uint64_t* empty = bars + 2 * STAGES;
    uint64_t* acc_full = bars + 3 * STAGES;
    uint64_t* acc_empty = acc_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            tc::mbar_init(&a_full[s], 1);
            tc::mbar_init(&b_full[s], DQ_THREADS);
            tc::mbar_init(&empty[s], 1);
        }
        tc::mbar_init(acc_full, 1);
        tc::mbar_init(acc_empty, 128);
        *abort_flag = 0;
        tc::mbar_fence_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int ntiles = *A.n_tiles;
    const uint32_t idesc = tc::idesc_f16(BM, 128);

    if (warp == 0) {
        // ---- TMA producer: activation high/low tiles ----
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int i = blockIdx.x; i < ntiles && ok; i += gridDim.x) {
                const TileInfo ti = tile_info(A, i);
                const CUtensorMap* mh = ti.routed ? &A.map_r_hi : &A.map_s_hi;
                const CUtensorMap* ml = ti.routed ? &A.map_r_lo : &A.map_s_lo;
                for (int kb = 0; kb < ti.nkb; ++kb, ++it) {
                    const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
                    if (!tc::mbar_wait(&empty[s], ph ^ 1, abort_flag, kWaitNs)) { ok = false; break; }
                    tc::mbar_arrive_expect_tx(&a_full[s], 2 * A_TILE);
                    tc::tma_load_2d(sAhi + s * A_TILE, mh, kb * BK, ti.t.row0, &a_full[s]);
                    tc::tma_load_2d(sAlo + s * A_TILE, ml, kb * BK, ti.t.row0, &a_full[s]);
                }
            }
            // do not leave the CTA while TMA writes into its shared memory are in flight
            for (uint32_t j = it > STAGES ? it - STAGES : 0; j < it; ++j) {
                volatile int dummy = 0;
                tc::mbar_wait(&a_full[j % STAGES], (j / STAGES) & 1, &dummy, kWaitNs);
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer ----
        if (lane == 0) {
            uint32_t it = 0, acc_it = 0;
            bool ok = true;
            for (int i = blockIdx.x; i < ntiles && ok; i += gridDim.x) {
                const TileInfo ti = tile_info(A, i);
                if (!tc::mbar_wait(acc_empty, (acc_it & 1) ^ 1, abort_flag, kWaitNs)) break;
                tc::tc_fence_after();
                for (int kb = 0; kb < ti.nkb; ++kb, ++it) {
                    const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
                    if (!tc::mbar_wait(&a_full[s], ph, abort_flag, kWaitNs) ||
                        !tc::mbar_wait(&b_full[s], ph, abort_flag, kWaitNs)) { ok = false; break; }
                    tc::tc_fence_after();
                    const uint64_t dhi = tc::sdesc_sw128(tc::smem_u32(sAhi + s * A_TILE));
                    const uint64_t dlo = tc::sdesc_sw128(tc::smem_u32(sAlo + s * A_TILE));
                    const uint64_t db = tc::sdesc_sw128(tc::smem_u32(sB + s * B_TILE));
                    for (int sub = 0; sub < ti.nsub; ++sub) {
#pragma unroll
                        for (int k = 0; k < BK / 16; ++k) {
                            const uint64_t bk = db + (uint64_t)(sub * (128 * 128 / 16)) + (uint64_t)(2 * k);
                            tc::mma_f16(tmem + sub * 128, dhi + 2 * k, bk, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                            tc::mma_f16(tmem + sub * 128, dlo + 2 * k, bk, idesc, 1u);
                        }
                    }
                    tc::mma_commit(&empty[s]);
                }
                if (!ok) break;
                tc::mma_commit(acc_full);
                ++acc_it;
            }
            // let issued MMAs finish before TMEM is released
            if (it > 0) {
                volatile int dummy = 0;
                const uint32_t j = it - 1;
                tc::mbar_wait(&empty[j % STAGES], (j / STAGES) & 1, &dummy, kWaitNs);
            }
        }
    } else {
        // ---- warps 2..7: B producers (dequant); warps 4..7 also the epilogue ----
        const int dq = tid - 64;
        const bool epi = warp >= 4;
        const int q = warp & 3;                   // TMEM lane quadrant of this warp
        uint32_t it = 0, acc_it = 0;
        for (int i = blockIdx.x; i < ntiles; i += gridDim.x) {
            const TileInfo ti = tile_info(A, i);
            const uint8_t* wbase = ti.routed ? A.experts + (uint64_t)ti.t.expert * A.expert_stride : A.resident;
            const GtmQuant& qa = ti.routed ? A.ex_a : A.sh_a;
            const GtmQuant& qb = ti.routed ? A.ex_b : A.sh_b;
            const int K = ti.K, G = K / kGroup;
            bool ok = true;
            for (int kb = 0; kb < ti.nkb; ++kb, ++it) {
                const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
                if (!tc::mbar_wait(&empty[s], ph ^ 1, abort_flag, kWaitNs)) { ok = false; break; }
                uint8_t* dst = sB + s * B_TILE;
                for (int r = dq; r < ti.nsub * 128; r += DQ_THREADS) {
                    const int g = ti.t.ftile * BNF + r;
                    const GtmQuant* qm;
                    int row;
                    if (MODE == 0) { qm = (g & 1) ? &qb : &qa; row = g >> 1; }
                    else { qm = &qa; row = g; }
                    const uint8_t* wrow = wbase + qm->weight + (uint64_t)row * (K / 2) + kb * 32;
                    const uint4 w0 = *reinterpret_cast<const uint4*>(wrow);
                    const uint4 w1 = *reinterpret_cast<const uint4*>(wrow + 16);
                    const uint32_t s2 = bf16_to_h2(*reinterpret_cast<const uint16_t*>(wbase + qm->scales + ((uint64_t)row * G + kb) * 2));
                    const uint32_t b2 = bf16_to_h2(*reinterpret_cast<const uint16_t*>(wbase + qm->biases + ((uint64_t)row * G + kb) * 2));
                    const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                    uint8_t* rowp = dst + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                        *reinterpret_cast<uint4*>(rowp + ((c ^ (r & 7)) << 4)) = dequant8(words[c], s2, b2);
                }
                tc::fence_proxy_async_smem();
                tc::mbar_arrive(&b_full[s]);
            }
            if (!ok) break;
            if (!epi) continue;
            // ---- epilogue: thread (quadrant q, lane) owns token row row0 + 32q + lane ----
            if (!tc::mbar_wait(acc_full, acc_it & 1, abort_flag, kWaitNs)) break;
            ++acc_it;
            tc::tc_fence_after();
            const int r = 32 * q + lane;
            const bool valid = r < ti.t.rows;
            const int row = ti.t.row0 + r;
            const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16);
            const float wgt = (MODE == 1 && ti.routed && valid) ? A.perm_w[row] : 1.0f;
            for (int sub = 0; sub < ti.nsub; ++sub) {
#pragma unroll 1
                for (int c16 = 0; c16 < 8; ++c16) {
                    uint32_t v[16];
                    tc::tmem_ld16_sync(taddr + sub * 128 + c16 * 16, v);
                    const int f0 = ti.t.ftile * BNF + sub * 128 + c16 * 16;
                    if (!valid || f0 >= ti.nf) continue;
                    if (MODE == 0) {
                        // columns alternate gate / up of intermediate rows f0/2 .. f0/2 + 7
                        __half hi[8], lo[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float a = gelu_tanh_f(__uint_as_float(v[2 * j])) * __uint_as_float(v[2 * j + 1]);
                            hi[j] = __float2half_rn(a);
                            lo[j] = __float2half_rn(a - __half2float(hi[j]));
                        }
                        const int kout = ti.nf / 2;
                        __half* dh = (ti.routed ? A.act_r_hi : A.act_s_hi) + (size_t)row * kout + f0 / 2;
                        __half* dl = (ti.routed ? A.act_r_lo : A.act_s_lo) + (size_t)row * kout + f0 / 2;
                        uint4 ph4, pl4;
                        ph4.x = (uint32_t)__half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[1]) << 16);
                        ph4.y = (uint32_t)__half_as_ushort(hi[2]) | ((uint32_t)__half_as_ushort(hi[3]) << 16);
                        ph4.z = (uint32_t)__half_as_ushort(hi[4]) | ((uint32_t)__half_as_ushort(hi[5]) << 16);
                        ph4.w = (uint32_t)__half_as_ushort(hi[6]) | ((uint32_t)__half_as_ushort(hi[7]) << 16);
                        pl4.x = (uint32_t)__half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[1]) << 16);
                        pl4.y = (uint32_t)__half_as_ushort(lo[2]) | ((uint32_t)__half_as_ushort(lo[3]) << 16);
                        pl4.z = (uint32_t)__half_as_ushort(lo[4]) | ((uint32_t)__half_as_ushort(lo[5]) << 16);
                        pl4.w = (uint32_t)__half_as_ushort(lo[6]) | ((uint32_t)__half_as_ushort(lo[7]) << 16);
                        *reinterpret_cast<uint4*>(dh) = ph4;
                        *reinterpret_cast<uint4*>(dl) = pl4;
                    } else {
                        float* dst = (ti.routed ? A.out_r : A.out_s) + (size_t)row * D + f0;
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            reinterpret_cast<float4*>(dst)[j] =
                                make_float4(__uint_as_float(v[4 * j]) * wgt, __uint_as_float(v[4 * j + 1]) * wgt,
                                            __uint_as_float(v[4 * j + 2]) * wgt, __uint_as_float(v[4 * j + 3]) * wgt);
                    }
                }
            }
            tc::tc_fence_before();
            tc::mbar_arrive(acc_empty);
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (tid == 0 && *abort_flag) atomicExch(A.err, 2);
    if (warp == 1) {
        __syncwarp();
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
        tc::tmem_relinquish();
    }
}

// ================================================================================================
// 6. combine + layer tail, one CTA per token
// ================================================================================================
struct CombineArgs {
    int T;
    const float* x_f32;
    const uint16_t* x_bf16;
    const int* pos;           // [T][8]
    const float* out_r;       // [8T][D], routing weight applied
    const float* out_s;       // [T][D]
    GtmLayer L;
    float eps;
    float* hidden_out;        // [T][D]
    float* h1_out;            // [T][D] or null
    float* h2_out;            // [T][D] or null
};

__device__ __forceinline__ double block_sum(double v, double* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double s = 0.0;
    for (int w = 0; w < nw; ++w) s += red[w];
    return s;
}

__global__ void __launch_bounds__(512) tok_combine(const __grid_constant__ CombineArgs A) {
    __shared__ __align__(16) float sh[D];
    __shared__ __align__(16) float h2[D];
    __shared__ double red[32];
    const int t = blockIdx.x, tid = threadIdx.x;
    const GtmLayer& L = A.L;
    int p[TOPK];
#pragma unroll
    for (int k = 0; k < TOPK; ++k) p[k] = A.pos[(size_t)t * TOPK + k];
    double a = 0.0, b = 0.0;
    for (int i = tid; i < D; i += blockDim.x) {
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < TOPK; ++k) acc += A.out_r[(size_t)p[k] * D + i];
        const float so = A.out_s[(size_t)t * D + i];
        h2[i] = acc;
        sh[i] = so;
        a += (double)so * so;
        b += (double)acc * acc;
    }
    const float inv1 = 1.0f / sqrtf((float)(block_sum(a, red) / D) + A.eps);
    const float inv2 = 1.0f / sqrtf((float)(block_sum(b, red) / D) + A.eps);
    const uint16_t* w_pf1 = rp16(L.resident_dev, L.post_ffn_norm_1);
    const uint16_t* w_pf2 = rp16(L.resident_dev, L.post_ffn_norm_2);
    const uint16_t* w_pf = rp16(L.resident_dev, L.post_ffn_norm);
    const float ls = bf16f(*rp16(L.resident_dev, L.layer_scalar));
    a = 0.0;
    for (int i = tid; i < D; i += blockDim.x) {
        const float h1 = (sh[i] * inv1) * bf16f(w_pf1[i]);
        if (A.h1_out) A.h1_out[(size_t)t * D + i] = h1;
        if (A.h2_out) A.h2_out[(size_t)t * D + i] = h2[i];
        const float tv = (h2[i] * inv2) * bf16f(w_pf2[i]) + h1;
        h2[i] = tv;
        a += (double)tv * tv;
    }
    const float inv3 = 1.0f / sqrtf((float)(block_sum(a, red) / D) + A.eps);
    for (int i = tid; i < D; i += blockDim.x) {
        const float x = A.x_f32 ? A.x_f32[(size_t)t * D + i] : bf16f(A.x_bf16[(size_t)t * D + i]);
        A.hidden_out[(size_t)t * D + i] = (x + (h2[i] * inv3) * bf16f(w_pf[i])) * ls;
    }
}

// ================================================================================================
// host side
// ================================================================================================
struct WsLayout {
    size_t dense_hi, dense_lo, routed, idx, w, counts, offsets, perm_token, perm_w, pos, tiles0, tiles1, n_tiles,
        xhi, xlo, act_r_hi, act_r_lo, act_s_hi, act_s_lo, out_r, out_s, total;
};

static size_t align256(size_t n) { return (n + 255) / 256 * 256; }

static WsLayout ws_layout(uint32_t T) {
    WsLayout W;
    const size_t R = (size_t)T * TOPK;
    const size_t mt_max = R / BM + NE + 1, mts = (T + BM - 1) / BM;
    size_t o = 256;   // [0, 256): error word
    auto take = [&](size_t bytes) { const size_t at = o; o = align256(o + bytes); return at; };
    W.dense_hi = take((size_t)T * D * 2);
    W.dense_lo = take((size_t)T * D * 2);
    W.routed = take((size_t)T * D * 4);
    W.idx = take(R * 4);
    W.w = take(R * 4);
    W.counts = take(NE * 4);
    W.offsets = take((NE + 1) * 4);
    W.perm_token = take(R * 4);
    W.perm_w = take(R * 4);
    W.pos = take(R * 4);
    W.tiles0 = take((mt_max * FT0_R + mts * FT0_S) * sizeof(Tile));
    W.tiles1 = take((mt_max * FT1 + mts * FT1) * sizeof(Tile));
    W.n_tiles = take(2 * 4);
    W.xhi = take(R * D * 2);
    W.xlo = take(R * D * 2);
    W.act_r_hi = take(R * FE * 2);
    W.act_r_lo = take(R * FE * 2);
    W.act_s_hi = take((size_t)T * FS * 2);
    W.act_s_lo = take((size_t)T * FS * 2);
    W.out_r = take(R * D * 4);
    W.out_s = take((size_t)T * D * 4);
    W.total = o;
    return W;
}

}  // namespace tok

size_t tokens_workspace_bytes(uint32_t max_tokens) { return tok::ws_layout(max_tokens).total; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static int encode_map(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t k) {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q);
        if (e != cudaSuccess || !f) return set_error(GTM_ERR_CUDA, "cuTensorMapEncodeTiled not available");
        fn = reinterpret_cast<EncodeTiledFn>(f);
    }
    const cuuint64_t dims[2] = {k, rows};
    const cuuint64_t strides[1] = {k * 2};
    const cuuint32_t box[2] = {tok::BK, tok::BM};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(GTM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return GTM_OK;
}

int launch_tokens(const GtmDims& dims, const GtmLayer& L, const GtmTokensIO& io, void* ws, size_t ws_bytes,
                  cudaStream_t st, int num_sms) {
    using namespace tok;
    const uint32_t T = io.num_tokens;
    const WsLayout W = ws_layout(T);
    if (ws_bytes < W.total) return set_error(GTM_ERR_WORKSPACE, "gtm_moe_tokens: workspace needs %zu bytes", W.total);
    uint8_t* w = static_cast<uint8_t*>(ws);
    auto P = [&](size_t off) { return static_cast<void*>(w + off); };
    int* err = reinterpret_cast<int*>(w);

    ViewsArgs va;
    memset(&va, 0, sizeof(va));
    va.T = (int)T; va.x_f32 = io.x_dev; va.x_bf16 = io.x_bf16_dev; va.L = L; va.eps = dims.eps;
    va.inv_sqrt_d = 1.0f / sqrtf((float)D);
    va.logit_bias = io.logit_bias_dev; va.route_logits = io.route_logits_dev;
    va.dense_hi = static_cast<__half*>(P(W.dense_hi)); va.dense_lo = static_cast<__half*>(P(W.dense_lo));
    va.routed = static_cast<float*>(P(W.routed));
    va.idx = static_cast<uint32_t*>(P(W.idx)); va.w = static_cast<float*>(P(W.w));
    va.logits_out = io.logits_dev;
    tok_views_router<<<T, 512, 0, st>>>(va);

    RouteArgs ra;
    ra.T = (int)T; ra.idx = va.idx; ra.w = va.w;
    ra.counts = static_cast<int*>(P(W.counts)); ra.offsets = static_cast<int*>(P(W.offsets));
    ra.perm_token = static_cast<int*>(P(W.perm_token)); ra.perm_w = static_cast<float*>(P(W.perm_w));
    ra.pos = static_cast<int*>(P(W.pos));
    ra.tiles0 = static_cast<Tile*>(P(W.tiles0)); ra.tiles1 = static_cast<Tile*>(P(W.tiles1));
    ra.n_tiles = static_cast<int*>(P(W.n_tiles));
    tok_route<<<1, 1024, 0, st>>>(ra);

    tok_gather<<<T * TOPK, 256, 0, st>>>(va.routed, ra.perm_token, static_cast<__half*>(P(W.xhi)),
                                         static_cast<__half*>(P(W.xlo)));

    const size_t smem = 1024 + 2 * STAGES * A_TILE + STAGES * B_TILE + 256;
    cudaFuncSetAttribute(grouped_gemm<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(grouped_gemm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const uint64_t R = (uint64_t)T * TOPK;
    GemmArgs g0;
    memset(&g0, 0, sizeof(g0));
    int rc;
    if ((rc = encode_map(&g0.map_r_hi, P(W.xhi), R, D)) || (rc = encode_map(&g0.map_r_lo, P(W.xlo), R, D)) ||
        (rc = encode_map(&g0.map_s_hi, P(W.dense_hi), T, D)) || (rc = encode_map(&g0.map_s_lo, P(W.dense_lo), T, D)))
        return rc;
    g0.tiles = ra.tiles0; g0.n_tiles = ra.n_tiles;
    g0.experts = static_cast<const uint8_t*>(L.experts_dev); g0.expert_stride = L.expert_stride;
    g0.ex_a = L.expert_gate; g0.ex_b = L.expert_up;
    g0.resident = static_cast<const uint8_t*>(L.resident_dev); g0.sh_a = L.shared_gate; g0.sh_b = L.shared_up;
    g0.k_r = D; g0.k_s = D; g0.nf_r = 2 * FE; g0.nf_s = 2 * FS;
    g0.act_r_hi = static_cast<__half*>(P(W.act_r_hi)); g0.act_r_lo = static_cast<__half*>(P(W.act_r_lo));
    g0.act_s_hi = static_cast<__half*>(P(W.act_s_hi)); g0.act_s_lo = static_cast<__half*>(P(W.act_s_lo));
    g0.err = err;
    grouped_gemm<0><<<num_sms, GEMM_THREADS, smem, st>>>(g0);

    GemmArgs g1;
    memset(&g1, 0, sizeof(g1));
    if ((rc = encode_map(&g1.map_r_hi, g0.act_r_hi, R, FE)) || (rc = encode_map(&g1.map_r_lo, g0.act_r_lo, R, FE)) ||
        (rc = encode_map(&g1.map_s_hi, g0.act_s_hi, T, FS)) || (rc = encode_map(&g1.map_s_lo, g0.act_s_lo, T, FS)))
        return rc;
    g1.tiles = ra.tiles1; g1.n_tiles = ra.n_tiles + 1;
    g1.experts = g0.experts; g1.expert_stride = L.expert_stride;
    g1.ex_a = L.expert_down; g1.ex_b = L.expert_down;
    g1.resident = g0.resident; g1.sh_a = L.shared_down; g1.sh_b = L.shared_down;
    g1.k_r = FE; g1.k_s = FS; g1.nf_r = D; g1.nf_s = D;
    g1.out_r = static_cast<float*>(P(W.out_r)); g1.out_s = static_cast<float*>(P(W.out_s));
    g1.perm_w = ra.perm_w;
    g1.err = err;
    grouped_gemm<1><<<num_sms, GEMM_THREADS, smem, st>>>(g1);

    CombineArgs ca;
    ca.T = (int)T; ca.x_f32 = io.x_dev; ca.x_bf16 = io.x_bf16_dev; ca.pos = ra.pos;
    ca.out_r = g1.out_r; ca.out_s = g1.out_s; ca.L = L; ca.eps = dims.eps;
    ca.hidden_out = io.hidden_out_dev; ca.h1_out = io.h1_dev; ca.h2_out = io.h2_dev;
    tok_combine<<<T, 512, 0, st>>>(ca);

    if (io.topk_idx_dev) cudaMemcpyAsync(io.topk_idx_dev, va.idx, R * 4, cudaMemcpyDeviceToDevice, st);
    if (io.topk_w_dev) cudaMemcpyAsync(io.topk_w_dev, va.w, R * 4, cudaMemcpyDeviceToDevice, st);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("gtm_moe_tokens", e);
    return GTM_OK;
}

int tokens_check(void* ws, cudaStream_t st) {
    int flag = 0;
    cudaError_t e = cudaMemcpyAsync(&flag, ws, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return set_cuda_error("gtm_moe_tokens_check", e);
    if (flag) {
        const int zero = 0;
        cudaMemcpy(ws, &zero, sizeof(int), cudaMemcpyHostToDevice);
        return set_error(GTM_ERR_TIMEOUT, "gtm_moe_tokens: a grouped-GEMM pipeline wait timed out (flag %d)", flag);
    }
    return GTM_OK;
}

}  // namespace gtm

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
//   4. grouped_gemm<0>    gate/up of the routed experts and the shared expert, GeGLU fused,
//                         activations written as fp16 high/low parts
//   5. grouped_gemm<1>    down projections, routing weight fused (routed rows)
//   6. tok_combine        h2 = sum over the 8 slots in router order, shared output, layer tail
//
// Grouped GEMM: one CTA per SM, persistent over a tile list built on the device. A tile is 256
// weight rows (two MMA M=128 halves) by up to 96 tokens of one expert (MMA N), over K in blocks of
// 64 (one quantisation group): D[row][token] += W[row][k] X[token][k]. Gate/up tiles put 128 gate
// rows in one half and the same 128 up rows in the other, so one epilogue thread holds both
// halves of its GeGLU pair. Tensor memory (512 columns) holds two accumulator sets of 2 x 96
// columns and two weight stages of 64 columns. Per K block:
//   * warps 8-15 (one thread per weight row) fetch the row's 32 packed bytes through a private
//     cp.async pipeline 6 blocks deep, dequantise them to fp16 w = q * scale + bias (the bf16
//     scale/bias prefetched into registers two blocks ahead; w is exact in fp16 when the bias is
//     a small multiple of the scale, as for zero-point-8 weights) and store the row straight into
//     its tensor-memory lane with tcgen05.st, so the weights never pass through shared memory;
//   * warp 0 loads the activation tile by TMA, the fp16 high part and the fp16 low part
//     (x - hi), so the MMAs against the same weights carry ~22 bits of the activation; it also
//     prefetches the CTA's next tile of weights into L2;
//   * one thread of warp 1 issues tcgen05.mma (kind::f16, M=128, N=16..96, K=16, A from tensor
//     memory, B from shared memory) for both halves and both activation parts into one of the two
//     accumulator sets, committing stage and tile completion to mbarriers;
//   * warps 4-7 drain the other accumulator set with tcgen05.ld while the next tile runs.
// Within every 8-element chunk of K the dequantised weights come out in the order
// (0,4,1,5,2,6,3,7), the order the nibble extraction yields; activations are stored in the same
// order, so the products are unchanged and no permute instructions are spent.
// Every wait is bounded; on expiry the CTA unwinds, frees its TMEM and reports through the error
// word of the workspace.
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
constexpr int BK = 64;                  // K block = one quantisation group
constexpr int NT = 96;                  // tokens per tile (MMA N, at most)
constexpr int SX = 4;                   // activation stages (shared memory)
constexpr int SW = 2;                   // dequantised-weight stages (tensor memory)
constexpr int NACC = 2;                 // accumulator sets (tensor memory, 2 x NT columns each)
constexpr uint32_t ACC_SET = 2 * NT;    // one set: the two 128-row halves, NT token columns each
constexpr uint32_t A_COL0 = NACC * ACC_SET;  // first TMEM column of the weight stages (64 columns each)
constexpr int DR = 6;                   // packed-weight cp.async depth per dequant thread
constexpr int THREADS = 512;
constexpr int DQ0 = 256, DQ_THREADS = 256;   // dequant threads: warps 8..15, one weight row each
constexpr uint32_t X_TILE = NT * BK * 2;     // 12 KB per activation part
constexpr uint32_t XBOX = 32 * BK * 2;       // 4 KB: one TMA box of 32 token rows
constexpr uint32_t RAW_TILE = 256 * 32;      // 8 KB packed int4 per K block
constexpr size_t SMEM_BYTES = 1024 + 2 * SX * X_TILE + DR * RAW_TILE + (2 * SX + 2 * SW + 2 * NACC) * 8 + 16;
static_assert(A_COL0 + SW * 64 <= 512, "tensor memory columns");
constexpr int FB0_R = (FE + 127) / 128, FB0_S = (FS + 127) / 128;   // gate/up tiles: 128 intermediate rows
constexpr int FB1 = D / 256;                                        // down tiles: 256 output rows
constexpr uint64_t kWaitNs = 1000000000ull;
constexpr int RIN_PITCH = 65;

static_assert(SMEM_BYTES <= 232448, "grouped GEMM shared memory");
static_assert(FE % 64 == 0 && FS % 64 == 0 && D % 256 == 0, "tile shapes");

struct Tile {
    int32_t expert;   // routed expert id, or -1 for the shared expert
    int32_t row0;     // first activation row of the token range
    int32_t rows;     // tokens (1..NT)
    int32_t fb;       // weight-row block
};

// K position of element k inside its 8-element chunk, in the order the dequant produces.
__host__ __device__ __forceinline__ int kperm(int k) { return (k & ~7) | ((k & 3) << 1) | ((k >> 2) & 1); }

__device__ __forceinline__ const uint16_t* rp16(const void* base, uint64_t off) {
    return reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(base) + off);
}

// ================================================================================================
// 1. views + router + top-8, one CTA per token
// ================================================================================================
struct ViewsArgs {
    int T;
    const float* x_f32;          // [T][D] or null
    const uint16_t* x_bf16;      // [T][D] or null
    GtmLayer L;
    float eps, inv_sqrt_d;
    const float* logit_bias;     // [E] or null
    const float* route_logits;   // [T][E] or null
    __half* dense_hi;            // [T][D] (K-permuted)
    __half* dense_lo;
    float* routed;               // [T][D] fp32
    uint32_t* idx;               // [T][8]
    float* w;                    // [T][8]
    float* logits_out;           // [T][E] or null
};

__global__ void __launch_bounds__(512) tok_views_router(const __grid_constant__ ViewsArgs A) {
    __shared__ __align__(16) float sx[D];
    __shared__ float srin[GD * RIN_PITCH];
    __shared__ float slog[NE];
    __shared__ double red[40];
    __shared__ float terms[11][GD];
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
        A.dense_hi[(size_t)t * D + kperm(i)] = hi;
        A.dense_lo[(size_t)t * D + kperm(i)] = __float2half_rn(dx - __half2float(hi));
        A.routed[(size_t)t * D + i] = __fmul_rn(h, bf16f(w_pre2[i]));
        srin[(i >> 6) * RIN_PITCH + (i & 63)] = __fmul_rn(__fmul_rn(h, bf16f(rs[i])), A.inv_sqrt_d);
    }
    __syncthreads();
    if (A.route_logits) {
        for (int e = tid; e < NE; e += blockDim.x) slog[e] = A.route_logits[(size_t)t * NE + e];
    } else {
        // logits in src/cpu_reference.cpp:86-106's order: 11 rows at a time, 44 threads a row
        const uint8_t* W = static_cast<const uint8_t*>(L.resident_dev) + L.router.weight;
        const uint16_t* Sc = rp16(L.resident_dev, L.router.scales);
        const uint16_t* Bi = rp16(L.resident_dev, L.router.biases);
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
                terms[rr][g] = __fadd_rn(__fmul_rn(bf16f(Sc[row * GD + g]), dot), __fmul_rn(bf16f(Bi[row * GD + g]), sum));
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
        // top-8 by (value desc, index asc), src/cpu_reference.cpp:447-480
        const int lane = tid;
        uint32_t key[4];
        bool taken[4] = {false, false, false, false};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = lane + 32 * j;
            const float v = A.logit_bias ? __fadd_rn(slog[e], A.logit_bias[e]) : slog[e];
            if (A.logits_out) A.logits_out[(size_t)t * NE + e] = v;
            const uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);
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
    int n;                   // routed entries (0: shared tiles only)
    int src_div;             // activation source row of entry i = i / src_div
    const uint32_t* idx;     // expert id of entry i at idx[i * stride]
    const float* w;          // routing weight of entry i at w[i * stride]
    int stride;
    int e0, ne;              // experts of this launch: [e0, e0 + ne); tiles carry e - e0
    int t_shared;            // tokens of the shared-expert tiles (0: none)
    int* perm_src;           // [n] source row of each expert-ordered row
    float* perm_w;           // [n] routing weight of each row
    int* pos;                // [n] expert-ordered row of each entry
    Tile* tiles0;            // gate/up tiles
    Tile* tiles1;            // down tiles
    int* n_tiles;            // [2]
};

__device__ __forceinline__ int ntok_tiles(int c) { return (c + NT - 1) / NT; }

__global__ void __launch_bounds__(1024) tok_route(const __grid_constant__ RouteArgs A) {
    __shared__ int cnt[NE], off[NE + 1], t0[NE + 1], t1[NE + 1];
    const int tid = threadIdx.x, n = A.n;
    for (int e = tid; e < NE; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
        const int e = (int)A.idx[(size_t)i * A.stride] - A.e0;
        A.pos[i] = (e >= 0 && e < A.ne) ? atomicAdd(&cnt[e], 1) : -1;
    }
    __syncthreads();
    if (tid == 0) {
        int o = 0, a = 0, b = 0;
        for (int e = 0; e < A.ne; ++e) {
            off[e] = o; t0[e] = a; t1[e] = b;
            const int nt = ntok_tiles(cnt[e]);
            o += cnt[e]; a += nt * FB0_R; b += nt * FB1;
        }
        off[A.ne] = o; t0[A.ne] = a; t1[A.ne] = b;
    }
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
        if (A.pos[i] < 0) continue;   // entry of another rank's expert (not produced by the dispatch)
        const int row = off[(int)A.idx[(size_t)i * A.stride] - A.e0] + A.pos[i];
        A.pos[i] = row;
        A.perm_src[row] = i / A.src_div;
        A.perm_w[row] = A.w[(size_t)i * A.stride];
    }
    // tiles of one (expert, row block) are adjacent over the token ranges, for L2 reuse of the weights
    for (int e = tid; e < A.ne; e += blockDim.x) {
        const int c = cnt[e], nt = ntok_tiles(c);
        for (int m = 0; m < nt; ++m) {
            const int r0 = c * m / nt, r1 = c * (m + 1) / nt;
            for (int f = 0; f < FB0_R; ++f) A.tiles0[t0[e] + f * nt + m] = Tile{e, off[e] + r0, r1 - r0, f};
            for (int f = 0; f < FB1; ++f) A.tiles1[t1[e] + f * nt + m] = Tile{e, off[e] + r0, r1 - r0, f};
        }
    }
    const int T = A.t_shared, nts = ntok_tiles(T), b0 = t0[A.ne], b1 = t1[A.ne];
    for (int i = tid; i < nts * FB0_S; i += blockDim.x) {
        const int f = i / nts, m = i - f * nts, r0 = T * m / nts, r1 = T * (m + 1) / nts;
        A.tiles0[b0 + i] = Tile{-1, r0, r1 - r0, f};
    }
    for (int i = tid; i < nts * FB1; i += blockDim.x) {
        const int f = i / nts, m = i - f * nts, r0 = T * m / nts, r1 = T * (m + 1) / nts;
        A.tiles1[b1 + i] = Tile{-1, r0, r1 - r0, f};
    }
    if (tid == 0) {
        A.n_tiles[0] = b0 + nts * FB0_S;
        A.n_tiles[1] = b1 + nts * FB1;
    }
}

// ================================================================================================
// 2b. expert-parallel dispatch: (token, slot) entries grouped by destination rank, in (token,
//     slot) order inside each group, so the layout is the same on every run
// ================================================================================================
struct DispatchArgs {
    int n;                   // entries (tokens x top_k)
    int world, epr;          // ranks, experts per rank
    const uint32_t* idx;     // [n]
    const float* w;          // [n]
    int* send_counts;        // [world]
    int* send_pos;           // [n] send row of each entry
    int* send_src;           // [n] token of each send row
    GtmEpMeta* send_meta;    // [n] (expert, weight) of each send row
};

constexpr int kMaxWorld = 64;

__global__ void __launch_bounds__(1024) tok_dispatch(const __grid_constant__ DispatchArgs A) {
    __shared__ int run[kMaxWorld], wtot[32][kMaxWorld], off[kMaxWorld];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int d = tid; d < A.world; d += blockDim.x) run[d] = 0;
    __syncthreads();
    for (int base = 0; base < A.n; base += blockDim.x) {
        const int i = base + tid;
        const int d = i < A.n ? (int)A.idx[i] / A.epr : -1;
        int mine = 0;
        for (int q = 0; q < A.world; ++q) {
            const unsigned m = __ballot_sync(0xffffffffu, d == q);
            if (d == q) mine = __popc(m & ((1u << lane) - 1u));
            if (lane == 0) wtot[warp][q] = __popc(m);
        }
        __syncthreads();
        if (d >= 0) {
            int before = run[d];
            for (int w2 = 0; w2 < warp; ++w2) before += wtot[w2][d];
            A.send_pos[i] = before + mine;   // position inside destination d's group
        }
        __syncthreads();
        for (int q = tid; q < A.world; q += blockDim.x) {
            int s = 0;
            for (int w2 = 0; w2 < 32; ++w2) s += wtot[w2][q];
            run[q] += s;
        }
        __syncthreads();
    }
    if (tid == 0) {
        int o = 0;
        for (int q = 0; q < A.world; ++q) { off[q] = o; o += run[q]; A.send_counts[q] = run[q]; }
    }
    __syncthreads();
    for (int i = tid; i < A.n; i += blockDim.x) {
        const int row = off[(int)A.idx[i] / A.epr] + A.send_pos[i];
        A.send_pos[i] = row;
        A.send_src[row] = i / TOPK;
        A.send_meta[row] = GtmEpMeta{A.idx[i], A.w[i]};
    }
}

__global__ void __launch_bounds__(256) tok_copy_rows(const float* src, const int* src_row, float* dst) {
    const int row = blockIdx.x;
    const float4* s4 = reinterpret_cast<const float4*>(src + (size_t)src_row[row] * D);
    float4* d4 = reinterpret_cast<float4*>(dst + (size_t)row * D);
    for (int c = threadIdx.x; c < D / 4; c += blockDim.x) d4[c] = s4[c];
}

// ================================================================================================
// 3. gather routed_x rows in expert order as fp16 high / low parts (K-permuted)
// ================================================================================================
__global__ void __launch_bounds__(128) tok_gather(const float* routed, const int* perm_src, __half* xhi, __half* xlo) {
    const int row = blockIdx.x;
    const float4* src = reinterpret_cast<const float4*>(routed + (size_t)perm_src[row] * D);
    for (int c = threadIdx.x; c < D / 8; c += blockDim.x) {
        const float4 a = src[2 * c], b = src[2 * c + 1];
        const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        uint16_t h[8], l[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const __half hv = __float2half_rn(f[e]);
            h[kperm(e)] = __half_as_ushort(hv);
            l[kperm(e)] = __half_as_ushort(__float2half_rn(f[e] - __half2float(hv)));
        }
        uint4 ph, pl;
        ph.x = h[0] | ((uint32_t)h[1] << 16); ph.y = h[2] | ((uint32_t)h[3] << 16);
        ph.z = h[4] | ((uint32_t)h[5] << 16); ph.w = h[6] | ((uint32_t)h[7] << 16);
        pl.x = l[0] | ((uint32_t)l[1] << 16); pl.y = l[2] | ((uint32_t)l[3] << 16);
        pl.z = l[4] | ((uint32_t)l[5] << 16); pl.w = l[6] | ((uint32_t)l[7] << 16);
        reinterpret_cast<uint4*>(xhi + (size_t)row * D)[c] = ph;
        reinterpret_cast<uint4*>(xlo + (size_t)row * D)[c] = pl;
    }
}

// ================================================================================================
// 4/5. grouped GEMM
// ================================================================================================
struct GemmArgs {
    CUtensorMap x_rhi, x_rlo, x_shi, x_slo;   // activations, 2D fp16, 32-row boxes
    const Tile* tiles;
    const int* n_tiles;
    const uint8_t* experts;
    uint64_t expert_stride;
    uint64_t r_wa, r_wb, r_sa, r_ba, r_sb, r_bb;   // routed weight / scale / bias byte offsets (matrix a, b)
    const uint8_t* resident;
    uint64_t s_wa, s_wb, s_sa, s_ba, s_sb, s_bb;   // shared
    int k_r, k_s;                         // K of the routed / shared matrices
    int rows_r, rows_s;                   // rows of each routed / shared matrix
    __half* act_r_hi; __half* act_r_lo;   // mode 0 outputs, rows of FE (routed) / FS (shared)
    __half* act_s_hi; __half* act_s_lo;
    float* out_r; float* out_s;           // mode 1 outputs [rows][D]
    const float* perm_w;                  // mode 1: routing weight per routed row
    const int* out_index;                 // mode 1: output row of each routed row (null: same row)
    int* err;
};

// 8 int4 (low nibble first) -> 8 fp16 w = q * s + b in the order (0,4,1,5,2,6,3,7).
__device__ __forceinline__ uint4 dq8(uint32_t w, uint32_t s2, uint32_t b2) {
    const uint32_t m = 0x64006400u, w8 = w >> 8;
    uint32_t l0, h0, l1, h1;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(l0) : "r"(w), "r"(0x000F000Fu), "r"(m));
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(h0) : "r"(w), "r"(0x00F000F0u), "r"(m));
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(l1) : "r"(w8), "r"(0x000F000Fu), "r"(m));
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(h1) : "r"(w8), "r"(0x00F000F0u), "r"(m));
    uint4 r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(l0) : "r"(l0), "r"(m));                                   // (n0, n4)
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(h0) : "r"(h0), "r"(0x2C002C00u), "r"(0xD400D400u));  // (n1, n5)
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(l1) : "r"(l1), "r"(m));                                   // (n2, n6)
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(h1) : "r"(h1), "r"(0x2C002C00u), "r"(0xD400D400u));  // (n3, n7)
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r.x) : "r"(l0), "r"(s2), "r"(b2));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r.y) : "r"(h0), "r"(s2), "r"(b2));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r.z) : "r"(l1), "r"(s2), "r"(b2));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r.w) : "r"(h1), "r"(s2), "r"(b2));
    return r;
}

__device__ __forceinline__ uint32_t bf16_to_h2(uint16_t b) {
    const uint32_t u = __half_as_ushort(__float2half_rn(bf16f(b)));
    return u | (u << 16);
}

__device__ __forceinline__ float gelu_tanh_f(float x) {
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

struct TileInfo {
    Tile t;
    bool routed;
    int nkb;
};

__device__ __forceinline__ TileInfo tile_info(const GemmArgs& A, int i) {
    TileInfo ti;
    ti.t = A.tiles[i];
    ti.routed = ti.t.expert >= 0;
    ti.nkb = (ti.routed ? A.k_r : A.k_s) / BK;
    return ti;
}

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1) grouped_gemm(const __grid_constant__ GemmArgs A) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sXh = base;                         // [SX][12 KB]    activation high parts, SW128
    uint8_t* sXl = sXh + SX * X_TILE;            // [SX][12 KB]    activation low parts
    uint8_t* sRaw = sXl + SX * X_TILE;           // [DR][256][32]  packed int4, one row per dequant thread
    uint64_t* bars = reinterpret_cast<uint64_t*>(sRaw + DR * RAW_TILE);
    uint64_t* act_full = bars;
    uint64_t* act_empty = act_full + SX;
    uint64_t* w_full = act_empty + SX;
    uint64_t* w_empty = w_full + SW;
    uint64_t* acc_full = w_empty + SW;       // [NACC]
    uint64_t* acc_empty = acc_full + NACC;   // [NACC]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + NACC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < SX; ++s) { tc::mbar_init(&act_full[s], 1); tc::mbar_init(&act_empty[s], 1); }
        for (int s = 0; s < SW; ++s) { tc::mbar_init(&w_full[s], DQ_THREADS); tc::mbar_init(&w_empty[s], 1); }
        for (int b = 0; b < NACC; ++b) { tc::mbar_init(&acc_full[b], 1); tc::mbar_init(&acc_empty[b], 128); }
        *abort_flag = 0;
        tc::mbar_fence_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int ntiles = *A.n_tiles;

    if (warp == 0) {
        // ---- activation producer; L2 prefetch of the next tile's weights ----
        if (lane == 0) {
            auto prefetch_tile = [&](int i2) {
                const TileInfo tn = tile_info(A, i2);
                const uint8_t* wb = tn.routed ? A.experts + (uint64_t)tn.t.expert * A.expert_stride : A.resident;
                const uint64_t K = (uint64_t)tn.nkb * BK, G = tn.nkb;
                const uint64_t nr = tn.routed ? A.rows_r : A.rows_s;
                const uint64_t span = MODE == 0 ? 128 : 256, j0 = (uint64_t)tn.t.fb * span;
                const uint64_t rows = j0 + span <= nr ? span : nr - j0;
                for (int mtx = 0; mtx < (MODE == 0 ? 2 : 1); ++mtx) {
                    const uint64_t wo = tn.routed ? (mtx ? A.r_wb : A.r_wa) : (mtx ? A.s_wb : A.s_wa);
                    const uint64_t so = tn.routed ? (mtx ? A.r_sb : A.r_sa) : (mtx ? A.s_sb : A.s_sa);
                    const uint64_t bo = tn.routed ? (mtx ? A.r_bb : A.r_ba) : (mtx ? A.s_bb : A.s_ba);
                    tc::prefetch_l2_bulk(wb + wo + j0 * (K / 2), rows * (K / 2));
                    tc::prefetch_l2_bulk(wb + so + j0 * G * 2, rows * G * 2);
                    tc::prefetch_l2_bulk(wb + bo + j0 * G * 2, rows * G * 2);
                }
            };
            if ((int)blockIdx.x < ntiles) prefetch_tile(blockIdx.x);
            uint32_t it = 0;
            bool ok = true;
            for (int i = blockIdx.x; i < ntiles && ok; i += gridDim.x) {
                if (i + (int)gridDim.x < ntiles) prefetch_tile(i + gridDim.x);
                const TileInfo ti = tile_info(A, i);
                const CUtensorMap* mh = ti.routed ? &A.x_rhi : &A.x_shi;
                const CUtensorMap* ml = ti.routed ? &A.x_rlo : &A.x_slo;
                const int nbox = (ti.t.rows + 31) >> 5;
                for (int kb = 0; kb < ti.nkb; ++kb, ++it) {
                    const uint32_t s = it % SX, ph = (it / SX) & 1;
                    if (!tc::mbar_wait(&act_empty[s], ph ^ 1, abort_flag, kWaitNs)) { ok = false; break; }
                    tc::mbar_arrive_expect_tx(&act_full[s], 2u * XBOX * (uint32_t)nbox);
                    for (int j = 0; j < nbox; ++j) {
                        tc::tma_load_2d(sXh + s * X_TILE + j * XBOX, mh, kb * BK, ti.t.row0 + 32 * j, &act_full[s]);
                        tc::tma_load_2d(sXl + s * X_TILE + j * XBOX, ml, kb * BK, ti.t.row0 + 32 * j, &act_full[s]);
                    }
                }
            }
            // no exit while TMA writes into this CTA's shared memory are in flight
            volatile int never = 0;
            for (uint32_t j = it > SX ? it - SX : 0; j < it; ++j)
                tc::mbar_wait(&act_full[j % SX], (j / SX) & 1, &never, kWaitNs);
        }
    } else if (warp == 1) {
        // ---- MMA issuer (the whole warp; one elected lane issues): per K step, both 128-row
        //      halves x (activation high, low). Waits are warp-uniform so the warp stays converged.
        uint32_t it = 0, acc_it = 0;
        bool ok = true;
        for (int i = blockIdx.x; i < ntiles && ok; i += gridDim.x) {
            const TileInfo ti = tile_info(A, i);
            const uint32_t ab = acc_it % NACC, aph = (acc_it / NACC) & 1;
            if (!__all_sync(0xffffffffu, tc::mbar_wait(&acc_empty[ab], aph ^ 1, abort_flag, kWaitNs))) break;
            tc::tc_fence_after();
            const uint32_t d = tmem + ab * ACC_SET;
            const uint32_t idesc = tc::idesc_f16(128, (uint32_t)((ti.t.rows + 15) & ~15));
            for (int kb = 0; kb < ti.nkb; ++kb, ++it) {
                const uint32_t sx = it % SX, phx = (it / SX) & 1, sw = it % SW, phw = (it / SW) & 1;
                if (!__all_sync(0xffffffffu, tc::mbar_wait(&w_full[sw], phw, abort_flag, kWaitNs) &&
                                                 tc::mbar_wait(&act_full[sx], phx, abort_flag, kWaitNs))) { ok = false; break; }
                tc::tc_fence_after();
                // weights in TMEM: half h of stage sw at columns A_COL0 + 64 sw + 32 h, 8 per K step
                const uint32_t ta0 = tmem + A_COL0 + sw * 64, ta1 = ta0 + 32;
                const uint64_t dh = tc::sdesc_sw128(tc::smem_u32(sXh + sx * X_TILE));
                const uint64_t dl = tc::sdesc_sw128(tc::smem_u32(sXl + sx * X_TILE));
#pragma unroll
                for (int k = 0; k < BK / 16; ++k) {
                    const uint32_t first = (kb > 0 || k > 0) ? 1u : 0u;
                    tc::mma_f16_ts(d, ta0 + 8 * k, dh + 2 * k, idesc, first);
                    tc::mma_f16_ts(d + NT, ta1 + 8 * k, dh + 2 * k, idesc, first);
                    tc::mma_f16_ts(d, ta0 + 8 * k, dl + 2 * k, idesc, 1u);
                    tc::mma_f16_ts(d + NT, ta1 + 8 * k, dl + 2 * k, idesc, 1u);
                }
                tc::mma_commit(&w_empty[sw]);
                tc::mma_commit(&act_empty[sx]);
            }
            if (!ok) break;
            tc::mma_commit(&acc_full[ab]);
            ++acc_it;
        }
        if (it > 0) {   // issued MMAs finish before TMEM is released
            volatile int never = 0;
            tc::mbar_wait(&w_empty[(it - 1) % SW], ((it - 1) / SW) & 1, &never, kWaitNs);
        }
    } else if (warp >= 8) {
        // ---- dequant: one weight row per thread; its packed bytes come through a private
        //      cp.async pipeline DR blocks deep (no barrier: each thread reads only what it copied) ----
        const int r = tid - DQ0;                    // tile row 0..255
        const int hr = r >> 7, rr = r & 127;        // 128-row half, row within the half
        // this thread's TMEM lane is rr (warp 8 + r/32 reaches lanes 32 (warp % 4) ..)
        const uint32_t tlane = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + A_COL0 + (uint32_t)hr * 32u;
        const uint32_t raw_row = tc::smem_u32(sRaw) + (uint32_t)r * 32u;
        const uint32_t rsw = (uint32_t)((r >> 2) & 1);   // 16-byte half swap: conflict-free 16-byte reads
        uint32_t it = 0;
        bool ok = true;
        for (int i = blockIdx.x; i < ntiles && ok; i += gridDim.x) {
            const TileInfo ti = tile_info(A, i);
            const uint8_t* wb = ti.routed ? A.experts + (uint64_t)ti.t.expert * A.expert_stride : A.resident;
            const int G = ti.nkb;
            const int nrows = ti.routed ? A.rows_r : A.rows_s;
            int row;
            uint64_t wo, so, bo;
            if (MODE == 0) {
                row = ti.t.fb * 128 + rr;
                wo = ti.routed ? (hr ? A.r_wb : A.r_wa) : (hr ? A.s_wb : A.s_wa);
                so = ti.routed ? (hr ? A.r_sb : A.r_sa) : (hr ? A.s_sb : A.s_sa);
                bo = ti.routed ? (hr ? A.r_bb : A.r_ba) : (hr ? A.s_bb : A.s_ba);
            } else {
                row = ti.t.fb * 256 + r;
                wo = ti.routed ? A.r_wa : A.s_wa;
                so = ti.routed ? A.r_sa : A.s_sa;
                bo = ti.routed ? A.r_ba : A.s_ba;
            }
            const bool valid = row < nrows;   // rows past the matrix (last gate/up block) dequantise to 0
            const uint8_t* wsrc = wb + wo + (uint64_t)(valid ? row : 0) * (uint64_t)(G * 32);
            const uint16_t* sp = reinterpret_cast<const uint16_t*>(wb + so) + (size_t)(valid ? row : 0) * G;
            const uint16_t* bp = reinterpret_cast<const uint16_t*>(wb + bo) + (size_t)(valid ? row : 0) * G;
            auto issue = [&](int kb) {
                if (valid && kb < G) {
                    const uint32_t dst = raw_row + (uint32_t)(kb % DR) * RAW_TILE;
                    cp_async16(dst + (rsw << 4), wsrc + kb * 32);
                    cp_async16(dst + ((rsw ^ 1u) << 4), wsrc + kb * 32 + 16);
                }
                cp_async_commit();
            };
#pragma unroll
            for (int k = 0; k < DR - 1; ++k) issue(k);
            auto step = [&](int kb, uint16_t sbits, uint16_t bbits) -> bool {
                issue(kb + DR - 1);
                cp_async_wait<DR - 1>();
                const uint8_t* src = sRaw + (uint32_t)(kb % DR) * RAW_TILE + r * 32;
                const uint4 q0 = *reinterpret_cast<const uint4*>(src + (rsw << 4));
                const uint4 q1 = *reinterpret_cast<const uint4*>(src + ((rsw ^ 1u) << 4));
                const uint32_t sc = valid ? bf16_to_h2(sbits) : 0u, bi = valid ? bf16_to_h2(bbits) : 0u;
                uint32_t o[32];
                *reinterpret_cast<uint4*>(&o[0]) = dq8(q0.x, sc, bi);
                *reinterpret_cast<uint4*>(&o[4]) = dq8(q0.y, sc, bi);
                *reinterpret_cast<uint4*>(&o[8]) = dq8(q0.z, sc, bi);
                *reinterpret_cast<uint4*>(&o[12]) = dq8(q0.w, sc, bi);
                *reinterpret_cast<uint4*>(&o[16]) = dq8(q1.x, sc, bi);
                *reinterpret_cast<uint4*>(&o[20]) = dq8(q1.y, sc, bi);
                *reinterpret_cast<uint4*>(&o[24]) = dq8(q1.z, sc, bi);
                *reinterpret_cast<uint4*>(&o[28]) = dq8(q1.w, sc, bi);
                const uint32_t sw = it % SW, phw = (it / SW) & 1;
                // warp-uniform outcome: tcgen05.st is warp-collective
                if (!__all_sync(0xffffffffu, tc::mbar_wait(&w_empty[sw], phw ^ 1, abort_flag, kWaitNs))) return false;
                tc::tc_fence_after();
                tc::tmem_st32(tlane + sw * 64, o);
                tc::tmem_st_wait();
                tc::tc_fence_before();
                tc::mbar_arrive(&w_full[sw]);
                ++it;
                return true;
            };
            // scale/bias of blocks kb, kb+1 in registers; those of kb+2, kb+3 load during two blocks' work
            uint16_t s0 = sp[0], b0 = bp[0], s1 = G > 1 ? sp[1] : 0, b1 = G > 1 ? bp[1] : 0;
            for (int kb = 0; kb < G; kb += 2) {
                const uint16_t s2 = kb + 2 < G ? sp[kb + 2] : 0, b2 = kb + 2 < G ? bp[kb + 2] : 0;
                const uint16_t s3 = kb + 3 < G ? sp[kb + 3] : 0, b3 = kb + 3 < G ? bp[kb + 3] : 0;
                if (!step(kb, s0, b0) || (kb + 1 < G && !step(kb + 1, s1, b1))) { ok = false; break; }
                s0 = s2; b0 = b2; s1 = s3; b1 = b3;
            }
            cp_async_wait<0>();
        }
    } else if (warp >= 4) {
        // ---- epilogue: warp (4 + q) reads TMEM lanes 32q..32q+31 of both accumulators ----
        const int q = warp & 3;
        uint32_t acc_it = 0;
        for (int i = blockIdx.x; i < ntiles; i += gridDim.x) {
            const TileInfo ti = tile_info(A, i);
            const uint32_t ab = acc_it % NACC, aph = (acc_it / NACC) & 1;
            // warp-uniform outcome: tcgen05.ld is warp-collective
            if (!__all_sync(0xffffffffu, tc::mbar_wait(&acc_full[ab], aph, abort_flag, kWaitNs))) break;
            tc::tc_fence_after();
            const uint32_t taddr = tmem + ab * ACC_SET + ((uint32_t)(32 * q) << 16);
            const int rows = ti.t.rows, row0 = ti.t.row0;
            if (MODE == 1) {
                // accumulator a holds output rows fb*256 + 128a + (32q + lane)
                const int f0 = ti.t.fb * 256 + 32 * q + lane;
                float* out = ti.routed ? A.out_r : A.out_s;
                for (int c0 = 0; c0 < rows; c0 += 16) {
                    const int tl = c0 + (lane & 15);
                    const float wl = ti.routed && tl < rows ? A.perm_w[row0 + tl] : 1.0f;
                    uint32_t v0[16], v1[16];
                    tc::tmem_ld16_sync(taddr + c0, v0);
                    tc::tmem_ld16_sync(taddr + NT + c0, v1);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int t = c0 + j;
                        const float wgt = __shfl_sync(0xffffffffu, wl, j);
                        if (t < rows) {
                            const int orow = ti.routed && A.out_index ? A.out_index[row0 + t] : row0 + t;
                            float* o = out + (size_t)orow * D + f0;
                            o[0] = __uint_as_float(v0[j]) * wgt;
                            o[128] = __uint_as_float(v1[j]) * wgt;
                        }
                    }
                }
            } else {
                // accumulator 0: gate rows, accumulator 1: the same up rows -> GeGLU in-thread
                const int kout = ti.routed ? FE : FS;
                const int f = ti.t.fb * 128 + 32 * q + lane;
                const bool fvalid = f < kout;
                const int fcol = kperm(fvalid ? f : 0);
                __half* oh = (ti.routed ? A.act_r_hi : A.act_s_hi) + fcol;
                __half* ol = (ti.routed ? A.act_r_lo : A.act_s_lo) + fcol;
                for (int c0 = 0; c0 < rows; c0 += 16) {
                    uint32_t g[16], u[16];
                    tc::tmem_ld16_sync(taddr + c0, g);
                    tc::tmem_ld16_sync(taddr + NT + c0, u);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int t = c0 + j;
                        if (t < rows && fvalid) {
                            const float a = gelu_tanh_f(__uint_as_float(g[j])) * __uint_as_float(u[j]);
                            const __half hi = __float2half_rn(a);
                            const size_t o = (size_t)(row0 + t) * kout;
                            oh[o] = hi;
                            ol[o] = __float2half_rn(a - __half2float(hi));
                        }
                    }
                }
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&acc_empty[ab]);
            ++acc_it;
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

// h1 = rms(shared)*w_pf1 (cpu_reference.cpp:492-493); h2 = sum_k w_k out_k in router order
// (:508-509); hidden = (x + rms(rms(h2)*w_pf2 + h1)*w_pf) * layer_scalar (:512-520).
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
    size_t dense_hi, dense_lo, routed, idx, w, perm_src, perm_w, pos, tiles0, tiles1, n_tiles, xhi, xlo, act_r_hi,
        act_r_lo, act_s_hi, act_s_lo, out_r, out_s, send_pos, send_src, total;
};

static size_t align256(size_t n) { return (n + 255) / 256 * 256; }

// T: own tokens; R: routed rows through the experts (T * top_k on one GPU, the received rows
// with expert parallelism); ep: room for the dispatch tables.
static WsLayout ws_layout(uint32_t T, uint32_t Rrows, bool ep) {
    WsLayout W;
    const size_t E8 = (size_t)T * TOPK, R = Rrows;
    const size_t ntr = R / NT + NE, nts = (T + NT - 1) / NT;   // bounds on routed / shared token tiles
    size_t o = 256;   // [0, 256): error word
    auto take = [&](size_t bytes) { const size_t at = o; o = align256(o + bytes); return at; };
    W.dense_hi = take((size_t)T * D * 2);
    W.dense_lo = take((size_t)T * D * 2);
    W.routed = take((size_t)T * D * 4);
    W.idx = take(E8 * 4);
    W.w = take(E8 * 4);
    W.perm_src = take(R * 4);
    W.perm_w = take(R * 4);
    W.pos = take(R * 4);
    W.tiles0 = take((ntr * FB0_R + nts * FB0_S) * sizeof(Tile));
    W.tiles1 = take((ntr * FB1 + nts * FB1) * sizeof(Tile));
    W.n_tiles = take(2 * 4);
    W.xhi = take(R * D * 2);
    W.xlo = take(R * D * 2);
    W.act_r_hi = take(R * FE * 2);
    W.act_r_lo = take(R * FE * 2);
    W.act_s_hi = take((size_t)T * FS * 2);
    W.act_s_lo = take((size_t)T * FS * 2);
    W.out_r = ep ? 0 : take(R * D * 4);
    W.out_s = take((size_t)T * D * 4);
    W.send_pos = ep ? take(E8 * 4) : 0;
    W.send_src = ep ? take(E8 * 4) : 0;
    W.total = o;
    return W;
}

}  // namespace tok

size_t tokens_workspace_bytes(uint32_t max_tokens) { return tok::ws_layout(max_tokens, max_tokens * tok::TOPK, false).total; }
size_t ep_workspace_bytes(uint32_t max_tokens, uint32_t max_recv) { return tok::ws_layout(max_tokens, max_recv, true).total; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    }
    return fn;
}

// Activation map: fp16 [rows][k], boxes of 64 (k) x 32 rows in the 128-byte swizzle layout.
static int map_act(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t k) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_error(GTM_ERR_CUDA, "cuTensorMapEncodeTiled not available");
    const cuuint64_t dims[2] = {k, rows};
    const cuuint64_t strides[1] = {k * 2};
    const cuuint32_t box[2] = {tok::BK, 32};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(GTM_ERR_CUDA, "cuTensorMapEncodeTiled (activations) failed (%d)", (int)r);
    return GTM_OK;
}

namespace {

using namespace tok;

struct Ws {
    WsLayout W;
    uint8_t* base;
    void* at(size_t off) const { return base + off; }
    template <class T> T* p(size_t off) const { return reinterpret_cast<T*>(base + off); }
};

void launch_views(const GtmDims& dims, const GtmLayer& L, const GtmTokensIO& io, const Ws& w, cudaStream_t st) {
    ViewsArgs va;
    memset(&va, 0, sizeof(va));
    va.T = (int)io.num_tokens; va.x_f32 = io.x_dev; va.x_bf16 = io.x_bf16_dev; va.L = L; va.eps = dims.eps;
    va.inv_sqrt_d = 1.0f / sqrtf((float)D);
    va.logit_bias = io.logit_bias_dev; va.route_logits = io.route_logits_dev;
    va.dense_hi = w.p<__half>(w.W.dense_hi); va.dense_lo = w.p<__half>(w.W.dense_lo);
    va.routed = w.p<float>(w.W.routed);
    va.idx = w.p<uint32_t>(w.W.idx); va.w = w.p<float>(w.W.w);
    va.logits_out = io.logits_dev;
    tok_views_router<<<io.num_tokens, 512, 0, st>>>(va);
}

// What one pass of the two grouped GEMMs runs over.
struct Plan {
    int n;                        // routed entries (rows through the experts)
    int src_div;                  // activation source row of entry i = i / src_div
    const uint32_t* idx;          // expert ids, stride `stride`
    const float* w;               // routing weights, stride `stride`
    int stride;
    int e0, ne;                   // experts [e0, e0 + ne), layer.experts_dev pointing at e0
    int t_shared;                 // tokens through the shared expert (0: none)
    const float* src_rows;        // fp32 routed_x rows the entries read
    const int* out_index;         // mode 1 output row of each expert-ordered row (null: same)
    float* out_r;                 // mode 1 routed output rows
};

int run_gemms(const GtmLayer& L, const Ws& w, const Plan& pl, int num_sms, cudaStream_t st) {
    const WsLayout& W = w.W;
    const uint8_t* res = static_cast<const uint8_t*>(L.resident_dev);
    const uint8_t* exb = static_cast<const uint8_t*>(L.experts_dev);
    const uint64_t R = pl.n > 0 ? (uint64_t)pl.n : 1, T = pl.t_shared > 0 ? (uint64_t)pl.t_shared : 1;

    GemmArgs g0, g1;
    memset(&g0, 0, sizeof(g0));
    memset(&g1, 0, sizeof(g1));
    int rc;
    if ((rc = map_act(&g0.x_rhi, w.at(W.xhi), R, D)) || (rc = map_act(&g0.x_rlo, w.at(W.xlo), R, D)) ||
        (rc = map_act(&g0.x_shi, w.at(W.dense_hi), T, D)) || (rc = map_act(&g0.x_slo, w.at(W.dense_lo), T, D)) ||
        (rc = map_act(&g1.x_rhi, w.at(W.act_r_hi), R, FE)) || (rc = map_act(&g1.x_rlo, w.at(W.act_r_lo), R, FE)) ||
        (rc = map_act(&g1.x_shi, w.at(W.act_s_hi), T, FS)) || (rc = map_act(&g1.x_slo, w.at(W.act_s_lo), T, FS)))
        return rc;

    RouteArgs ra;
    ra.n = pl.n; ra.src_div = pl.src_div; ra.idx = pl.idx; ra.w = pl.w; ra.stride = pl.stride;
    ra.e0 = pl.e0; ra.ne = pl.ne; ra.t_shared = pl.t_shared;
    ra.perm_src = w.p<int>(W.perm_src); ra.perm_w = w.p<float>(W.perm_w); ra.pos = w.p<int>(W.pos);
    ra.tiles0 = w.p<Tile>(W.tiles0); ra.tiles1 = w.p<Tile>(W.tiles1); ra.n_tiles = w.p<int>(W.n_tiles);
    tok_route<<<1, 1024, 0, st>>>(ra);
    if (pl.n > 0)
        tok_gather<<<(unsigned)pl.n, 128, 0, st>>>(pl.src_rows, ra.perm_src, w.p<__half>(W.xhi), w.p<__half>(W.xlo));

    cudaFuncSetAttribute(grouped_gemm<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    cudaFuncSetAttribute(grouped_gemm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);

    g0.tiles = ra.tiles0; g0.n_tiles = ra.n_tiles;
    g0.experts = exb; g0.expert_stride = L.expert_stride; g0.resident = res;
    g0.r_wa = L.expert_gate.weight; g0.r_wb = L.expert_up.weight;
    g0.s_wa = L.shared_gate.weight; g0.s_wb = L.shared_up.weight;
    g0.r_sa = L.expert_gate.scales; g0.r_ba = L.expert_gate.biases; g0.r_sb = L.expert_up.scales; g0.r_bb = L.expert_up.biases;
    g0.s_sa = L.shared_gate.scales; g0.s_ba = L.shared_gate.biases; g0.s_sb = L.shared_up.scales; g0.s_bb = L.shared_up.biases;
    g0.k_r = D; g0.k_s = D; g0.rows_r = FE; g0.rows_s = FS;
    g0.act_r_hi = w.p<__half>(W.act_r_hi); g0.act_r_lo = w.p<__half>(W.act_r_lo);
    g0.act_s_hi = w.p<__half>(W.act_s_hi); g0.act_s_lo = w.p<__half>(W.act_s_lo);
    g0.err = w.p<int>(0);
    grouped_gemm<0><<<num_sms, THREADS, SMEM_BYTES, st>>>(g0);

    g1.tiles = ra.tiles1; g1.n_tiles = ra.n_tiles + 1;
    g1.experts = exb; g1.expert_stride = L.expert_stride; g1.resident = res;
    g1.r_wa = L.expert_down.weight; g1.r_wb = g1.r_wa; g1.s_wa = L.shared_down.weight; g1.s_wb = g1.s_wa;
    g1.r_sa = L.expert_down.scales; g1.r_ba = L.expert_down.biases; g1.r_sb = g1.r_sa; g1.r_bb = g1.r_ba;
    g1.s_sa = L.shared_down.scales; g1.s_ba = L.shared_down.biases; g1.s_sb = g1.s_sa; g1.s_bb = g1.s_ba;
    g1.k_r = FE; g1.k_s = FS; g1.rows_r = D; g1.rows_s = D;
    g1.out_r = pl.out_r; g1.out_s = w.p<float>(W.out_s);
    g1.perm_w = ra.perm_w; g1.out_index = pl.out_index;
    g1.err = w.p<int>(0);
    grouped_gemm<1><<<num_sms, THREADS, SMEM_BYTES, st>>>(g1);
    return GTM_OK;
}

void launch_combine(const GtmDims& dims, const GtmLayer& L, const GtmTokensIO& io, const Ws& w, const int* pos,
                    const float* out_r, cudaStream_t st) {
    CombineArgs ca;
    ca.T = (int)io.num_tokens; ca.x_f32 = io.x_dev; ca.x_bf16 = io.x_bf16_dev; ca.pos = pos;
    ca.out_r = out_r; ca.out_s = w.p<float>(w.W.out_s); ca.L = L; ca.eps = dims.eps;
    ca.hidden_out = io.hidden_out_dev; ca.h1_out = io.h1_dev; ca.h2_out = io.h2_dev;
    tok_combine<<<io.num_tokens, 512, 0, st>>>(ca);
}

int finish(const char* what, const GtmTokensIO* io, const Ws* w, cudaStream_t st) {
    if (io && w) {
        const size_t n = (size_t)io->num_tokens * TOPK * 4;
        if (io->topk_idx_dev) cudaMemcpyAsync(io->topk_idx_dev, w->at(w->W.idx), n, cudaMemcpyDeviceToDevice, st);
        if (io->topk_w_dev) cudaMemcpyAsync(io->topk_w_dev, w->at(w->W.w), n, cudaMemcpyDeviceToDevice, st);
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(what, e);
    return GTM_OK;
}

}  // namespace

int launch_tokens(const GtmDims& dims, const GtmLayer& L, const GtmTokensIO& io, void* ws, size_t ws_bytes,
                  cudaStream_t st, int num_sms) {
    const uint32_t T = io.num_tokens;
    const Ws w{ws_layout(T, T * TOPK, false), static_cast<uint8_t*>(ws)};
    if (ws_bytes < w.W.total) return set_error(GTM_ERR_WORKSPACE, "gtm_moe_tokens: workspace needs %zu bytes", w.W.total);
    launch_views(dims, L, io, w, st);
    Plan pl;
    pl.n = (int)(T * TOPK); pl.src_div = TOPK; pl.idx = w.p<uint32_t>(w.W.idx); pl.w = w.p<float>(w.W.w); pl.stride = 1;
    pl.e0 = 0; pl.ne = NE; pl.t_shared = (int)T; pl.src_rows = w.p<float>(w.W.routed); pl.out_index = nullptr;
    pl.out_r = w.p<float>(w.W.out_r);
    const int rc = run_gemms(L, w, pl, num_sms, st);
    if (rc) return rc;
    launch_combine(dims, L, io, w, w.p<int>(w.W.pos), pl.out_r, st);
    return finish("gtm_moe_tokens", &io, &w, st);
}

// ---- expert parallelism ----------------------------------------------------------------------
// Every phase of a rank lays the workspace out from (max_tokens, max_recv_rows) of its config, so
// the regions that carry data from one phase to the next (views, dispatch tables, shared-expert
// output) are the same in all of them.
static Ws ep_ws(const GtmEpConfig& ep, void* ws) {
    return Ws{ws_layout(ep.max_tokens, ep.max_recv_rows, true), static_cast<uint8_t*>(ws)};
}

int launch_ep_dispatch(const GtmDims& dims, const GtmLayer& L, const GtmTokensIO& io, const GtmEpConfig& ep,
                       float* send_rows, GtmEpMeta* send_meta, int32_t* send_counts, void* ws, cudaStream_t st) {
    const uint32_t T = io.num_tokens;
    const Ws w = ep_ws(ep, ws);
    launch_views(dims, L, io, w, st);
    DispatchArgs da;
    da.n = (int)(T * TOPK); da.world = (int)ep.world; da.epr = NE / (int)ep.world;
    da.idx = w.p<uint32_t>(w.W.idx); da.w = w.p<float>(w.W.w);
    da.send_counts = send_counts; da.send_pos = w.p<int>(w.W.send_pos); da.send_src = w.p<int>(w.W.send_src);
    da.send_meta = send_meta;
    tok_dispatch<<<1, 1024, 0, st>>>(da);
    tok_copy_rows<<<T * TOPK, 256, 0, st>>>(w.p<float>(w.W.routed), da.send_src, send_rows);
    return finish("gtm_moe_ep_dispatch", &io, &w, st);
}

int launch_ep_shared(const GtmLayer& L, const GtmTokensIO& io, const GtmEpConfig& ep, void* ws, cudaStream_t st,
                     int num_sms) {
    const Ws w = ep_ws(ep, ws);
    Plan pl;
    memset(&pl, 0, sizeof(pl));
    pl.n = 0; pl.src_div = 1; pl.idx = w.p<uint32_t>(w.W.idx); pl.w = w.p<float>(w.W.w); pl.stride = 1;
    pl.e0 = 0; pl.ne = 0; pl.t_shared = (int)io.num_tokens;
    const int rc = run_gemms(L, w, pl, num_sms, st);
    if (rc) return rc;
    return finish("gtm_moe_ep_shared", nullptr, nullptr, st);
}

int launch_ep_experts(const GtmLayer& L, const GtmEpConfig& ep, const float* recv_rows, const GtmEpMeta* recv_meta,
                      uint32_t n_recv, float* ret_rows, void* ws, cudaStream_t st, int num_sms) {
    if (n_recv == 0) return GTM_OK;
    const Ws w = ep_ws(ep, ws);
    const int epr = NE / (int)ep.world;
    Plan pl;
    pl.n = (int)n_recv; pl.src_div = 1;
    pl.idx = &recv_meta->expert; pl.w = &recv_meta->weight; pl.stride = 2;
    pl.e0 = (int)ep.rank * epr; pl.ne = epr; pl.t_shared = 0;
    pl.src_rows = recv_rows; pl.out_index = w.p<int>(w.W.perm_src); pl.out_r = ret_rows;
    const int rc = run_gemms(L, w, pl, num_sms, st);
    if (rc) return rc;
    return finish("gtm_moe_ep_experts", nullptr, nullptr, st);
}

int launch_ep_combine(const GtmDims& dims, const GtmLayer& L, const GtmTokensIO& io, const GtmEpConfig& ep,
                      const float* ret_rows, void* ws, cudaStream_t st) {
    const Ws w = ep_ws(ep, ws);
    launch_combine(dims, L, io, w, w.p<int>(w.W.send_pos), ret_rows, st);
    return finish("gtm_moe_ep_combine", nullptr, nullptr, st);
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

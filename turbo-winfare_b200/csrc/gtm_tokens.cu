// MoE block for T > 1 tokens (batched decode, prefill) on sm_100a.
//
// The reference runs every token through the per-expert GEMV chain one at a time
// (src/runner.cpp:845-854 for prefill, :612-657 per expert). Here the T tokens of a layer are
// grouped by expert and the expert products become dense contractions on the tcgen05 tensor
// cores:
//   1. tok_views_router   per token: views (exact RMS), router logits in the reference's exact
//                         order (or caller-given routing logits), optional logit bias, top-8
//   2. tok_route_*        counts per expert, token-slot rows grouped by expert (in entry order),
//                         GEMM tile lists
//   3. grouped_gemm<0>    gate/up of the routed experts and the shared expert, GeGLU fused,
//                         activations written as fp16 high/low parts; the routed tiles gather
//                         their token rows from the per-token routed views themselves
//   4. grouped_gemm<1>    down projections
//   5. tok_combine        h2 = routing-weighted sum over the 8 slots in router order, shared
//                         output, layer tail
//
// Grouped GEMM: one CTA per SM, persistent over a tile list built on the device. A tile is 256
// weight rows (two M=128 row blocks, one tensor-memory lane per row) by up to 128 tokens of one
// expert (MMA N), over K in blocks of 64 (one quantisation group): D[row][token] += W[row][k]
// X[token][k]. Both row blocks share each activation stage, which halves the activation bytes per
// MMA against 128-row tiles: at 128 tokens the activation (high + low part) is 32 KB per K block,
// and streaming it per 128 weight rows would need about the whole L2-to-SM bandwidth of an SM. A
// gate/up tile holds 128 features (row block b: features 64b..64b+63; in each 32-lane quarter,
// lanes 0-15 the gate rows and lanes 16-31 the up rows of the same 16 features, so GeGLU needs
// one shuffle). Tensor memory (512 columns): three accumulator slots of 128 columns that the row
// blocks rotate through (row block b of tile n in slot (2n + b) % 3) and two weight stages of
// 2 x 32 columns. On B200 a 128 x N x 16 MMA costs ~62 cycles for any N up to
// ~128 (measured), so N = 128 is the narrowest tile that keeps the tensor pipe busy. Warp roles:
//   * warp 0 loads the activation tile per K block, the fp16 high part and the fp16 low part
//     (x - hi), so the MMAs against the same weights carry ~22 bits of the activation: by TMA
//     from the dense tensors, or, for the gate/up of routed experts, gathered row by row from the
//     per-token routed views with cp.async (no expert-ordered copy of the rows is materialised);
//   * warp 2 loads the tile's 256 packed int4 rows per K block by TMA (rows of 32 bytes, 32-byte
//     swizzle);
//   * warps 12-19, one thread per weight row, dequantise to fp16 w = q * scale + bias (exact in
//     fp16 when the bias is a small multiple of the scale, as for zero-point-8 weights) and store
//     the block straight into the row's tensor-memory lane;
//   * warp 1 issues tcgen05.mma (kind::f16, M=128, N=16..128, K=16, A from tensor memory, B from
//     shared memory) with the whole warp converged and one elected lane issuing;
//   * warps 4-11 (two per lane quarter, alternate 32-token chunks) drain row block 0's slot and
//     release it, then row block 1's: the next tile's row block 0 already has the third slot,
//     and its row block 1 waits only for the first half of the drain.
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
constexpr int MW = 256;                 // weight rows per tile: two M=128 row blocks
constexpr int NT = 128;                 // tokens per tile (MMA N, at most)
constexpr int SX = 4;                   // activation stages (shared memory, high + low part each)
// Packed-weight stages (shared memory). A TMA weight load takes ~4,800 cycles from issue to the
// dequant warps under load (clock stamps at 64 and 4096 tokens), so the weight ring is the deeper
// one; activations are ready ~8,000 cycles before the MMA with 6 stages, so 4 suffice (3 starve it).
constexpr int RS = 12;
constexpr int SW = 2;                   // dequantised-weight stages (tensor memory, 2 x 32 columns each)
constexpr int NSLOT = 3;                // accumulator slots of NT columns; row blocks rotate through them
constexpr uint32_t A_COL0 = NSLOT * NT; // first tensor-memory column of the weight stages
constexpr int THREADS = 640;            // 20 warps; roles in grouped_gemm
constexpr int EPI0 = 128, EPI_THREADS = 256;  // epilogue: warps 4..11, two per tensor-memory lane quarter
constexpr int DQ0 = 384, DQ_THREADS = 256;    // dequant: warps 12..19, one thread per weight row
constexpr uint32_t X_TILE = NT * BK * 2;      // 16 KB per activation part
constexpr uint32_t XBOX = 32 * BK * 2;        // 4 KB: one TMA box of 32 token rows
// TMA moves a few large boxes faster than many small ones (~64 cycles a box on top of the bytes,
// measured): tiles of more than 64 tokens load each activation part as one 128-row box.
constexpr int XWIDE_MIN = 65;
// Tiles of at most 64 tokens stack the high and low activation parts as rows of one B operand
// (high rows, then low rows, each rounded up to 32), so one MMA per K step and row block covers
// both; the epilogue adds the two column ranges. A 128 x N x 16 MMA costs ~62 cycles for any
// N <= 128, so this halves the tensor time of small tiles.
constexpr int STACK_MAX = 64;
__device__ __forceinline__ int stacked_hi_rows(int rows) { return rows <= STACK_MAX ? ((rows + 31) >> 5) * 32 : 0; }
constexpr uint32_t RAW_TILE = MW * BK / 2;    // 8 KB packed int4 per K block, rows of 32 bytes
constexpr size_t SMEM_BYTES = 1024 + 2 * SX * X_TILE + RS * RAW_TILE + (2 * SX + 2 * RS + 2 * SW + 1 + NSLOT) * 8 + 16;
static_assert(A_COL0 + SW * 64 <= 512, "tensor memory columns");
constexpr int FB0_R = (FE + 127) / 128, FB0_S = (FS + 127) / 128;   // gate/up tiles: 128 features (gate + up)
constexpr int FB1 = D / MW;                                         // down tiles: 256 output rows
constexpr uint64_t kWaitNs = 1000000000ull;
constexpr int RIN_PITCH = 68;   // router input per group of 64, padded: 16-byte rows, float4 reads
constexpr int kMaxPeers = 8;   // ranks of a peer-memory expert-parallel group (NVLink domain of one box)
static_assert(kMaxPeers == GTM_EP_PEER_MAX_WORLD, "peer group size");

static_assert(SMEM_BYTES <= 232448, "grouped GEMM shared memory");
static_assert(FE % 64 == 0 && FS % 64 == 0 && D % MW == 0, "tile shapes");

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
    __half* routed_hl;           // [T][2][D] routed view: fp16 high part, then low part (K-permuted)
    uint32_t* idx;               // [T][8]
    float* w;                    // [T][8]
    float* logits_out;           // [T][E] or null
    // peer-memory expert parallelism: this rank's slots in every rank's workspace (null: own
    // rank, or not expert parallel). Every rank gets each token's top-8 ids; the routed view
    // goes only to the ranks that own one of the token's experts (epr experts per rank).
    uint32_t* push_idx[kMaxPeers];
    __half* push_views[kMaxPeers];
    int npeers, epr;
};

// Top-8 of one token's 128 logits by (value desc, index asc), softmax over the 8 times the
// per-expert scale (src/cpu_reference.cpp:447-480). One warp; lane holds experts lane + 32 j
// (`raw`: before the logit bias). Writes the token's ids and weights (and its biased logits when
// asked); lane k < 8 returns the k-th id.
__device__ __forceinline__ int route_top8(const ViewsArgs& A, int t, const float (&raw)[4]) {
    const GtmLayer& L = A.L;
    const int lane = threadIdx.x & 31;
    uint32_t key[4];
    bool taken[4] = {false, false, false, false};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int e = lane + 32 * j;
        const float v = A.logit_bias ? __fadd_rn(raw[j], A.logit_bias[e]) : raw[j];
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
    return my_idx;
}

// Views of one token when the routing logits are given (by the caller, or by tok_router_rows), no
// peer takes the rows (no staging for pushes) and x is 16-byte aligned: 128 threads, each holding three 8-element chunks of x in
// registers; the RMS is the same certified double sum as exact_rms_inv (bit-identical result in
// any summation order, sequential recomputation when too close to a rounding midpoint); the four
// fp16 views of a chunk go out as one 16-byte store each (kperm permutes inside 8 elements). Same
// arithmetic, element for element, as tok_views_router.
constexpr int VG_THREADS = 128, VG_CH = (D / 8 + VG_THREADS - 1) / VG_THREADS;
// Elements 8c .. 8c+7 of a bf16 vector as floats: one 16-byte load when p is 16-byte aligned.
__device__ __forceinline__ void ld8_bf16(const uint16_t* p, int c, float (&w)[8]) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        const uint4 g = __ldg(reinterpret_cast<const uint4*>(p) + c);
        const uint32_t v[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            w[2 * k] = __uint_as_float(v[k] << 16);
            w[2 * k + 1] = __uint_as_float(v[k] & 0xFFFF0000u);
        }
    } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) w[e] = bf16f(p[8 * c + e]);
    }
}
__global__ void __launch_bounds__(VG_THREADS) tok_views_given(const __grid_constant__ ViewsArgs A) {
    __shared__ double red[VG_THREADS / 32 + 1];
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const GtmLayer& L = A.L;
    float x[VG_CH][8];
    double acc = 0.0;
#pragma unroll
    for (int c = 0; c < VG_CH; ++c) {
        const int ch = tid + c * VG_THREADS;
        if (ch < D / 8) {
            if (A.x_f32) {
                const float4* p4 = reinterpret_cast<const float4*>(A.x_f32 + (size_t)t * D + 8 * ch);
                const float4 a = p4[0], b = p4[1];
                x[c][0] = a.x; x[c][1] = a.y; x[c][2] = a.z; x[c][3] = a.w;
                x[c][4] = b.x; x[c][5] = b.y; x[c][6] = b.z; x[c][7] = b.w;
            } else {
                const uint4 q = *reinterpret_cast<const uint4*>(A.x_bf16 + (size_t)t * D + 8 * ch);
                const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    x[c][2 * k] = __uint_as_float(wv[k] << 16);
                    x[c][2 * k + 1] = __uint_as_float(wv[k] & 0xFFFF0000u);
                }
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) acc = __dadd_rn(acc, __dmul_rn((double)x[c][e], (double)x[c][e]));
        }
    }
    acc = warp_sum_d(acc);
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (tid == 0) {
        double sm = 0.0;
        for (int w = 0; w < VG_THREADS / 32; ++w) sm = __dadd_rn(sm, red[w]);
        const double q = __ddiv_rn(sm, (double)D);
        float f = __double2float_rn(q);
        const double fd = (double)f;
        const double lo = (fd + (double)nextafterf(f, -INFINITY)) * 0.5;
        const double hi = (fd + (double)nextafterf(f, INFINITY)) * 0.5;
        const double bound = q * ((double)D + 48.0) * 1.1102230246251565e-16;   // (n + 48) 2^-53
        if (!(q - lo > bound && hi - q > bound)) {   // too close to call: the sequential sum
            double seq = 0.0;
            for (int i = 0; i < D; ++i) {
                const double v = A.x_f32 ? (double)A.x_f32[(size_t)t * D + i] : (double)bf16f(A.x_bf16[(size_t)t * D + i]);
                seq = __dadd_rn(seq, __dmul_rn(v, v));
            }
            f = __double2float_rn(__ddiv_rn(seq, (double)D));
        }
        red[VG_THREADS / 32] = (double)__fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(f, A.eps)));
    }
    __syncthreads();
    const float inv = (float)red[VG_THREADS / 32];
    const uint16_t* w_pre = rp16(L.resident_dev, L.pre_ffn_norm);
    const uint16_t* w_pre2 = rp16(L.resident_dev, L.pre_ffn_norm_2);
#pragma unroll
    for (int c = 0; c < VG_CH; ++c) {
        const int ch = tid + c * VG_THREADS;
        if (ch >= D / 8) continue;
        const int i0 = 8 * ch;
        float wp[8], wp2[8];
        ld8_bf16(w_pre, ch, wp);
        ld8_bf16(w_pre2, ch, wp2);
        uint16_t dh[8], dl[8], rh[8], rl[8];   // at positions kperm(i) - i0
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int pe = kperm(e);
            const float h = __fmul_rn(x[c][e], inv);
            const float dx = __fmul_rn(h, wp[e]);
            const __half hi = __float2half_rn(dx);
            dh[pe] = __half_as_ushort(hi);
            dl[pe] = __half_as_ushort(__float2half_rn(dx - __half2float(hi)));
            const float rx = __fmul_rn(h, wp2[e]);
            const __half r = __float2half_rn(rx);
            rh[pe] = __half_as_ushort(r);
            rl[pe] = __half_as_ushort(__float2half_rn(rx - __half2float(r)));
        }
        auto pack = [](const uint16_t (&v)[8]) {
            return make_uint4(v[0] | ((uint32_t)v[1] << 16), v[2] | ((uint32_t)v[3] << 16), v[4] | ((uint32_t)v[5] << 16),
                              v[6] | ((uint32_t)v[7] << 16));
        };
        *reinterpret_cast<uint4*>(A.dense_hi + (size_t)t * D + i0) = pack(dh);
        *reinterpret_cast<uint4*>(A.dense_lo + (size_t)t * D + i0) = pack(dl);
        *reinterpret_cast<uint4*>(A.routed_hl + (size_t)t * 2 * D + i0) = pack(rh);
        *reinterpret_cast<uint4*>(A.routed_hl + (size_t)t * 2 * D + D + i0) = pack(rl);
    }
    if (warp == 0) {
        float raw[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) raw[j] = A.route_logits[(size_t)t * NE + lane + 32 * j];
        route_top8(A, t, raw);
    }
}

// Router logits of token blockIdx.x, rows 16 blockIdx.y .. + 15, in src/cpu_reference.cpp:86-106's
// order (per row and group the 64 products summed in element order, the group's scale times that
// plus its bias times the group's input sum, the 44 group terms summed in group order): the same
// arithmetic as the router rows of tok_views_router, one round of 16 rows x 44 groups; the serial
// sums read their operands four at a time. Every CTA of a token recomputes the token's exact RMS
// and router input (2816 elements, against its 45 KB of router rows; measured, 8-row CTAs were
// slower). The logits go to `rlog` (before the logit bias) for tok_views_given.
constexpr int RR_ROWS = 16, RR_THREADS = RR_ROWS * GD;   // 704
__global__ void __launch_bounds__(RR_THREADS) tok_router_rows(const __grid_constant__ ViewsArgs A, float* rlog) {
    __shared__ __align__(16) float sx[D];
    __shared__ __align__(16) float srin[GD * RIN_PITCH];
    __shared__ float xsum[GD];
    __shared__ __align__(16) float terms[RR_ROWS][GD];
    __shared__ double red[40];
    const int t = blockIdx.x, tid = threadIdx.x;
    const GtmLayer& L = A.L;
    for (int i = tid; i < D; i += RR_THREADS)
        sx[i] = A.x_f32 ? A.x_f32[(size_t)t * D + i] : bf16f(A.x_bf16[(size_t)t * D + i]);
    __syncthreads();
    const float inv = exact_rms_inv(sx, D, A.eps, red);
    const uint16_t* rs = rp16(L.resident_dev, L.router_scale);
    for (int i = tid; i < D; i += RR_THREADS)
        srin[(i >> 6) * RIN_PITCH + (i & 63)] = __fmul_rn(__fmul_rn(__fmul_rn(sx[i], inv), bf16f(rs[i])), A.inv_sqrt_d);
    __syncthreads();
    if (tid < GD) {
        const float4* s4 = reinterpret_cast<const float4*>(srin + tid * RIN_PITCH);
        float sm = 0.0f;
#pragma unroll
        for (int k = 0; k < kGroup / 4; ++k) {
            const float4 v = s4[k];
            sm = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sm, v.x), v.y), v.z), v.w);
        }
        xsum[tid] = sm;
    }
    __syncthreads();
    const int rr = tid / GD, g = tid - rr * GD, row = blockIdx.y * RR_ROWS + rr;
    const uint8_t* W = static_cast<const uint8_t*>(L.resident_dev) + L.router.weight;
    const uint4* wg = reinterpret_cast<const uint4*>(W + (size_t)row * D + g * kGroup);
    const float4* x4 = reinterpret_cast<const float4*>(srin + g * RIN_PITCH);
    float dot = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 q = ldg_stream_u4(wg + i);
        const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float4 xv = x4[i * 4 + c];
            const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const float wf = __uint_as_float(__byte_perm(wv[c], 0x4B000000u, 0x7540u | (uint32_t)b)) - 8388608.0f;
                dot = __fadd_rn(dot, __fmul_rn(wf, xs[b]));
            }
        }
    }
    const uint16_t* Sc = rp16(L.resident_dev, L.router.scales);
    const uint16_t* Bi = rp16(L.resident_dev, L.router.biases);
    terms[rr][g] = __fadd_rn(__fmul_rn(bf16f(Sc[row * GD + g]), dot), __fmul_rn(bf16f(Bi[row * GD + g]), xsum[g]));
    __syncthreads();
    if (tid < RR_ROWS) {
        const float4* t4 = reinterpret_cast<const float4*>(&terms[tid][0]);
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < GD / 4; ++k) {
            const float4 v = t4[k];
            acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, v.x), v.y), v.z), v.w);
        }
        rlog[(size_t)t * NE + blockIdx.y * RR_ROWS + tid] = acc;
    }
}

// 512 threads a token when the routing logits are given; 1024 when the router GEMV runs, so that
// one round covers 23 router rows (44 threads a row) instead of 11.
constexpr int VIEWS_RR_MAX = 1024 / GD;
__global__ void __launch_bounds__(1024) tok_views_router(const __grid_constant__ ViewsArgs A) {
    __shared__ __align__(16) float sx[D];
    __shared__ __align__(16) __half srh[2 * D];   // routed view (high row, low row), K-permuted
    __shared__ uint32_t sdest;                    // peer mode: ranks owning one of the token's experts
    __shared__ __align__(16) float srin[GD * RIN_PITCH];
    __shared__ float xsum[GD];
    __shared__ float slog[NE];
    __shared__ double red[40];
    __shared__ float terms[VIEWS_RR_MAX][GD];
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
        const float rx = __fmul_rn(h, bf16f(w_pre2[i]));
        const __half rh = __float2half_rn(rx);
        srh[kperm(i)] = rh;
        srh[D + kperm(i)] = __float2half_rn(rx - __half2float(rh));
        srin[(i >> 6) * RIN_PITCH + (i & 63)] = __fmul_rn(__fmul_rn(h, bf16f(rs[i])), A.inv_sqrt_d);
    }
    __syncthreads();
    {
        const uint4* s4 = reinterpret_cast<const uint4*>(srh);
        uint4* d4 = reinterpret_cast<uint4*>(A.routed_hl + (size_t)t * 2 * D);
        for (int c = tid; c < 2 * D / 8; c += blockDim.x) d4[c] = s4[c];
    }
    if (A.route_logits) {
        for (int e = tid; e < NE; e += blockDim.x) slog[e] = A.route_logits[(size_t)t * NE + e];
    } else {
        // logits in src/cpu_reference.cpp:86-106's order: RR rows at a time, 44 threads a row. A
        // group's x-sum is the same for every row: summed once, in the same element order. Bytes
        // become floats exactly as 0x4B0000bb - 2^23 (no conversion unit).
        const int RR = (int)blockDim.x / GD;
        if (tid < GD) {
            float sm = 0.0f;
            for (int k = 0; k < kGroup; ++k) sm = __fadd_rn(sm, srin[tid * RIN_PITCH + k]);
            xsum[tid] = sm;
        }
        __syncthreads();
        const uint8_t* W = static_cast<const uint8_t*>(L.resident_dev) + L.router.weight;
        const uint16_t* Sc = rp16(L.resident_dev, L.router.scales);
        const uint16_t* Bi = rp16(L.resident_dev, L.router.biases);
        for (int r0 = 0; r0 < NE; r0 += RR) {
            const int rr = tid / GD, g = tid - rr * GD, row = r0 + rr;
            if (rr < RR && row < NE) {
                const uint4* wg = reinterpret_cast<const uint4*>(W + (size_t)row * D + g * kGroup);
                const float4* x4 = reinterpret_cast<const float4*>(srin + g * RIN_PITCH);
                float dot = 0.0f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint4 q = ldg_stream_u4(wg + i);
                    const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const float4 xv = x4[i * 4 + c];
                        const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const float wf = __uint_as_float(__byte_perm(wv[c], 0x4B000000u, 0x7540u | (uint32_t)b)) - 8388608.0f;
                            dot = __fadd_rn(dot, __fmul_rn(wf, xs[b]));
                        }
                    }
                }
                terms[rr][g] = __fadd_rn(__fmul_rn(bf16f(Sc[row * GD + g]), dot), __fmul_rn(bf16f(Bi[row * GD + g]), xsum[g]));
            }
            __syncthreads();
            if (tid < RR && r0 + tid < NE) {
                float acc = 0.0f;
                for (int g2 = 0; g2 < GD; ++g2) acc = __fadd_rn(acc, terms[tid][g2]);
                slog[r0 + tid] = acc;
            }
            __syncthreads();
        }
    }
    __syncthreads();
    if (tid < 32) {
        float raw[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) raw[j] = slog[tid + 32 * j];
        const int my_idx = route_top8(A, t, raw);
        if (A.npeers > 0) {
            const uint32_t dest = __reduce_or_sync(0xffffffffu, tid < TOPK ? 1u << (my_idx / A.epr) : 0u);
            if (tid == 0) sdest = dest;
            for (int s = 0; s < A.npeers; ++s)
                if (A.push_idx[s] && tid < TOPK) A.push_idx[s][(size_t)t * TOPK + tid] = (uint32_t)my_idx;
        }
    }
    if (A.npeers > 0) {
        // the routed view to each peer that owns one of the token's experts: 16-byte NVLink stores
        __syncthreads();
        const uint32_t dest = sdest;
        const uint4* s4 = reinterpret_cast<const uint4*>(srh);
        for (int s = 0; s < A.npeers; ++s) {
            if (!A.push_views[s] || !((dest >> s) & 1u)) continue;
            uint4* d4 = reinterpret_cast<uint4*>(A.push_views[s] + (size_t)t * 2 * D);
            for (int c = tid; c < 2 * D / 8; c += blockDim.x) d4[c] = s4[c];
        }
    }
}

// ================================================================================================
// 2. routing tables and tile lists
// ================================================================================================

struct RouteArgs {
    int n;                   // routed entries (0: shared tiles only)
    int src_div;             // activation source row of entry i = i / src_div
    const uint32_t* idx;     // expert id of entry i at idx[i * stride]
    int stride;
    int e0, ne;              // experts of this launch: [e0, e0 + ne); tiles carry e - e0
    int t_shared;            // tokens of the shared-expert tiles (0: none)
    int nchunks;             // ceil(n / RC)
    // peer-memory expert parallelism: entry i is entry i % per_src of source rank i / per_src,
    // read from that rank's workspace (src_idx), valid below 8 x its token count (src_ntok)
    int nsrc, per_src;
    const uint32_t* src_idx[kMaxPeers];
    const int* src_ntok[kMaxPeers];
    int* nrows;              // peer mode: rows through this launch's experts (for the gather)
    int* chunk;              // [nchunks][NE]: per-chunk counts, then each chunk's first row per expert
    int* perm_src;           // [n] source row of each expert-ordered row
    int* pos;                // [n] expert-ordered row of each entry (-1: another rank's expert)
    Tile* tiles0;            // gate/up tiles
    Tile* tiles1;            // down tiles
    int* n_tiles;            // [2]
};

__device__ __forceinline__ int ntok_tiles(int c) { return (c + NT - 1) / NT; }

// Expert id of entry i (-1: not one of this launch's experts, or past its source's tokens).
__device__ __forceinline__ int route_expert(const RouteArgs& A, int i) {
    if (i >= A.n) return -1;
    int e;
    if (A.nsrc > 0) {
        const int s = i / A.per_src, j = i - s * A.per_src;
        if (j >= *A.src_ntok[s] * TOPK) return -1;
        e = (int)A.src_idx[s][j] - A.e0;
    } else {
        e = (int)A.idx[(size_t)i * A.stride] - A.e0;
    }
    return (e >= 0 && e < A.ne) ? e : -1;
}

// Routing tables in three steps. Rows of one expert keep the entries' order, so the layout is the
// same on every run: an entry's row = its expert's first row + the entries of that expert in
// earlier chunks + those before it in its own chunk.
constexpr int RC = 1024;   // entries per counting CTA

// 2a. per-chunk counts and in-chunk ranks (warp match_any, then a prefix over the warps)
__device__ __forceinline__ void route_count(const RouteArgs& A, int chunk) {
    __shared__ int wc[RC / 32][NE];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int j = tid; j < (RC / 32) * NE; j += RC) (&wc[0][0])[j] = 0;
    __syncthreads();
    const int i = chunk * RC + tid;
    const int e = route_expert(A, i);   // -1: another rank's expert (or no entry)
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank_w = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && rank_w == 0) wc[warp][e] = __popc(peers);
    __syncthreads();
    for (int ex = tid; ex < A.ne; ex += RC) {
        int run = 0;
        for (int w = 0; w < RC / 32; ++w) { const int c = wc[w][ex]; wc[w][ex] = run; run += c; }
        A.chunk[(size_t)chunk * NE + ex] = run;
    }
    __syncthreads();
    if (i < A.n) A.pos[i] = e >= 0 ? wc[warp][e] + rank_w : -1;
}
__global__ void __launch_bounds__(RC) tok_route_count(const __grid_constant__ RouteArgs A) { route_count(A, blockIdx.x); }

// 2b. expert offsets, each chunk's first row per expert, and the tile lists (one CTA)
__device__ __forceinline__ void route_scan(const RouteArgs& A) {
    constexpr int SP = 8;   // threads per expert in the chunk scan (1024 / NE)
    __shared__ int cnt[NE], off[NE + 1], t0[NE + 1], t1[NE + 1];
    __shared__ int wsum[NE / 32][3];
    const int tid = threadIdx.x, lane = tid & 31;
    // (1) per expert, the total and each of the SP threads' exclusive prefix of its per-chunk counts:
    //     SP adjacent lanes per expert, each a contiguous run of chunks, combined by shuffles
    const int se = tid / SP, sp = tid % SP;
    const int per = (A.nchunks + SP - 1) / SP, sc0 = sp * per, sc1 = min(A.nchunks, sc0 + per);
    int srun;
    {
        int local = 0;
        if (se < A.ne)
            for (int c = sc0; c < sc1; ++c) local += A.chunk[(size_t)c * NE + se];
        int incl = local;
#pragma unroll
        for (int o = 1; o < SP; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o, SP);
            if (sp >= o) incl += v;
        }
        srun = incl - local;
        const int total = __shfl_sync(0xffffffffu, incl, SP - 1, SP);
        if (se < A.ne && sp == 0) cnt[se] = total;
    }
    __syncthreads();
    // (2) expert offsets and tile-list bases: a block scan over the experts
    if (tid < NE) {
        const int c = tid < A.ne ? cnt[tid] : 0, nt = ntok_tiles(c);
        int v0 = c, v1 = nt * FB0_R, v2 = nt * FB1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a0 = __shfl_up_sync(0xffffffffu, v0, o), a1 = __shfl_up_sync(0xffffffffu, v1, o),
                      a2 = __shfl_up_sync(0xffffffffu, v2, o);
            if (lane >= o) { v0 += a0; v1 += a1; v2 += a2; }
        }
        if (lane == 31) { wsum[tid >> 5][0] = v0; wsum[tid >> 5][1] = v1; wsum[tid >> 5][2] = v2; }
        cnt[tid] = c;
        off[tid + 1] = v0; t0[tid + 1] = v1; t1[tid + 1] = v2;   // inclusive within the warp
    }
    __syncthreads();
    if (tid < NE) {
        int b0 = 0, b1 = 0, b2 = 0;
        for (int w = 0; w < (tid >> 5); ++w) { b0 += wsum[w][0]; b1 += wsum[w][1]; b2 += wsum[w][2]; }
        off[tid + 1] += b0; t0[tid + 1] += b1; t1[tid + 1] += b2;
    }
    if (tid == 0) { off[0] = 0; t0[0] = 0; t1[0] = 0; }
    __syncthreads();
    if (tid == 0 && A.nrows) *A.nrows = off[A.ne];
    // each chunk's first row per expert: the expert's offset plus the chunks before it (the same
    // threads as in (1), which read these counts)
    if (se < A.ne) {
        int run = off[se] + srun;
        for (int c = sc0; c < sc1; ++c) {
            const int v = A.chunk[(size_t)c * NE + se];
            A.chunk[(size_t)c * NE + se] = run;
            run += v;
        }
    }
    // (3) routed tiles, a warp per expert: entry t0[e] + f * nt + m of expert e covers token range
    //     m of nt and row block f, so the tiles of one (expert, row block) stay adjacent over the token
    //     ranges (L2 reuse of the weights)
    for (int e = tid >> 5; e < A.ne; e += blockDim.x >> 5) {
        const int c = cnt[e], nt = ntok_tiles(c);
        for (int k = lane; k < nt * FB0_R; k += 32) {
            const int f = k / nt, m = k - f * nt, r0 = c * m / nt, r1 = c * (m + 1) / nt;
            A.tiles0[t0[e] + k] = Tile{e, off[e] + r0, r1 - r0, f};
        }
        for (int k = lane; k < nt * FB1; k += 32) {
            const int f = k / nt, m = k - f * nt, r0 = c * m / nt, r1 = c * (m + 1) / nt;
            A.tiles1[t1[e] + k] = Tile{e, off[e] + r0, r1 - r0, f};
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
__global__ void __launch_bounds__(1024) tok_route_scan(const __grid_constant__ RouteArgs A) { route_scan(A); }

// 2c. final rows: pos = expert-ordered row of each entry, perm_src = its source row
__device__ __forceinline__ void route_scatter(const RouteArgs& A, int chunk) {
    const int i = chunk * RC + threadIdx.x;
    if (i >= A.n) return;
    const int r = A.pos[i];
    if (r < 0) return;
    const int e = route_expert(A, i);
    const int row = A.chunk[(size_t)chunk * NE + e] + r;
    A.pos[i] = row;
    A.perm_src[row] = i / A.src_div;
}
__global__ void __launch_bounds__(RC) tok_route_scatter(const __grid_constant__ RouteArgs A) { route_scatter(A, blockIdx.x); }

// At most one chunk (up to RC entries: up to 128 tokens on one GPU): the three steps in one CTA.
// A thread's global writes are visible to the CTA's other threads after __syncthreads.
__global__ void __launch_bounds__(RC) tok_route_one(const __grid_constant__ RouteArgs A) {
    if (A.nchunks > 0) route_count(A, 0);
    __syncthreads();
    route_scan(A);
    __syncthreads();
    if (A.nchunks > 0) route_scatter(A, 0);
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

// Peer mode: this rank's token count into its slot of every rank's header.
struct CountArgs { int* dst[kMaxPeers]; int n, v; };
__global__ void tok_set_count(const __grid_constant__ CountArgs A) {
    for (int s = 0; s < A.n; ++s) *A.dst[s] = A.v;
}

// ================================================================================================
// 4/5. grouped GEMM
// ================================================================================================
struct GemmArgs {
    CUtensorMap x_rhi, x_rlo, x_shi, x_slo;   // activations: 2D fp16, 32-row boxes, 128-byte swizzle
    CUtensorMap y_rhi, y_rlo, y_shi, y_slo;   // the same tensors in 128-row boxes (tiles of > 64 tokens)
                                              // (mode 0 routed tiles gather instead, see act_src)
    CUtensorMap w_ra, w_rb, w_sa, w_sb;       // packed int4 weights (matrix a, b): routed 3D (byte, row,
                                              // expert), shared 2D; rows of 32 bytes, 32-byte swizzle
    const Tile* tiles;
    const int* n_tiles;
    const uint8_t* experts;
    uint64_t expert_stride;
    uint64_t r_sa, r_ba, r_sb, r_bb;      // routed scale / bias byte offsets (matrix a, b)
    const uint8_t* resident;
    uint64_t s_sa, s_ba, s_sb, s_bb;      // shared
    int k_r, k_s;                         // K of the routed / shared matrices
    int rows_r, rows_s;                   // rows of each routed / shared matrix (mode 0: features)
    int wide_r, wide_s;                   // the 128-row box maps exist (the tensor has >= 128 rows)
    __half* act_r_hi; __half* act_r_lo;   // mode 0 outputs, rows of FE (routed) / FS (shared)
    __half* act_s_hi; __half* act_s_lo;
    float* out_r; float* out_s;           // mode 1 outputs [rows][D]
    const int* out_index;                 // mode 1: output row of each routed row (null: same row)
    // mode 1, peer-memory expert parallelism (per_src > 0): output row o of a routed row goes to
    // rank o / per_src's return region, row o % per_src (a peer store over NVLink)
    int per_src;
    float* out_peer[kMaxPeers];
    // mode 0 routed tiles: activation row r is routed view act_row[r] / act_div of act_src
    // ([rows][2][D] fp16, high row then low row), copied into the stage by the producer warp
    const __half* act_src;
    const int* act_row;
    int act_div;
    int* err;
    int test_wait;                        // GTM_TOKENS_TEST_WAIT_RUNS_OUT: the MMA warp's first wait never ends
};

__device__ __forceinline__ float* remap_row(const GemmArgs& A, int orow) {
    if (A.per_src > 0) {
        const int s = orow / A.per_src;
        return A.out_peer[s] + (size_t)(orow - s * A.per_src) * D;
    }
    return A.out_r + (size_t)orow * D;
}

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

// x * 0.5 * (1 + tanh(u)) written as x / (1 + exp(-2u)), u = sqrt(2/pi) (x + 0.044715 x^3): the
// same function as gelu_pytorch_tanh (cpu_reference.cpp:34-38), evaluated with one exponential.
__device__ __forceinline__ float gelu_tanh_fast(float x) {
    const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
    return __fdividef(x, 1.0f + __expf(-2.0f * u));
}

// a = hi + lo with hi, lo fp16 (~22 significant bits together), returned as one fp16x2 word (lo in
// the low half), for |a| inside the fp16 range. hi is a rounded to 11 significant bits by
// Veltkamp splitting in fp32 (exact in fp16 for |a| >= 2^-14; below that the fp16 conversion
// rounds it again, an absolute error under 2^-25), lo = a - hi is exact in fp32; one packed
// conversion then produces both halves.
__device__ __forceinline__ uint32_t split_hi_lo(float a) {
    const float c = __fmul_rn(a, 8193.0f);   // 2^13 + 1: keeps 24 - 13 = 11 bits
    const float hi = __fsub_rn(c, __fsub_rn(c, a));
    const float lo = __fsub_rn(a, hi);
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// v[u] += the accumulator column taddr + u (u < 32), loaded 16 columns at a time.
__device__ __forceinline__ void add_low_part(uint32_t taddr, uint32_t (&v)[32]) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        uint32_t w[16];
        tc::tmem_ld16_sync(taddr + 16 * h, w);
#pragma unroll
        for (int u = 0; u < 16; ++u) v[16 * h + u] = __float_as_uint(__uint_as_float(v[16 * h + u]) + __uint_as_float(w[u]));
    }
}

// Gate/up tile of 128 features f0 .. f0+127: row block b holds features f0 + 64b + (0..63); in
// each 32-lane quarter q, lanes 0-15 are the gate rows and lanes 16-31 the up rows of features
// f0 + 64b + 16q + (0..15), so GeGLU needs one shuffle. Packed rows sit in shared memory as the
// 128 gate rows, then the 128 up rows.
__device__ __forceinline__ int gu_feature(int b, int q, int lane) { return 64 * b + 16 * q + (lane & 15); }

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1) grouped_gemm(const __grid_constant__ GemmArgs A) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sXh = base;                         // [SX][16 KB]   activation high parts, 128-byte swizzle
    uint8_t* sXl = sXh + SX * X_TILE;            // [SX][16 KB]   activation low parts
    uint8_t* sRaw = sXl + SX * X_TILE;           // [RS][256][32] packed int4 rows, 32-byte swizzle
    uint64_t* bars = reinterpret_cast<uint64_t*>(sRaw + RS * RAW_TILE);
    uint64_t* act_full = bars;                   // [SX]
    uint64_t* act_empty = act_full + SX;         // [SX]
    uint64_t* raw_full = act_empty + SX;         // [RS]
    uint64_t* raw_empty = raw_full + RS;         // [RS]
    uint64_t* w_full = raw_empty + RS;           // [SW]
    uint64_t* w_empty = w_full + SW;             // [SW]
    uint64_t* acc_full = w_empty + SW;           // [1]
    uint64_t* acc_empty = acc_full + 1;          // [NSLOT] one per accumulator slot
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + NSLOT);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    __shared__ uint64_t never_bar;               // test hook: a barrier nothing arrives at
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        tc::mbar_init(&never_bar, 1);
        for (int s = 0; s < SX; ++s) { tc::mbar_init(&act_full[s], 2); tc::mbar_init(&act_empty[s], 1); }
        for (int s = 0; s < RS; ++s) { tc::mbar_init(&raw_full[s], 1); tc::mbar_init(&raw_empty[s], DQ_THREADS); }
        for (int s = 0; s < SW; ++s) { tc::mbar_init(&w_full[s], DQ_THREADS); tc::mbar_init(&w_empty[s], 1); }
        tc::mbar_init(&acc_full[0], 1);
        for (int b = 0; b < NSLOT; ++b) tc::mbar_init(&acc_empty[b], EPI_THREADS);
        *abort_flag = 0;
        tc::mbar_fence_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int ntiles = *A.n_tiles;

    if (warp == 0 || warp == 3) {
        // ---- activation producers (two arrivals per stage): per K block the tile's token rows,
        //      high and low part. Shared-expert and mode 1 tiles: warp 0 loads TMA boxes of the
        //      dense activation tensors, warp 3 only arrives. Mode 0 routed tiles: warp 0 (high
        //      part) and warp 3 (low part) gather the rows from the routed views with 16-byte
        //      cp.async copies into the 128-byte-swizzled layout TMA would produce (row r at
        //      r * 128, chunk c at c ^ (r & 7)); a warp hands its part of a stage to the MMA warp
        //      GLAG stages later, after its copies have landed and been fenced for the tensor
        //      core. The two warps sit on different schedulers ----
        constexpr int GLAG = 2;
        const int part = warp == 3 ? 1 : 0;
        uint32_t it = 0, gath = 0;   // gath bit j: stage it - 1 - j was gathered (arrive pending)
        bool ok = true;
        for (int i = blockIdx.x; i < ntiles && ok; i += gridDim.x) {
            const TileInfo ti = tile_info(A, i);
            const int rows = ti.t.rows, row0 = ti.t.row0, hrows = stacked_hi_rows(rows);
            const bool gather = MODE == 0 && ti.routed;
            // gathered tiles: source row (in views) of tile rows lane + 32 m
            int srow[NT / 32];
#pragma unroll
            for (int m = 0; m < NT / 32; ++m) {
                const int r = lane + 32 * m;
                srow[m] = gather && r < rows ? A.act_row[row0 + r] / A.act_div : 0;
            }
            const bool wide = rows >= XWIDE_MIN && (ti.routed ? A.wide_r : A.wide_s);
            const CUtensorMap* mh = wide ? (ti.routed ? &A.y_rhi : &A.y_shi) : (ti.routed ? &A.x_rhi : &A.x_shi);
            const CUtensorMap* ml = wide ? (ti.routed ? &A.y_rlo : &A.y_slo) : (ti.routed ? &A.x_rlo : &A.x_slo);
            const int nbox = wide ? 1 : (rows + 31) >> 5;
            const uint32_t box_bytes = wide ? X_TILE : XBOX;
            for (int kb = 0; kb < ti.nkb; ++kb, ++it) {
                const uint32_t s = it % SX, ph = (it / SX) & 1;
                if (!__all_sync(0xffffffffu, tc::mbar_wait(&act_empty[s], ph ^ 1, abort_flag, kWaitNs))) { ok = false; break; }
                uint8_t* hi_dst = sXh + s * X_TILE;
                // stacked tiles: low part right after the high part in the same stage
                uint8_t* lo_dst = hrows ? hi_dst + hrows * 128 : sXl + s * X_TILE;
                if (gather) {
                    const int c = lane & 7, rq = lane >> 3;
                    const uint32_t dst = tc::smem_u32(part ? lo_dst : hi_dst) + (uint32_t)rq * 128;
                    // row r & 7 = rq + 4 (jj & 1): the swizzled chunk of the two row parities
                    const uint32_t cx0 = (uint32_t)((c ^ rq) << 4), cx1 = (uint32_t)((c ^ (rq + 4)) << 4);
                    const __half* col = A.act_src + part * D + kb * BK + c * 8;
                    // rows 32 m + 4 jj + rq; lane % 8 = the row's 16-byte chunk
#pragma unroll
                    for (int m = 0; m < NT / 32; ++m) {
                        if (32 * m >= rows) break;
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj) {
                            const int rl = 4 * jj + rq;
                            const int sr = __shfl_sync(0xffffffffu, srow[m], rl);
                            if (32 * m + rl < rows)
                                tc::cp_async16(dst + (uint32_t)(32 * m + 4 * jj) * 128 + ((jj & 1) ? cx1 : cx0),
                                               col + (size_t)sr * 2 * D);
                        }
                    }
                } else if (part == 0 && lane == 0) {
                    tc::mbar_arrive_expect_tx(&act_full[s], 2u * box_bytes * (uint32_t)nbox);
                    for (int j = 0; j < nbox; ++j) {
                        tc::tma_load_2d(hi_dst + j * XBOX, mh, kb * BK, row0 + 32 * j, &act_full[s]);
                        tc::tma_load_2d(lo_dst + j * XBOX, ml, kb * BK, row0 + 32 * j, &act_full[s]);
                    }
                } else if (lane == 0) {
                    tc::mbar_arrive(&act_full[s]);
                }
                tc::cp_async_commit();
                gath = (gath << 1) | (gather ? 1u : 0u);
                if (it >= (uint32_t)GLAG) {
                    tc::cp_async_wait<GLAG>();
                    if ((gath >> GLAG) & 1u) {   // stage it - GLAG: its copies have landed
                        tc::fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive(&act_full[(it - GLAG) % SX]);
                    }
                }
            }
        }
        // hand over the stages still pending, then no exit while TMA writes into this CTA's
        // shared memory are in flight
        tc::cp_async_wait<0>();
        tc::fence_proxy_async_smem();
        __syncwarp();
        for (uint32_t j = it > (uint32_t)GLAG ? it - GLAG : 0; j < it; ++j)
            if (((gath >> (it - 1 - j)) & 1u) && lane == 0) tc::mbar_arrive(&act_full[j % SX]);
        if (part == 0 && lane == 0) {
            volatile int never = 0;
            for (uint32_t j = it > SX ? it - SX : 0; j < it; ++j)
                tc::mbar_wait(&act_full[j % SX], (j / SX) & 1, &never, kWaitNs);
        }
    } else if (warp == 2) {
        // ---- weight producer: per K block the tile's 256 packed rows (TMA, 32 bytes a row) ----
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int i = blockIdx.x; i < ntiles && ok; i += gridDim.x) {
                const TileInfo ti = tile_info(A, i);
                for (int kb = 0; kb < ti.nkb; ++kb, ++it) {
                    const uint32_t s = it % RS, ph = (it / RS) & 1;
                    if (!tc::mbar_wait(&raw_empty[s], ph ^ 1, abort_flag, kWaitNs)) { ok = false; break; }
                    tc::mbar_arrive_expect_tx(&raw_full[s], RAW_TILE);
                    uint8_t* dst = sRaw + s * RAW_TILE;
                    if (MODE == 0) {   // 128 gate rows then 128 up rows (rows past the matrix read as 0)
                        if (ti.routed) {
                            tc::tma_load_3d(dst, &A.w_ra, kb * 32, ti.t.fb * 128, ti.t.expert, &raw_full[s]);
                            tc::tma_load_3d(dst + RAW_TILE / 2, &A.w_rb, kb * 32, ti.t.fb * 128, ti.t.expert, &raw_full[s]);
                        } else {
                            tc::tma_load_2d(dst, &A.w_sa, kb * 32, ti.t.fb * 128, &raw_full[s]);
                            tc::tma_load_2d(dst + RAW_TILE / 2, &A.w_sb, kb * 32, ti.t.fb * 128, &raw_full[s]);
                        }
                    } else {
                        if (ti.routed) tc::tma_load_3d(dst, &A.w_ra, kb * 32, ti.t.fb * MW, ti.t.expert, &raw_full[s]);
                        else tc::tma_load_2d(dst, &A.w_sa, kb * 32, ti.t.fb * MW, &raw_full[s]);
                    }
                }
            }
            volatile int never = 0;
            for (uint32_t j = it > RS ? it - RS : 0; j < it; ++j)
                tc::mbar_wait(&raw_full[j % RS], (j / RS) & 1, &never, kWaitNs);
        }
    } else if (warp == 1) {
        // ---- MMA issuer (the whole warp; one elected lane issues). Per K step and row block:
        //      weights (A, tensor memory) x activation high part, then x low part (B, shared
        //      memory). Row block b of tile n accumulates in slot (2n + b) % 3, so the next
        //      tile's row block 0 finds a free slot while the epilogue drains this tile. Row
        //      block 1 of the last gate/up tile lies past the matrix: skipped. ----
        uint32_t it = 0, acc_it = 0;
        bool ok = true;
        if (A.test_wait && !__all_sync(0xffffffffu, tc::mbar_wait(&never_bar, 0, abort_flag, 2000000ull))) ok = false;
        for (int i = blockIdx.x; i < ntiles && ok; i += gridDim.x, ++acc_it) {
            const TileInfo ti = tile_info(A, i);
            const int kout = ti.routed ? A.rows_r : A.rows_s;
            const bool rb1 = MODE == 1 || ti.t.fb * 128 + 64 < kout;
            const int hrows = stacked_hi_rows(ti.t.rows);
            const uint32_t idesc = tc::idesc_f16(128, hrows ? 2u * (uint32_t)hrows : (uint32_t)((ti.t.rows + 15) & ~15));
            for (int kb = 0; kb < ti.nkb; ++kb, ++it) {
                const uint32_t sx = it % SX, phx = (it / SX) & 1, sw = it % SW, phw = (it / SW) & 1;
                if (!__all_sync(0xffffffffu, tc::mbar_wait(&w_full[sw], phw, abort_flag, kWaitNs) &&
                                                 tc::mbar_wait(&act_full[sx], phx, abort_flag, kWaitNs))) { ok = false; break; }
                tc::tc_fence_after();
                const uint64_t dh = tc::sdesc_sw128(tc::smem_u32(sXh + sx * X_TILE));
                const uint64_t dl = tc::sdesc_sw128(tc::smem_u32(sXl + sx * X_TILE));
                for (int b = 0; b < 2; ++b) {
                    const uint32_t rbg = 2 * acc_it + (uint32_t)b, slot = rbg % NSLOT;
                    if (kb == 0) {   // the epilogue has drained the slot's previous row block
                        if (!__all_sync(0xffffffffu, tc::mbar_wait(&acc_empty[slot], ((rbg / NSLOT) & 1) ^ 1, abort_flag,
                                                                   kWaitNs))) { ok = false; break; }
                        tc::tc_fence_after();
                    }
                    if (b == 1 && !rb1) break;
                    const uint32_t d = tmem + slot * NT;
                    const uint32_t wa = tmem + A_COL0 + sw * 64 + (uint32_t)b * 32;   // 8 columns per K step
                    if (hrows) {
#pragma unroll
                        for (int k = 0; k < BK / 16; ++k)
                            tc::mma_f16_ts(d, wa + 8 * k, dh + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    } else {
#pragma unroll
                        for (int k = 0; k < BK / 16; ++k) {
                            tc::mma_f16_ts(d, wa + 8 * k, dh + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                            tc::mma_f16_ts(d, wa + 8 * k, dl + 2 * k, idesc, 1u);
                        }
                    }
                }
                if (!ok) break;
                tc::mma_commit(&w_empty[sw]);
                tc::mma_commit(&act_empty[sx]);
            }
            if (!ok) break;
            tc::mma_commit(&acc_full[0]);
        }
        if (it > 0) {   // issued MMAs finish before tensor memory is released
            volatile int never = 0;
            tc::mbar_wait(&w_empty[(it - 1) % SW], ((it - 1) / SW) & 1, &never, kWaitNs);
        }
    } else if (warp >= DQ0 / 32) {
        // ---- dequant: one thread per weight row (row block b = warps 12-15 / 16-19, lane quarter
        //      warp % 4); packed bytes from the TMA stage, bf16 scale/bias loaded two blocks ahead,
        //      the block's 64 fp16 weights stored into the row's tensor-memory lane ----
        const int q = warp & 3, b = (warp - DQ0 / 32) >> 2;
        const int L = 32 * q + lane;                                   // tensor-memory lane
        const int srow = MODE == 0 ? (lane >> 4) * 128 + gu_feature(b, q, lane) : 128 * b + L;
        const uint32_t sw_bit = (uint32_t)((srow >> 2) & 1);           // 32-byte swizzle: 16-byte halves swap
        const uint32_t raw_c0 = (uint32_t)srow * 32u + (sw_bit << 4), raw_c1 = (uint32_t)srow * 32u + ((sw_bit ^ 1u) << 4);
        const uint32_t tl_addr = tmem + ((uint32_t)(32 * q) << 16) + A_COL0 + 32u * (uint32_t)b;
        uint32_t it = 0;
        bool ok = true;
        for (int i = blockIdx.x; i < ntiles && ok; i += gridDim.x) {
            const TileInfo ti = tile_info(A, i);
            const int G = ti.nkb;
            const uint8_t* wb = ti.routed ? A.experts + (uint64_t)ti.t.expert * A.expert_stride : A.resident;
            int grow, nrows;
            uint64_t so, bo;
            if (MODE == 0) {
                const bool up = lane >= 16;
                grow = ti.t.fb * 128 + gu_feature(b, q, lane);
                nrows = ti.routed ? A.rows_r : A.rows_s;
                so = ti.routed ? (up ? A.r_sb : A.r_sa) : (up ? A.s_sb : A.s_sa);
                bo = ti.routed ? (up ? A.r_bb : A.r_ba) : (up ? A.s_bb : A.s_ba);
            } else {
                grow = ti.t.fb * MW + 128 * b + L;
                nrows = D;
                so = ti.routed ? A.r_sa : A.s_sa;
                bo = ti.routed ? A.r_ba : A.s_ba;
            }
            const bool valid = grow < nrows;   // rows past the matrix dequantise to 0
            const uint16_t* sp = reinterpret_cast<const uint16_t*>(wb + so) + (size_t)(valid ? grow : 0) * G;
            const uint16_t* bp = reinterpret_cast<const uint16_t*>(wb + bo) + (size_t)(valid ? grow : 0) * G;
            auto step = [&](int kb, uint16_t sbits, uint16_t bbits) -> bool {
                const uint32_t rs = it % RS, rph = (it / RS) & 1, sw = it % SW, wph = (it / SW) & 1;
                if (!__all_sync(0xffffffffu, tc::mbar_wait(&raw_full[rs], rph, abort_flag, kWaitNs))) return false;
                const uint4 q0 = *reinterpret_cast<const uint4*>(sRaw + rs * RAW_TILE + raw_c0);
                const uint4 q1 = *reinterpret_cast<const uint4*>(sRaw + rs * RAW_TILE + raw_c1);
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
                // warp-uniform outcome: tcgen05.st is warp-collective
                if (!__all_sync(0xffffffffu, tc::mbar_wait(&w_empty[sw], wph ^ 1, abort_flag, kWaitNs))) return false;
                tc::tc_fence_after();
                tc::tmem_st32(tl_addr + sw * 64, o);
                tc::tmem_st_wait();
                tc::tc_fence_before();
                tc::mbar_arrive(&w_full[sw]);
                // The packed stage goes back to the TMA only now, after its words have been used:
                // releasing it straight after the shared-memory loads let the next TMA write land
                // before the loads had read it (measured: a few weight rows per run corrupted).
                tc::mbar_arrive(&raw_empty[rs]);
                ++it;
                return true;
            };
            // scale/bias of blocks kb, kb+1 in registers; those of kb+2, kb+3 load during two blocks' work
            uint16_t s0 = valid ? sp[0] : 0, b0 = valid ? bp[0] : 0;
            uint16_t s1 = valid && G > 1 ? sp[1] : 0, b1 = valid && G > 1 ? bp[1] : 0;
            for (int kb = 0; kb < G; kb += 2) {
                const uint16_t s2 = valid && kb + 2 < G ? sp[kb + 2] : 0, b2 = valid && kb + 2 < G ? bp[kb + 2] : 0;
                const uint16_t s3 = valid && kb + 3 < G ? sp[kb + 3] : 0, b3 = valid && kb + 3 < G ? bp[kb + 3] : 0;
                if (!step(kb, s0, b0) || (kb + 1 < G && !step(kb + 1, s1, b1))) { ok = false; break; }
                s0 = s2; b0 = b2; s1 = s3; b1 = b3;
            }
        }
    } else if (warp >= EPI0 / 32) {
        // ---- epilogue: warps 4..7 and 8..11 each cover tensor-memory lane quarter (warp % 4),
        //      taking alternate 32-token column chunks; row block 0's slot is drained and
        //      released first ----
        const int q = warp & 3, c = (warp - EPI0 / 32) >> 2;
        uint32_t acc_it = 0;
        for (int i = blockIdx.x; i < ntiles; i += gridDim.x, ++acc_it) {
            const TileInfo ti = tile_info(A, i);
            const int rows = ti.t.rows, row0 = ti.t.row0;
            // mode 1, expert parallelism: output row of token (chunk j, lane), loaded before the wait
            const bool remap = MODE == 1 && ti.routed && A.out_index != nullptr;
            float* ol[NT / 64];
#pragma unroll
            for (int j = 0; j < NT / 64; ++j) {
                const int tl = 32 * c + 64 * j + lane;
                ol[j] = remap && tl < rows ? remap_row(A, A.out_index[row0 + tl]) : nullptr;
            }
            // warp-uniform outcome: tcgen05.ld is warp-collective
            if (!__all_sync(0xffffffffu, tc::mbar_wait(&acc_full[0], acc_it & 1, abort_flag, kWaitNs))) break;
            tc::tc_fence_after();
            const int kout = ti.routed ? A.rows_r : A.rows_s;
            const int hrows = stacked_hi_rows(rows);   // stacked tile: low-part sums at column + hrows
            for (int b = 0; b < 2; ++b) {
                const uint32_t slot = (2 * acc_it + (uint32_t)b) % NSLOT;
                const uint32_t taddr = tmem + slot * NT + ((uint32_t)(32 * q) << 16);
                if (MODE == 1) {
                    // lane = output row f; per token one coalesced 128-byte store per warp
                    const int f = ti.t.fb * MW + 128 * b + 32 * q + lane;
                    float* out = (ti.routed ? A.out_r : A.out_s) + f;
#pragma unroll
                    for (int j = 0; j < NT / 64; ++j) {
                        const int c0 = 32 * c + 64 * j;
                        if (c0 >= rows) break;
                        uint32_t v[32];
                        tc::tmem_ld32_sync(taddr + c0, v);
                        if (hrows) add_low_part(taddr + hrows + c0, v);
                        if (remap) {
#pragma unroll
                            for (int u = 0; u < 32; ++u) {
                                float* orow = reinterpret_cast<float*>(
                                    __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(ol[j]), u));
                                if (c0 + u < rows) orow[f] = __uint_as_float(v[u]);
                            }
                        } else {
                            float* o = out + (size_t)(row0 + c0) * D;
#pragma unroll
                            for (int u = 0; u < 32; ++u)
                                if (c0 + u < rows) o[(size_t)u * D] = __uint_as_float(v[u]);
                        }
                    }
                } else if (ti.t.fb * 128 + 64 * b < kout) {
                    // lanes 0-15 hold gate, lanes 16-31 up of the same 16 features; one exchange
                    // gives lanes 0-15 tokens 0..15 and lanes 16-31 tokens 16..31 of each chunk
                    const int f = ti.t.fb * 128 + gu_feature(b, q, lane);
                    const bool up = lane >= 16;
                    const int fcol = kperm(f);
                    __half* oh = (ti.routed ? A.act_r_hi : A.act_s_hi) + fcol;
                    __half* olo = (ti.routed ? A.act_r_lo : A.act_s_lo) + fcol;
                    for (int c0 = 32 * c; c0 < rows; c0 += 64) {
                        uint32_t v[32];
                        tc::tmem_ld32_sync(taddr + c0, v);
                        if (hrows) add_low_part(taddr + hrows + c0, v);
                        // all 16 activations first, branch-free, so their exp/reciprocal chains
                        // overlap; the stores for tokens past the tile follow under a predicate
                        uint32_t hl[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const float own = __uint_as_float(up ? v[16 + j] : v[j]);
                            const float other = __shfl_xor_sync(0xffffffffu, __uint_as_float(up ? v[j] : v[16 + j]), 16);
                            const float g = up ? other : own, u = up ? own : other;
                            hl[j] = split_hi_lo(gelu_tanh_fast(g) * u);
                        }
                        const int t0 = c0 + (up ? 16 : 0);
                        uint16_t* ph = reinterpret_cast<uint16_t*>(oh) + (size_t)(row0 + t0) * kout;
                        uint16_t* pl = reinterpret_cast<uint16_t*>(olo) + (size_t)(row0 + t0) * kout;
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (t0 + j < rows) {
                                ph[(size_t)j * kout] = (uint16_t)(hl[j] >> 16);
                                pl[(size_t)j * kout] = (uint16_t)(hl[j] & 0xFFFFu);
                            }
                    }
                }
                tc::tc_fence_before();
                tc::mbar_arrive(&acc_empty[slot]);
            }
        }
    }
    // peer stores complete at system scope before this kernel ends (the ranks' barrier follows)
    if (MODE == 1 && A.per_src > 0) __threadfence_system();
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
    const int* pos;           // [T][8] row of each (token, slot) in out_r (null: token x 8 + slot)
    const float* w;           // [T][8] routing weights
    const float* out_r;       // [8T][D], expert outputs (routing weight not applied)
    const float* out_s;       // [T][D]
    GtmLayer L;
    float eps;
    float* hidden_out;        // [T][D]
    float* h1_out;            // [T][D] or null
    float* h2_out;            // [T][D] or null
};

// Four bf16 (elements 4c .. 4c+3) as floats: one 8-byte load when p is 8-byte aligned.
__device__ __forceinline__ void ld4_bf16(const uint16_t* p, int c, float (&w)[4]) {
    if ((reinterpret_cast<uintptr_t>(p) & 7) == 0) {
        const uint2 g = reinterpret_cast<const uint2*>(p)[c];
        w[0] = __uint_as_float(g.x << 16); w[1] = __uint_as_float(g.x & 0xFFFF0000u);
        w[2] = __uint_as_float(g.y << 16); w[3] = __uint_as_float(g.y & 0xFFFF0000u);
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = bf16f(p[4 * c + e]);
    }
}

// Elements 4c .. 4c+3 of a float row: one 16-byte access when the row is 16-byte aligned (the
// io pointers of gtm_moe_tokens need only 4-byte alignment).
__device__ __forceinline__ void ld4_f32(const float* p, int c, float (&v)[4]) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        const float4 f = reinterpret_cast<const float4*>(p)[c];
        v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = p[4 * c + e];
    }
}
__device__ __forceinline__ void st4_f32(float* p, int c, const float (&v)[4]) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        reinterpret_cast<float4*>(p)[c] = make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) p[4 * c + e] = v[e];
    }
}

constexpr int CT = D / 4;                     // combine: threads per token, one float4 of each row
constexpr int CV = (D / 4 + CT - 1) / CT;     // float4 chunks of a row per thread

// Block-wide sums of (a, b), every thread gets the same bits (warp partials added in warp
// order). Consecutive calls alternate `buf`.
__device__ __forceinline__ double2 combine_sum2(double a, double b, double (*red)[CT / 32][2], int buf) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    if (lane == 0) { red[buf][warp][0] = a; red[buf][warp][1] = b; }
    __syncthreads();
    double ra = 0.0, rb = 0.0;
#pragma unroll
    for (int w = 0; w < CT / 32; ++w) { ra += red[buf][w][0]; rb += red[buf][w][1]; }
    return make_double2(ra, rb);
}

// h1 = rms(shared)*w_pf1 (cpu_reference.cpp:492-493); h2 = sum_k w_k out_k in router order
// (:508-509); hidden = (x + rms(rms(h2)*w_pf2 + h1)*w_pf) * layer_scalar (:512-520).
// One CTA per token; each thread keeps its float4 chunks of every vector in registers and
// issues all of its row loads before the first reduction.
__global__ void __launch_bounds__(CT, 2) tok_combine(const __grid_constant__ CombineArgs A) {
    __shared__ double red[2][CT / 32][2];
    const int t = blockIdx.x, tid = threadIdx.x;
    const GtmLayer& L = A.L;
    int p[TOPK];
    float wk[TOPK];
#pragma unroll
    for (int k = 0; k < TOPK; ++k) {
        p[k] = A.pos ? A.pos[(size_t)t * TOPK + k] : t * TOPK + k;
        wk[k] = A.w[(size_t)t * TOPK + k];
    }
    const float4* outs = reinterpret_cast<const float4*>(A.out_s) + (size_t)t * (D / 4);
    float sv[CV][4], hv[CV][4], xv[CV][4];
    double a = 0.0, b = 0.0;
#pragma unroll
    for (int v = 0; v < CV; ++v) {
        const int c = tid + v * CT;
        if (c < D / 4) {
            const float4 so = outs[c];
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int k = 0; k < TOPK; ++k) {
                const float4 r = reinterpret_cast<const float4*>(A.out_r + (size_t)p[k] * D)[c];
                acc[0] = __fadd_rn(acc[0], __fmul_rn(wk[k], r.x));
                acc[1] = __fadd_rn(acc[1], __fmul_rn(wk[k], r.y));
                acc[2] = __fadd_rn(acc[2], __fmul_rn(wk[k], r.z));
                acc[3] = __fadd_rn(acc[3], __fmul_rn(wk[k], r.w));
            }
            sv[v][0] = so.x; sv[v][1] = so.y; sv[v][2] = so.z; sv[v][3] = so.w;
            if (A.x_f32) ld4_f32(A.x_f32 + (size_t)t * D, c, xv[v]);
            else ld4_bf16(A.x_bf16 + (size_t)t * D, c, xv[v]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                hv[v][e] = acc[e];
                a += (double)sv[v][e] * sv[v][e];
                b += (double)acc[e] * acc[e];
            }
        }
    }
    double2 r = combine_sum2(a, b, red, 0);
    const float inv1 = 1.0f / sqrtf((float)(r.x / D) + A.eps);
    const float inv2 = 1.0f / sqrtf((float)(r.y / D) + A.eps);
    const uint16_t* w_pf1 = rp16(L.resident_dev, L.post_ffn_norm_1);
    const uint16_t* w_pf2 = rp16(L.resident_dev, L.post_ffn_norm_2);
    const uint16_t* w_pf = rp16(L.resident_dev, L.post_ffn_norm);
    const float ls = bf16f(*rp16(L.resident_dev, L.layer_scalar));
    a = 0.0;
#pragma unroll
    for (int v = 0; v < CV; ++v) {
        const int c = tid + v * CT;
        if (c < D / 4) {
            float w1[4], w2[4], h1[4];
            ld4_bf16(w_pf1, c, w1);
            ld4_bf16(w_pf2, c, w2);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                h1[e] = (sv[v][e] * inv1) * w1[e];
                const float tv = (hv[v][e] * inv2) * w2[e] + h1[e];
                sv[v][e] = hv[v][e];   // h2, kept for its store
                hv[v][e] = tv;
                a += (double)tv * tv;
            }
            if (A.h1_out) st4_f32(A.h1_out + (size_t)t * D, c, h1);
            if (A.h2_out) st4_f32(A.h2_out + (size_t)t * D, c, sv[v]);
        }
    }
    r = combine_sum2(a, 0.0, red, 1);
    const float inv3 = 1.0f / sqrtf((float)(r.x / D) + A.eps);
#pragma unroll
    for (int v = 0; v < CV; ++v) {
        const int c = tid + v * CT;
        if (c < D / 4) {
            float w[4], o[4];
            ld4_bf16(w_pf, c, w);
#pragma unroll
            for (int e = 0; e < 4; ++e) o[e] = (xv[v][e] + (hv[v][e] * inv3) * w[e]) * ls;
            st4_f32(A.hidden_out + (size_t)t * D, c, o);
        }
    }
}

// ================================================================================================
// host side
// ================================================================================================
struct WsLayout {
    size_t dense_hi, dense_lo, routed, idx, w, perm_src, pos, chunk, tiles0, tiles1, n_tiles, stiles0, stiles1, sn_tiles, act_r_hi,
        act_r_lo, act_s_hi, act_s_lo, out_r, out_s, send_pos, send_src, views_all, idx_all, hdr, ret, rlog, total;
};

// single GPU; expert parallelism with the caller's all-to-all; expert parallelism over peer memory
enum WsMode { WS_SINGLE, WS_EP, WS_PEER };

static size_t align256(size_t n) { return (n + 255) / 256 * 256; }

// T: own tokens; R: routed rows through the experts (T * top_k on one GPU, the received rows
// with expert parallelism, every rank's entries (world * T * top_k) over peer memory).
// Over peer memory (P ranks) every rank has the same layout, so a peer's regions sit at the same
// offsets; the routed views and top-8 ids of rank s live in slot s of views_all / idx_all on
// every rank (written there by rank s's dispatch), and `routed` / `idx` name this rank's slot.
static WsLayout ws_layout(uint32_t T, uint32_t Rrows, WsMode mode, uint32_t P = 1, uint32_t rank = 0) {
    const bool ep = mode != WS_SINGLE;
    WsLayout W;
    const size_t E8 = (size_t)T * TOPK, R = Rrows;
    const size_t ntr = R / NT + NE, nts = (T + NT - 1) / NT;   // bounds on routed / shared token tiles
    size_t o = 256;   // [0, 256): error word
    auto take = [&](size_t bytes) { const size_t at = o; o = align256(o + bytes); return at; };
    W.dense_hi = take((size_t)T * D * 2);
    W.dense_lo = take((size_t)T * D * 2);
    if (mode == WS_PEER) {
        W.views_all = take((size_t)P * T * D * 4);
        W.idx_all = take((size_t)P * E8 * 4);
        W.routed = W.views_all + (size_t)rank * T * D * 4;
        W.idx = W.idx_all + (size_t)rank * E8 * 4;
    } else {
        W.views_all = W.idx_all = 0;
        W.routed = take((size_t)T * D * 4);
        W.idx = take(E8 * 4);
    }
    W.w = take(E8 * 4);
    W.perm_src = take(R * 4);
    W.pos = take(R * 4);
    W.chunk = take((R + RC - 1) / RC * NE * 4);
    W.tiles0 = take((ntr * FB0_R + nts * FB0_S) * sizeof(Tile));
    W.tiles1 = take((ntr * FB1 + nts * FB1) * sizeof(Tile));
    W.n_tiles = take(2 * 4);
    // expert parallelism: the shared-expert phase keeps its own tile lists, so it can run on
    // another stream while the experts phase (same workspace) runs
    W.stiles0 = ep ? take(nts * FB0_S * sizeof(Tile)) : 0;
    W.stiles1 = ep ? take(nts * FB1 * sizeof(Tile)) : 0;
    W.sn_tiles = ep ? take(2 * 4) : 0;
    W.act_r_hi = take(R * FE * 2);
    W.act_r_lo = take(R * FE * 2);
    W.act_s_hi = take((size_t)T * FS * 2);
    W.act_s_lo = take((size_t)T * FS * 2);
    W.out_r = ep ? 0 : take(R * D * 4);
    W.out_s = take((size_t)T * D * 4);
    W.send_pos = mode == WS_EP ? take(E8 * 4) : 0;
    W.send_src = mode == WS_EP ? take(E8 * 4) : 0;
    // peer memory: [s] token count of rank s (written by its dispatch), [P] rows routed here;
    // ret: [T * top_k][D] expert outputs of the own entries, stored by the experts' owners
    W.hdr = mode == WS_PEER ? take((P + 1) * 4) : 0;
    W.ret = mode == WS_PEER ? take(E8 * D * 4) : 0;
    W.rlog = take((size_t)T * NE * 4);
    W.total = o;
    return W;
}

}  // namespace tok

size_t tokens_workspace_bytes(uint32_t max_tokens) {
    return tok::ws_layout(max_tokens, max_tokens * tok::TOPK, tok::WS_SINGLE).total;
}
size_t ep_workspace_bytes(uint32_t max_tokens, uint32_t max_recv) {
    return tok::ws_layout(max_tokens, max_recv, tok::WS_EP).total;
}
size_t ep_peer_workspace_bytes(uint32_t world, uint32_t max_tokens) {
    return tok::ws_layout(max_tokens, world * max_tokens * tok::TOPK, tok::WS_PEER, world, 0).total;
}

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

// Activation map: fp16 [rows][k], boxes of 64 (k) x `box_rows` rows in the 128-byte swizzle layout.
static int map_act(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t k, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_error(GTM_ERR_CUDA, "cuTensorMapEncodeTiled not available");
    const cuuint64_t dims[2] = {k, rows};
    const cuuint64_t strides[1] = {k * 2};
    const cuuint32_t box[2] = {tok::BK, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(GTM_ERR_CUDA, "cuTensorMapEncodeTiled (activations) failed (%d)", (int)r);
    return GTM_OK;
}

// Packed int4 weights of one matrix kind: rows of k/2 bytes, boxes of 32 bytes (one K block) x
// `box_rows` rows in the 32-byte swizzle layout. Routed: 3D over (byte, row, expert) with the
// expert block stride; shared: 2D.
static int map_w(CUtensorMap* m, const void* ptr, uint64_t k, uint64_t rows, uint64_t experts, uint64_t stride,
                 uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_error(GTM_ERR_CUDA, "cuTensorMapEncodeTiled not available");
    const cuuint64_t dims[3] = {k / 2, rows, experts ? experts : 1};
    const cuuint64_t strides[2] = {k / 2, experts ? stride : k / 2 * rows};
    const cuuint32_t box[3] = {32, box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, experts ? 3 : 2, const_cast<void*>(ptr), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(GTM_ERR_CUDA, "cuTensorMapEncodeTiled (weights) failed (%d)", (int)r);
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

// peer_ws: every rank's workspace (peer-memory expert parallelism; null otherwise)
void launch_views(const GtmDims& dims, const GtmLayer& L, const GtmTokensIO& io, const Ws& w, cudaStream_t st,
                  const GtmEpConfig* ep = nullptr, void* const* peer_ws = nullptr) {
    ViewsArgs va;
    memset(&va, 0, sizeof(va));
    va.T = (int)io.num_tokens; va.x_f32 = io.x_dev; va.x_bf16 = io.x_bf16_dev; va.L = L; va.eps = dims.eps;
    va.inv_sqrt_d = 1.0f / sqrtf((float)D);
    va.logit_bias = io.logit_bias_dev; va.route_logits = io.route_logits_dev;
    va.dense_hi = w.p<__half>(w.W.dense_hi); va.dense_lo = w.p<__half>(w.W.dense_lo);
    va.routed_hl = w.p<__half>(w.W.routed);
    va.idx = w.p<uint32_t>(w.W.idx); va.w = w.p<float>(w.W.w);
    va.logits_out = io.logits_dev;
    if (peer_ws) {
        va.npeers = (int)ep->world; va.epr = NE / (int)ep->world;
        for (uint32_t s = 0; s < ep->world; ++s) {
            if (s == ep->rank) continue;
            const Ws ps{w.W, static_cast<uint8_t*>(peer_ws[s])};
            va.push_idx[s] = ps.p<uint32_t>(w.W.idx);
            va.push_views[s] = ps.p<__half>(w.W.routed);
        }
    }
    const uintptr_t xa = reinterpret_cast<uintptr_t>(io.x_dev ? static_cast<const void*>(io.x_dev) : io.x_bf16_dev);
    if (!peer_ws && (xa & 15) == 0) {
        if (!io.route_logits_dev) {   // the router rows first, 16 rows per CTA
            tok_router_rows<<<dim3(io.num_tokens, NE / RR_ROWS), RR_THREADS, 0, st>>>(va, w.p<float>(w.W.rlog));
            va.route_logits = w.p<float>(w.W.rlog);
        }
        tok_views_given<<<io.num_tokens, VG_THREADS, 0, st>>>(va);
    } else {
        tok_views_router<<<io.num_tokens, io.route_logits_dev ? 512 : 1024, 0, st>>>(va);
    }
}

// What one pass of the two grouped GEMMs runs over.
struct Plan {
    int n;                        // routed entries (rows through the experts)
    int src_div;                  // activation source row of entry i = i / src_div
    const uint32_t* idx;          // expert ids, stride `stride`
    int stride;
    int e0, ne;                   // experts [e0, e0 + ne), layer.experts_dev pointing at e0
    int t_shared;                 // tokens through the shared expert (0: none)
    const __half* act_src;        // routed views (high row, low row): row perm_src[r] / act_div
    const int* out_index;         // mode 1 output row of each expert-ordered row (null: same)
    float* out_r;                 // mode 1 routed output rows
    bool own_tiles;               // shared-expert-only plan: tile lists in the stiles* regions
    bool test_wait;               // GTM_TOKENS_TEST_WAIT_RUNS_OUT (gate/up GEMM)
    // peer-memory expert parallelism (nsrc > 0): entry i is entry i % per_src of rank i / per_src,
    // read from that rank's workspace; its result goes to that rank's return region
    int nsrc, per_src;
    const uint32_t* src_idx[kMaxPeers];
    const int* src_ntok[kMaxPeers];
    float* src_ret[kMaxPeers];
    int act_div;                  // routed view of row r = perm_src[r] / act_div (1 when not set)
    int* nrows;                   // rows routed to this rank (written by the routing scan)
};

// Stage events of gtm_set_phase_events (thread-local: each host thread times its own calls).
thread_local cudaEvent_t t_phase_ev[GTM_PHASE_EVENTS];
thread_local int t_phase_n = 0;
inline void mark_phase(int i, cudaStream_t st) {
    if (i < t_phase_n) cudaEventRecord(t_phase_ev[i], st);
}

int run_gemms(const GtmLayer& L, const Ws& w, const Plan& pl, int num_sms, cudaStream_t st) {
    const WsLayout& W = w.W;
    const uint8_t* res = static_cast<const uint8_t*>(L.resident_dev);
    const uint8_t* exb = static_cast<const uint8_t*>(L.experts_dev);
    const uint64_t R = pl.n > 0 ? (uint64_t)pl.n : 1, T = pl.t_shared > 0 ? (uint64_t)pl.t_shared : 1;

    GemmArgs g0, g1;
    memset(&g0, 0, sizeof(g0));
    memset(&g1, 0, sizeof(g1));
    int rc;
    g0.wide_r = g1.wide_r = R >= (uint64_t)NT;
    g0.wide_s = g1.wide_s = T >= (uint64_t)NT;
    // 32-row boxes over every activation tensor; 128-row boxes where the tensor has >= 128 rows
    struct ActMap { CUtensorMap* narrow; CUtensorMap* wide; const void* ptr; uint64_t rows, k; };
    // (mode 0 routed tiles gather their rows from the routed views instead of a map)
    const ActMap maps[] = {
        {&g0.x_shi, &g0.y_shi, w.at(W.dense_hi), T, D},     {&g0.x_slo, &g0.y_slo, w.at(W.dense_lo), T, D},
        {&g1.x_rhi, &g1.y_rhi, w.at(W.act_r_hi), R, FE},    {&g1.x_rlo, &g1.y_rlo, w.at(W.act_r_lo), R, FE},
        {&g1.x_shi, &g1.y_shi, w.at(W.act_s_hi), T, FS},    {&g1.x_slo, &g1.y_slo, w.at(W.act_s_lo), T, FS}};
    for (const ActMap& m : maps) {
        if ((rc = map_act(m.narrow, m.ptr, m.rows, m.k, 32))) return rc;
        if (m.rows >= (uint64_t)NT && (rc = map_act(m.wide, m.ptr, m.rows, m.k, NT))) return rc;
    }

    RouteArgs ra;
    memset(&ra, 0, sizeof(ra));
    ra.n = pl.n; ra.src_div = pl.src_div; ra.idx = pl.idx; ra.stride = pl.stride;
    ra.e0 = pl.e0; ra.ne = pl.ne; ra.t_shared = pl.t_shared;
    ra.nchunks = (pl.n + RC - 1) / RC; ra.chunk = w.p<int>(W.chunk);
    ra.perm_src = w.p<int>(W.perm_src); ra.pos = w.p<int>(W.pos);
    ra.tiles0 = w.p<Tile>(pl.own_tiles ? W.stiles0 : W.tiles0);
    ra.tiles1 = w.p<Tile>(pl.own_tiles ? W.stiles1 : W.tiles1);
    ra.n_tiles = w.p<int>(pl.own_tiles ? W.sn_tiles : W.n_tiles);
    ra.nsrc = pl.nsrc; ra.per_src = pl.per_src;
    for (int s = 0; s < pl.nsrc; ++s) { ra.src_idx[s] = pl.src_idx[s]; ra.src_ntok[s] = pl.src_ntok[s]; }
    ra.nrows = pl.nrows;
    mark_phase(1, st);
    if (ra.nchunks <= 1) {
        tok_route_one<<<1, RC, 0, st>>>(ra);
    } else {
        tok_route_count<<<(unsigned)ra.nchunks, RC, 0, st>>>(ra);
        tok_route_scan<<<1, 1024, 0, st>>>(ra);
        tok_route_scatter<<<(unsigned)ra.nchunks, RC, 0, st>>>(ra);
    }
    cudaFuncSetAttribute(grouped_gemm<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    cudaFuncSetAttribute(grouped_gemm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);

    const uint64_t ne = pl.ne > 0 ? (uint64_t)pl.ne : 1, es = L.expert_stride;
    if ((rc = map_w(&g0.w_ra, exb + L.expert_gate.weight, D, FE, ne, es, 128)) ||
        (rc = map_w(&g0.w_rb, exb + L.expert_up.weight, D, FE, ne, es, 128)) ||
        (rc = map_w(&g0.w_sa, res + L.shared_gate.weight, D, FS, 0, 0, 128)) ||
        (rc = map_w(&g0.w_sb, res + L.shared_up.weight, D, FS, 0, 0, 128)) ||
        (rc = map_w(&g1.w_ra, exb + L.expert_down.weight, FE, D, ne, es, MW)) ||
        (rc = map_w(&g1.w_sa, res + L.shared_down.weight, FS, D, 0, 0, MW)))
        return rc;
    g1.w_rb = g1.w_ra;
    g1.w_sb = g1.w_sa;

    g0.tiles = ra.tiles0; g0.n_tiles = ra.n_tiles; g0.test_wait = pl.test_wait ? 1 : 0;
    g0.experts = exb; g0.expert_stride = L.expert_stride; g0.resident = res;
    g0.r_sa = L.expert_gate.scales; g0.r_ba = L.expert_gate.biases; g0.r_sb = L.expert_up.scales; g0.r_bb = L.expert_up.biases;
    g0.s_sa = L.shared_gate.scales; g0.s_ba = L.shared_gate.biases; g0.s_sb = L.shared_up.scales; g0.s_bb = L.shared_up.biases;
    g0.k_r = D; g0.k_s = D; g0.rows_r = FE; g0.rows_s = FS;
    g0.act_r_hi = w.p<__half>(W.act_r_hi); g0.act_r_lo = w.p<__half>(W.act_r_lo);
    g0.act_s_hi = w.p<__half>(W.act_s_hi); g0.act_s_lo = w.p<__half>(W.act_s_lo);
    g0.act_src = pl.act_src; g0.act_row = ra.perm_src; g0.act_div = pl.act_div > 0 ? pl.act_div : 1;
    g0.err = w.p<int>(0);
    mark_phase(2, st);
    grouped_gemm<0><<<num_sms, THREADS, SMEM_BYTES, st>>>(g0);

    g1.tiles = ra.tiles1; g1.n_tiles = ra.n_tiles + 1;
    g1.experts = exb; g1.expert_stride = L.expert_stride; g1.resident = res;
    g1.r_sa = L.expert_down.scales; g1.r_ba = L.expert_down.biases; g1.r_sb = g1.r_sa; g1.r_bb = g1.r_ba;
    g1.s_sa = L.shared_down.scales; g1.s_ba = L.shared_down.biases; g1.s_sb = g1.s_sa; g1.s_bb = g1.s_ba;
    g1.k_r = FE; g1.k_s = FS; g1.rows_r = D; g1.rows_s = D;
    g1.out_r = pl.out_r; g1.out_s = w.p<float>(W.out_s);
    g1.out_index = pl.out_index;
    g1.per_src = pl.nsrc > 0 ? pl.per_src : 0;
    for (int s = 0; s < pl.nsrc; ++s) g1.out_peer[s] = pl.src_ret[s];
    g1.err = w.p<int>(0);
    mark_phase(3, st);
    grouped_gemm<1><<<num_sms, THREADS, SMEM_BYTES, st>>>(g1);
    return GTM_OK;
}

void launch_combine(const GtmDims& dims, const GtmLayer& L, const GtmTokensIO& io, const Ws& w, const int* pos,
                    const float* out_r, cudaStream_t st) {
    CombineArgs ca;
    ca.T = (int)io.num_tokens; ca.x_f32 = io.x_dev; ca.x_bf16 = io.x_bf16_dev; ca.pos = pos; ca.w = w.p<float>(w.W.w);
    ca.out_r = out_r; ca.out_s = w.p<float>(w.W.out_s); ca.L = L; ca.eps = dims.eps;
    ca.hidden_out = io.hidden_out_dev; ca.h1_out = io.h1_dev; ca.h2_out = io.h2_dev;
    tok_combine<<<io.num_tokens, CT, 0, st>>>(ca);
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
    const Ws w{ws_layout(T, T * TOPK, WS_SINGLE), static_cast<uint8_t*>(ws)};
    if (ws_bytes < w.W.total) return set_error(GTM_ERR_WORKSPACE, "gtm_moe_tokens: workspace needs %zu bytes", w.W.total);
    mark_phase(0, st);
    launch_views(dims, L, io, w, st);
    Plan pl;
    memset(&pl, 0, sizeof(pl));
    pl.n = (int)(T * TOPK); pl.src_div = TOPK; pl.idx = w.p<uint32_t>(w.W.idx); pl.stride = 1;
    pl.e0 = 0; pl.ne = NE; pl.t_shared = (int)T; pl.act_src = w.p<__half>(w.W.routed); pl.out_index = nullptr;
    pl.out_r = w.p<float>(w.W.out_r);
    pl.test_wait = (io.flags & GTM_TOKENS_TEST_WAIT_RUNS_OUT) != 0;
    const int rc = run_gemms(L, w, pl, num_sms, st);
    if (rc) return rc;
    mark_phase(4, st);
    launch_combine(dims, L, io, w, w.p<int>(w.W.pos), pl.out_r, st);
    mark_phase(5, st);
    return finish("gtm_moe_tokens", &io, &w, st);
}

// ---- expert parallelism ----------------------------------------------------------------------
// Every phase of a rank lays the workspace out from (max_tokens, max_recv_rows) of its config, so
// the regions that carry data from one phase to the next (views, dispatch tables, shared-expert
// output) are the same in all of them.
static Ws ep_ws(const GtmEpConfig& ep, void* ws) {
    return Ws{ws_layout(ep.max_tokens, ep.max_recv_rows, WS_EP), static_cast<uint8_t*>(ws)};
}
static Ws peer_ws(const GtmEpConfig& ep, void* ws) {
    return Ws{ws_layout(ep.max_tokens, ep.world * ep.max_tokens * TOPK, WS_PEER, ep.world, ep.rank),
              static_cast<uint8_t*>(ws)};
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
                     int num_sms, bool peer) {
    const Ws w = peer ? peer_ws(ep, ws) : ep_ws(ep, ws);
    Plan pl;
    memset(&pl, 0, sizeof(pl));
    pl.n = 0; pl.src_div = 1; pl.idx = w.p<uint32_t>(w.W.idx); pl.stride = 1;
    pl.e0 = 0; pl.ne = 0; pl.t_shared = (int)io.num_tokens;
    pl.own_tiles = true;
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
    memset(&pl, 0, sizeof(pl));
    pl.n = (int)n_recv; pl.src_div = 1;
    pl.idx = &recv_meta->expert; pl.stride = 2;
    pl.e0 = (int)ep.rank * epr; pl.ne = epr; pl.t_shared = 0;
    pl.act_src = reinterpret_cast<const __half*>(recv_rows); pl.out_index = w.p<int>(w.W.perm_src); pl.out_r = ret_rows;
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

// ---- expert parallelism over peer memory -------------------------------------------------------
int launch_ep_peer_dispatch(const GtmDims& dims, const GtmLayer& L, const GtmTokensIO& io, const GtmEpConfig& ep,
                            void* const* peer_ws_dev, cudaStream_t st) {
    const Ws w = peer_ws(ep, peer_ws_dev[ep.rank]);
    if (io.num_tokens > 0) launch_views(dims, L, io, w, st, &ep, peer_ws_dev);   // a rank may have no tokens
    CountArgs ca;
    memset(&ca, 0, sizeof(ca));
    ca.n = (int)ep.world; ca.v = (int)io.num_tokens;
    for (uint32_t s = 0; s < ep.world; ++s) ca.dst[s] = reinterpret_cast<int*>(static_cast<uint8_t*>(peer_ws_dev[s]) + w.W.hdr) + ep.rank;
    tok_set_count<<<1, 1, 0, st>>>(ca);
    return finish("gtm_moe_ep_peer_dispatch", &io, &w, st);
}

int launch_ep_peer_experts(const GtmLayer& L, const GtmEpConfig& ep, void* const* peer_ws_dev, cudaStream_t st,
                           int num_sms) {
    const Ws w = peer_ws(ep, peer_ws_dev[ep.rank]);
    const int P = (int)ep.world, epr = NE / P;
    Plan pl;
    memset(&pl, 0, sizeof(pl));
    pl.nsrc = P; pl.per_src = (int)ep.max_tokens * TOPK;
    pl.n = P * pl.per_src; pl.src_div = 1; pl.stride = 1;
    pl.e0 = (int)ep.rank * epr; pl.ne = epr; pl.t_shared = 0;
    pl.out_index = w.p<int>(w.W.perm_src);
    pl.nrows = w.p<int>(w.W.hdr) + P;
    // every rank's top-8 ids, token counts and routed views were stored into this workspace by
    // their dispatch; only the results cross NVLink here. Entry i = s * per_src + token * 8 + slot
    // reads row i / 8 = s * max_tokens + token of views_all.
    pl.act_src = w.p<__half>(w.W.views_all);
    pl.act_div = TOPK;
    for (int s = 0; s < P; ++s) {
        pl.src_idx[s] = w.p<uint32_t>(w.W.idx_all) + (size_t)s * pl.per_src;
        pl.src_ntok[s] = w.p<int>(w.W.hdr) + s;
        pl.src_ret[s] = reinterpret_cast<float*>(static_cast<uint8_t*>(peer_ws_dev[s]) + w.W.ret);
    }
    const int rc = run_gemms(L, w, pl, num_sms, st);
    if (rc) return rc;
    return finish("gtm_moe_ep_peer_experts", nullptr, nullptr, st);
}

int launch_ep_peer_combine(const GtmDims& dims, const GtmLayer& L, const GtmTokensIO& io, const GtmEpConfig& ep,
                           void* ws, cudaStream_t st) {
    const Ws w = peer_ws(ep, ws);
    launch_combine(dims, L, io, w, nullptr, w.p<float>(w.W.ret), st);
    return finish("gtm_moe_ep_peer_combine", nullptr, nullptr, st);
}

int set_phase_events(void* const* events, int n) {
    if (n < 0 || n > GTM_PHASE_EVENTS || (n > 0 && !events))
        return set_error(GTM_ERR_INVALID, "gtm_set_phase_events: n=%d (0..%d) and events needed", n, GTM_PHASE_EVENTS);
    for (int i = 0; i < n; ++i) {
        if (!events[i]) return set_error(GTM_ERR_INVALID, "gtm_set_phase_events: event %d is NULL", i);
        t_phase_ev[i] = static_cast<cudaEvent_t>(events[i]);
    }
    t_phase_n = n;
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

// Fused batch-1 MoE decode for sm_100a: one persistent cooperative launch runs a token through
// `num_layers` MoE blocks with every expert resident in HBM and no host round trip.
//
// Replaces the per-layer MoE sequence of ForwardRunner::produce_token (src/runner.cpp:549-716):
// MulBF16 -> GemvInt8 -> RouterTopK -> CPU read-back -> shared expert (GemvInt4 x3, GeGLU,
// RMSNormK) -> per expert GemvInt4 gate/up, GeGLU, GemvInt4 down, ScaleAccum -> LayerTail.
//
// Per layer, three phases separated by bounded grid barriers:
//   P1  every CTA rebuilds the block input from the previous layer's h2 / shared output (layer
//       tail, optional between-layer RMSNorm) and the three views (dense_x, routed_x and the
//       router input) in shared memory; CTAs 0..127 each compute one router logit with the
//       reference's exact accumulation order (bit-identical logits).
//   P2  every CTA selects the top-8 itself from the 128 logits, then computes its share of the
//       7744 gate/up row pairs (8 x 704 routed + 2112 shared) with GeGLU fused.
//   P3  every CTA computes ~19 rows of the 2816-wide down projection: the shared expert's row
//       and the 8 routed experts' rows, combined with the routing weights (h2) in one pass.
// Within a CTA the 352 threads split the input dimension of each row (one 32-bit word = 8
// int4 weights per thread and row) and rows are reduced with a warp transpose-reduce.
#include <cstdint>
#include <cuda_runtime.h>

#include "gtm_common.cuh"
#include "gtm_internal.h"

namespace gtm {
namespace dec {

constexpr int D = 2816, FE = 704, FS = 2112, NE = 128, TOPK = 8;
constexpr int NT = D / 8;                     // 352 threads, one word of a K=2816 row each
constexpr int NWARP = NT / 32;                // 11
constexpr int GD = D / kGroup;                // 44
constexpr int UNITS_R = TOPK * FE;            // 5632 routed gate/up row pairs
constexpr int UNITS = UNITS_R + FS;           // + 2112 shared
constexpr int DW_SH = FS / 8;                 // 264 words in a shared-down row
constexpr int DW_EX = FE / 8;                 // 88 words in a routed-down row
constexpr int DWORDS = DW_SH + TOPK * DW_EX;  // 968 words in a combined down row
constexpr int ROW_GU = D / 2;                 // 1408 bytes per gate/up row
constexpr int CH2 = 16;                       // gate/up row pairs per chunk (32 rows)
constexpr int CH3 = 8;                        // down rows per chunk (16 accumulators)
constexpr int RIN_PITCH = 65;                 // padded router-input row (bank spread)
constexpr uint64_t kTimeoutNs = 2000000000ull;

struct Params {
    GtmLayer layers[GTM_MAX_LAYERS];
    GtmDecodeIO io;
    int num_layers;
    float eps;
    float inv_sqrt_d;
    // workspace
    unsigned* flags;
    int* err;          // this launch's error word
    int* sticky;       // error word read and cleared by gtm_moe_decode_check
    float* logits;     // [NE]
    float* act;        // [UNITS]: routed (slot-major) then shared
    float* h2;         // [D]
    float* sh_out;     // [D]
};

struct Smem {
    float hid[D];
    float a[D];
    float b[D];
    float xr[D];
    float xd[D];
    float rin[GD * RIN_PITCH];
    float part[NWARP][32];
    float terms[GD];
    double red[40];
    uint64_t rows[32][3];
    float topw[TOPK];
    int topi[TOPK];
    int flag;
};

__device__ __forceinline__ const uint8_t* rp(const void* base, uint64_t off) {
    return static_cast<const uint8_t*>(base) + off;
}

// ---- P1 helpers --------------------------------------------------------------------------
// Layer tail of layer `L` (src/cpu_reference.cpp:512-520) on the block's copies of h2 (a) and
// the shared expert's output (b), updating s.hid in place; h1 is produced on the way.
__device__ void layer_tail(Smem& s, const GtmLayer& L, float eps, float* h1_out, float* h2_out) {
    const int tid = threadIdx.x;
    const uint16_t* w_pf1 = reinterpret_cast<const uint16_t*>(rp(L.resident_dev, L.post_ffn_norm_1));
    const uint16_t* w_pf2 = reinterpret_cast<const uint16_t*>(rp(L.resident_dev, L.post_ffn_norm_2));
    const uint16_t* w_pf = reinterpret_cast<const uint16_t*>(rp(L.resident_dev, L.post_ffn_norm));
    const float ls = bf16f(*reinterpret_cast<const uint16_t*>(rp(L.resident_dev, L.layer_scalar)));
    const float inv1 = exact_rms_inv(s.b, D, eps, s.red);   // h1 = rms(shared_out) * w_pf1
    const float inv2 = exact_rms_inv(s.a, D, eps, s.red);   // rms(h2) * w_pf2
    for (int i = tid; i < D; i += blockDim.x) {
        const float h1 = __fmul_rn(__fmul_rn(s.b[i], inv1), bf16f(w_pf1[i]));
        if (h1_out) h1_out[i] = h1;
        if (h2_out) h2_out[i] = s.a[i];
        s.a[i] = __fadd_rn(__fmul_rn(__fmul_rn(s.a[i], inv2), bf16f(w_pf2[i])), h1);
    }
    __syncthreads();
    const float inv3 = exact_rms_inv(s.a, D, eps, s.red);
    for (int i = tid; i < D; i += blockDim.x) {
        const float t2 = __fmul_rn(__fmul_rn(s.a[i], inv3), bf16f(w_pf[i]));
        s.hid[i] = __fmul_rn(__fadd_rn(s.hid[i], t2), ls);
    }
    __syncthreads();
}

// dense_x = h*w_pre, routed_x = h*w_pre2, router_in = h*bf16(router.scale)*(1/sqrt(D)) with
// h = rmsnorm_no_scale(hidden) (src/cpu_reference.cpp:425-443).
__device__ void views(Smem& s, const GtmLayer& L, float eps, float inv_sqrt_d) {
    const uint16_t* w_pre = reinterpret_cast<const uint16_t*>(rp(L.resident_dev, L.pre_ffn_norm));
    const uint16_t* w_pre2 = reinterpret_cast<const uint16_t*>(rp(L.resident_dev, L.pre_ffn_norm_2));
    const uint16_t* rs = reinterpret_cast<const uint16_t*>(rp(L.resident_dev, L.router_scale));
    const float inv = exact_rms_inv(s.hid, D, eps, s.red);
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        const float h = __fmul_rn(s.hid[i], inv);
        s.xd[i] = __fmul_rn(h, bf16f(w_pre[i]));
        s.xr[i] = __fmul_rn(h, bf16f(w_pre2[i]));
        s.rin[(i >> 6) * RIN_PITCH + (i & 63)] = __fmul_rn(__fmul_rn(h, bf16f(rs[i])), inv_sqrt_d);
    }
    __syncthreads();
}

// One router logit with src/cpu_reference.cpp:86-106's order: per group a sequential dot and
// x-sum over 64 bytes, then the group terms summed in group order.
__device__ float router_row(Smem& s, const GtmLayer& L, int row) {
    const int tid = threadIdx.x;
    const uint8_t* W = rp(L.resident_dev, L.router.weight) + (size_t)row * D;
    const uint16_t* S = reinterpret_cast<const uint16_t*>(rp(L.resident_dev, L.router.scales)) + row * GD;
    const uint16_t* B = reinterpret_cast<const uint16_t*>(rp(L.resident_dev, L.router.biases)) + row * GD;
    if (tid < GD) {
        const uint4* wg = reinterpret_cast<const uint4*>(W + tid * kGroup);
        uint4 q[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] = ldg_stream_u4(wg + i);
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
        s.terms[tid] = __fadd_rn(__fmul_rn(bf16f(ldg_u16(S + tid)), dot), __fmul_rn(bf16f(ldg_u16(B + tid)), sum));
    }
    __syncthreads();
    float acc = 0.0f;
    if (tid == 0) {
        for (int g = 0; g < GD; ++g) acc = __fadd_rn(acc, s.terms[g]);
    }
    __syncthreads();
    return acc;
}

// Top-8 of the 128 logits by (value desc, index asc), softmax over the 8, times
// per_expert_scale (src/cpu_reference.cpp:447-480). Warp 0.
__device__ void select_topk(Smem& s, const GtmLayer& L, const float* logits, bool write_out,
                            uint32_t* idx_out, float* w_out, float* logits_out) {
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    float v[4];
    bool taken[4] = {false, false, false, false};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        v[j] = __ldcg(logits + lane + 32 * j);
        if (write_out && logits_out) logits_out[lane + 32 * j] = v[j];
    }
    float sel[TOPK];
    int seli[TOPK];
#pragma unroll
    for (int k = 0; k < TOPK; ++k) {
        float bv = -INFINITY;
        int bi = 1 << 30;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = lane + 32 * j;
            if (!taken[j] && (bi == (1 << 30) || v[j] > bv || (v[j] == bv && e < bi))) { bv = v[j]; bi = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != (1 << 30) && (bi == (1 << 30) || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
        }
        sel[k] = bv;
        seli[k] = bi;
#pragma unroll
        for (int j = 0; j < 4; ++j) if (lane + 32 * j == bi) taken[j] = true;
    }
    if (lane == 0) {
        const uint16_t* pes = reinterpret_cast<const uint16_t*>(rp(L.resident_dev, L.per_expert_scale));
        float e[TOPK], sum = 0.0f;
        for (int k = 0; k < TOPK; ++k) { e[k] = expf(__fsub_rn(sel[k], sel[0])); sum = __fadd_rn(sum, e[k]); }
        for (int k = 0; k < TOPK; ++k) {
            const float w = __fmul_rn(__fdiv_rn(e[k], sum), bf16f(pes[seli[k]]));
            s.topi[k] = seli[k];
            s.topw[k] = w;
            if (write_out && idx_out) idx_out[k] = (uint32_t)seli[k];
            if (write_out && w_out) w_out[k] = w;
        }
    }
}

__device__ __forceinline__ float sum8(const float* x) {
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) a += x[i];
    return a;
}

// ---- P2: gate/up row pairs [u0, u1) of one kind with GeGLU ------------------------------
// routed == true: units index (slot k, row r) = (u / FE, u % FE); else shared row u - UNITS_R.
__device__ void gate_up_range(Smem& s, const GtmLayer& L, const Params& P, int u0, int u1, bool routed,
                              const XSlice& xs, float xsum) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int c = u0; c < u1; c += CH2) {
        const int n = min(CH2, u1 - c);
        if (tid < 2 * CH2) {
            const int p = tid >> 1, up = tid & 1;
            uint64_t w = 0, sc = 0, bi = 0;
            if (p < n) {
                const int u = c + p;
                if (routed) {
                    const int k = u / FE, r = u - k * FE;
                    const uint8_t* blk = rp(L.experts_dev, (uint64_t)s.topi[k] * L.expert_stride);
                    const GtmQuant& q = up ? L.expert_up : L.expert_gate;
                    w = (uint64_t)(blk + q.weight + (uint64_t)r * ROW_GU);
                    sc = (uint64_t)(blk + q.scales + (uint64_t)r * GD * 2);
                    bi = (uint64_t)(blk + q.biases + (uint64_t)r * GD * 2);
                } else {
                    const int r = u - UNITS_R;
                    const GtmQuant& q = up ? L.shared_up : L.shared_gate;
                    const uint8_t* base = static_cast<const uint8_t*>(L.resident_dev);
                    w = (uint64_t)(base + q.weight + (uint64_t)r * ROW_GU);
                    sc = (uint64_t)(base + q.scales + (uint64_t)r * GD * 2);
                    bi = (uint64_t)(base + q.biases + (uint64_t)r * GD * 2);
                }
            }
            s.rows[tid][0] = w; s.rows[tid][1] = sc; s.rows[tid][2] = bi;
        }
        __syncthreads();
        uint32_t wv[2 * CH2];
        uint16_t sv[2 * CH2], bv[2 * CH2];
        const int g = tid >> 3;
#pragma unroll
        for (int r = 0; r < 2 * CH2; ++r) {
            if ((r >> 1) < n) {
                wv[r] = ldg_stream_u32(reinterpret_cast<const uint8_t*>(s.rows[r][0]) + 4 * tid);
                sv[r] = ldg_u16(reinterpret_cast<const uint16_t*>(s.rows[r][1]) + g);
                bv[r] = ldg_u16(reinterpret_cast<const uint16_t*>(s.rows[r][2]) + g);
            } else {
                wv[r] = 0; sv[r] = 0; bv[r] = 0;
            }
        }
        float v[2 * CH2];
#pragma unroll
        for (int r = 0; r < 2 * CH2; ++r) v[r] = fmaf(bf16f(sv[r]), dot_word(wv[r], xs), bf16f(bv[r]) * xsum);
        const float red = warp_transpose_reduce(v);
        s.part[warp][lane] = red;
        __syncthreads();
        if (tid < 2 * CH2) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < NWARP; ++w) tot += s.part[w][tid];
            const float other = __shfl_xor_sync(0xffffffffu, tot, 1);
            if ((tid & 1) == 0 && (tid >> 1) < n) {
                // tot = gate row, other = up row: gelu_pytorch_tanh(gate) * up
                const float x = tot;
                const float t = tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x));
                P.act[c + (tid >> 1)] = 0.5f * x * (1.0f + t) * other;
            }
        }
        __syncthreads();
    }
}

// Reduce R = 16 per-lane values across the warp: lane l (< 16) ends with value l's total.
__device__ __forceinline__ float warp_transpose_reduce16(float (&v)[16]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int half = 8; half >= 1; half >>= 1) {
        const bool upper = (lane & half) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, half);
        }
    }
    return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 16);
}

// ---- P3: down rows [j0, j1): shared row and the 8 routed rows, combined ------------------
__device__ void down_range(Smem& s, const GtmLayer& L, const Params& P, int j0, int j1) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // this thread's (up to) three words of the combined 968-word row
    const uint8_t* wb[3];
    const uint8_t* sb[3];
    const uint8_t* bb[3];
    uint32_t wstride[3], sstride[3];
    float fac[3];
    bool shared_seg[3], valid[3];
    XSlice xs[3];
    float xsum[3];
#pragma unroll
    for (int m = 0; m < 3; ++m) {
        const int i = tid + NT * m;
        valid[m] = i < DWORDS;
        const int ii = valid[m] ? i : 0;
        float x8[8];
        if (ii < DW_SH) {
            const uint8_t* base = static_cast<const uint8_t*>(L.resident_dev);
            wb[m] = base + L.shared_down.weight + 4 * ii;
            sb[m] = base + L.shared_down.scales + 2 * (ii >> 3);
            bb[m] = base + L.shared_down.biases + 2 * (ii >> 3);
            wstride[m] = FS / 2;
            sstride[m] = (FS / kGroup) * 2;
            fac[m] = 1.0f;
            shared_seg[m] = true;
            const float4* a = reinterpret_cast<const float4*>(P.act + UNITS_R + 8 * ii);
            const float4 a0 = __ldcg(a), a1 = __ldcg(a + 1);
            x8[0] = a0.x; x8[1] = a0.y; x8[2] = a0.z; x8[3] = a0.w; x8[4] = a1.x; x8[5] = a1.y; x8[6] = a1.z; x8[7] = a1.w;
        } else {
            const int k = (ii - DW_SH) / DW_EX, wis = (ii - DW_SH) - k * DW_EX;
            const uint8_t* blk = rp(L.experts_dev, (uint64_t)s.topi[k] * L.expert_stride);
            wb[m] = blk + L.expert_down.weight + 4 * wis;
            sb[m] = blk + L.expert_down.scales + 2 * (wis >> 3);
            bb[m] = blk + L.expert_down.biases + 2 * (wis >> 3);
            wstride[m] = FE / 2;
            sstride[m] = (FE / kGroup) * 2;
            fac[m] = s.topw[k];
            shared_seg[m] = false;
            const float4* a = reinterpret_cast<const float4*>(P.act + k * FE + 8 * wis);
            const float4 a0 = __ldcg(a), a1 = __ldcg(a + 1);
            x8[0] = a0.x; x8[1] = a0.y; x8[2] = a0.z; x8[3] = a0.w; x8[4] = a1.x; x8[5] = a1.y; x8[6] = a1.z; x8[7] = a1.w;
        }
        xs[m] = make_xslice(x8);
        xsum[m] = sum8(x8);
    }
    for (int c = j0; c < j1; c += CH3) {
        const int n = min(CH3, j1 - c);
        uint32_t wv[CH3][3];
        uint16_t sv[CH3][3], bv[CH3][3];
#pragma unroll
        for (int r = 0; r < CH3; ++r) {
#pragma unroll
            for (int m = 0; m < 3; ++m) {
                if (r < n && valid[m]) {
                    const uint32_t j = (uint32_t)(c + r);
                    wv[r][m] = ldg_stream_u32(wb[m] + (uint64_t)j * wstride[m]);
                    sv[r][m] = ldg_u16(sb[m] + (uint64_t)j * sstride[m]);
                    bv[r][m] = ldg_u16(bb[m] + (uint64_t)j * sstride[m]);
                } else {
                    wv[r][m] = 0; sv[r][m] = 0; bv[r][m] = 0;
                }
            }
        }
        float v[16];
#pragma unroll
        for (int r = 0; r < CH3; ++r) {
            float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
            for (int m = 0; m < 3; ++m) {
                const float t = fmaf(bf16f(sv[r][m]), dot_word(wv[r][m], xs[m]), bf16f(bv[r][m]) * xsum[m]);
                if (shared_seg[m]) a0 += t; else a1 = fmaf(fac[m], t, a1);
            }
            v[2 * r] = a0;
            v[2 * r + 1] = a1;
        }
        const float red = warp_transpose_reduce16(v);
        if (lane < 16) s.part[warp][lane] = red;
        __syncthreads();
        if (tid < 2 * CH3) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < NWARP; ++w) tot += s.part[w][tid];
            const int r = tid >> 1;
            if (r < n) {
                if (tid & 1) P.h2[c + r] = tot; else P.sh_out[c + r] = tot;
            }
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(NT, 1) moe_decode_kernel(const __grid_constant__ Params P) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_raw);
    const int tid = threadIdx.x;
    const int G = gridDim.x, cta = blockIdx.x;
    const GridSync gs{P.flags, P.err, P.sticky};
    unsigned epoch = 0;
    const GtmDecodeIO& io = P.io;
    const bool writer = cta == 0;

    for (int i = tid; i < D; i += NT) s.hid[i] = io.hidden_in_dev[i];
    __syncthreads();

    for (int l = 0; l < P.num_layers; ++l) {
        const GtmLayer& L = P.layers[l];
        // ---- P1: tail of the previous layer, views, router -------------------------------
        if (l > 0) {
            for (int i = tid; i < D; i += NT) { s.a[i] = __ldcg(P.h2 + i); s.b[i] = __ldcg(P.sh_out + i); }
            __syncthreads();
            const GtmLayer& Lp = P.layers[l - 1];
            layer_tail(s, Lp, P.eps, writer && io.h1_dev ? io.h1_dev + (size_t)(l - 1) * D : nullptr,
                       writer && io.h2_dev ? io.h2_dev + (size_t)(l - 1) * D : nullptr);
            if (io.flags & GTM_DECODE_NORM_BETWEEN_LAYERS) {
                const float inv = exact_rms_inv(s.hid, D, P.eps, s.red);
                for (int i = tid; i < D; i += NT) s.hid[i] = __fmul_rn(s.hid[i], inv);
                __syncthreads();
            }
            if (writer && io.hidden_layers_dev)
                for (int i = tid; i < D; i += NT) io.hidden_layers_dev[(size_t)(l - 1) * D + i] = s.hid[i];
        }
        views(s, L, P.eps, P.inv_sqrt_d);
        for (int row = cta; row < NE; row += G) {
            float lg = router_row(s, L, row);
            if (tid == 0) {
                if (io.logit_bias_dev) lg = __fadd_rn(lg, io.logit_bias_dev[(size_t)l * NE + row]);
                P.logits[row] = lg;
            }
        }
        if (!grid_barrier(gs, ++epoch, kTimeoutNs, &s.flag)) return;

        // ---- P2: top-8, gate/up + GeGLU -------------------------------------------------
        select_topk(s, L, P.logits, writer, io.topk_idx_dev ? io.topk_idx_dev + (size_t)l * TOPK : nullptr,
                    io.topk_w_dev ? io.topk_w_dev + (size_t)l * TOPK : nullptr,
                    io.logits_dev ? io.logits_dev + (size_t)l * NE : nullptr);
        __syncthreads();
        {
            const int u0 = (int)((long long)cta * UNITS / G), u1 = (int)((long long)(cta + 1) * UNITS / G);
            if (u0 < UNITS_R) {
                const XSlice xs = make_xslice(s.xr + 8 * tid);
                gate_up_range(s, L, P, u0, min(u1, UNITS_R), true, xs, sum8(s.xr + 8 * tid));
            }
            if (u1 > UNITS_R) {
                const XSlice xs = make_xslice(s.xd + 8 * tid);
                gate_up_range(s, L, P, max(u0, UNITS_R), u1, false, xs, sum8(s.xd + 8 * tid));
            }
        }
        if (!grid_barrier(gs, ++epoch, kTimeoutNs, &s.flag)) return;

        // ---- P3: down + combine ------------------------------------------------------------
        {
            const int j0 = (int)((long long)cta * D / G), j1 = (int)((long long)(cta + 1) * D / G);
            down_range(s, L, P, j0, j1);
        }
        if (!grid_barrier(gs, ++epoch, kTimeoutNs, &s.flag)) return;
    }

    // final tail by CTA 0
    if (!writer) return;
    const int l = P.num_layers;
    for (int i = tid; i < D; i += NT) { s.a[i] = __ldcg(P.h2 + i); s.b[i] = __ldcg(P.sh_out + i); }
    __syncthreads();
    layer_tail(s, P.layers[l - 1], P.eps, io.h1_dev ? io.h1_dev + (size_t)(l - 1) * D : nullptr,
               io.h2_dev ? io.h2_dev + (size_t)(l - 1) * D : nullptr);
    for (int i = tid; i < D; i += NT) {
        io.hidden_out_dev[i] = s.hid[i];
        if (io.hidden_layers_dev) io.hidden_layers_dev[(size_t)(l - 1) * D + i] = s.hid[i];
    }
}

}  // namespace dec

// Workspace: [0, 1024) barrier flags and [1024] this launch's error word (both cleared before
// every launch), [1032] the sticky error word (zero-initialised once by the owner of the
// workspace, read and cleared by gtm_moe_decode_check), then logits, act, h2, shared out.
constexpr size_t kStickyOffset = 1032;
size_t decode_workspace_bytes() {
    return 2048 + sizeof(float) * (dec::NE + dec::UNITS + 2 * dec::D) + 256;
}

int launch_decode(const GtmDims& dims, const GtmLayer* layers, int num_layers, const GtmDecodeIO& io,
                  void* ws, size_t ws_bytes, cudaStream_t stream, int num_ctas) {
    using namespace dec;
    Params P;  // ~17 KB, copied into the launch's parameter space by the launch call
    memset(&P, 0, sizeof(P));
    for (int l = 0; l < num_layers; ++l) P.layers[l] = layers[l];
    P.io = io;
    P.num_layers = num_layers;
    P.eps = dims.eps;
    P.inv_sqrt_d = 1.0f / sqrtf((float)D);
    unsigned char* w = static_cast<unsigned char*>(ws);
    P.flags = reinterpret_cast<unsigned*>(w);
    P.err = reinterpret_cast<int*>(w + 1024);
    P.sticky = reinterpret_cast<int*>(w + kStickyOffset);
    float* f = reinterpret_cast<float*>(w + 2048);
    P.logits = f;
    P.act = f + NE;
    P.h2 = P.act + UNITS;
    P.sh_out = P.h2 + D;
    (void)ws_bytes;
    cudaError_t e = cudaMemsetAsync(w, 0, 1028, stream);   // barrier flags restart at epoch 0
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

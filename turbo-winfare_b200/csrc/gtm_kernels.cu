// The reference's MoE compute kernels as sm_100a CUDA kernels, for the drop-in dispatch path
// (one kernel per HLSL shader). Where the reference CPU forward evaluates an expression with
// plain float operations, these evaluate it with the same operations in the same order
// (__fmul_rn / __fadd_rn, no contraction), so their outputs are bit-identical with
// src/cpu_reference.cpp; GeGLU and the routing softmax use CUDA's tanhf / expf.
#include <cstdint>
#include <cuda_runtime.h>

#include "gtm_common.cuh"
#include "gtm_internal.h"

namespace gtm {

// ---- GemvInt4 / GemvInt8 -------------------------------------------------------------------
// One thread per (row, group) forms the group's dot and x-sum in element order, then one thread
// per row adds the group terms in group order (src/cpu_reference.cpp:55-106).
template <int BITS>
__global__ void gemv_exact_kernel(uint32_t in_dim, const uint8_t* __restrict__ w, const uint16_t* __restrict__ s,
                                  const uint16_t* __restrict__ b, const float* __restrict__ x, float* __restrict__ out,
                                  uint32_t row_begin, uint32_t row_end, uint32_t out_rows) {
    extern __shared__ float terms[];          // [rows_per_block][groups]
    // vector blockIdx.y: x row y of in_dim floats, out row y of out_rows floats
    x += (size_t)blockIdx.y * in_dim;
    out += (size_t)blockIdx.y * out_rows;
    const uint32_t groups = in_dim / kGroup;
    const uint32_t rpb = blockDim.x / groups;  // rows per block (>= 1)
    const uint32_t t = threadIdx.x;
    const uint32_t lr = t / groups, g = t - lr * groups;
    const uint32_t row = row_begin + blockIdx.x * rpb + lr;
    if (lr < rpb && row < row_end) {
        const float* xg = x + (size_t)g * kGroup;
        float dot = 0.0f, sum = 0.0f;
        if (BITS == 4) {
            const uint4* wq = reinterpret_cast<const uint4*>(w + (size_t)row * (in_dim / 2) + (size_t)g * 32);
            const uint4 q0 = __ldg(wq), q1 = __ldg(wq + 1);
            const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
            for (int j = 0; j < 32; ++j) {        // byte j holds elements 2j (low) and 2j+1 (high)
                const uint32_t byte = (words[j >> 2] >> (8 * (j & 3))) & 0xFFu;
                const float x0 = __ldg(xg + 2 * j), x1 = __ldg(xg + 2 * j + 1);
                dot = __fadd_rn(dot, __fmul_rn((float)(byte & 0x0Fu), x0));
                dot = __fadd_rn(dot, __fmul_rn((float)(byte >> 4), x1));
                sum = __fadd_rn(sum, __fadd_rn(x0, x1));
            }
        } else {
            const uint4* wq = reinterpret_cast<const uint4*>(w + (size_t)row * in_dim + (size_t)g * 64);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 q = __ldg(wq + i);
                const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float xv = __ldg(xg + 16 * i + j);
                    dot = __fadd_rn(dot, __fmul_rn((float)((words[j >> 2] >> (8 * (j & 3))) & 0xFFu), xv));
                    sum = __fadd_rn(sum, xv);
                }
            }
        }
        const size_t si = (size_t)row * groups + g;
        terms[lr * groups + g] = __fadd_rn(__fmul_rn(bf16f(__ldg(s + si)), dot), __fmul_rn(bf16f(__ldg(b + si)), sum));
    }
    __syncthreads();
    if (t < rpb) {
        const uint32_t r = row_begin + blockIdx.x * rpb + t;
        if (r < row_end) {
            float acc = 0.0f;
            for (uint32_t gg = 0; gg < groups; ++gg) acc = __fadd_rn(acc, terms[t * groups + gg]);
            out[r] = acc;
        }
    }
}

// int4 rows of n vectors (gtm_gemv_q4_rows): the same arithmetic, in the same order, as
// gemv_exact_kernel<4> for each vector, mapped for the load path. A thread owns (group g, vector
// v): the group's 64 inputs of its vector in registers and their sum taken once in the reference's
// order (x0 + x1 per byte, then accumulated); it then walks GR rows, loading only their 32 bytes
// of packed weights (shared through L1 by the block's GV vector threads) and running the group's
// products in element order. The (row, vector) sums over the groups, in group order, follow.
constexpr int GV = 4, GR = 16;
__global__ void gemv_exact_rows4_kernel(uint32_t in_dim, uint32_t n, const uint8_t* __restrict__ w,
                                        const uint16_t* __restrict__ s, const uint16_t* __restrict__ b,
                                        const float* __restrict__ x, float* __restrict__ out, uint32_t rows) {
    extern __shared__ float terms[];   // [GR][GV][groups]
    const uint32_t groups = in_dim / kGroup;
    const uint32_t t = threadIdx.x, v = t / groups, g = t - v * groups;
    const uint32_t row0 = blockIdx.x * GR, vv = blockIdx.y * GV + v;
    const uint32_t nr = min((uint32_t)GR, rows - row0);
    const bool live = vv < n;
    float xr[kGroup];
    float gsum = 0.0f;
    if (live) {
        const float4* x4 = reinterpret_cast<const float4*>(x + (size_t)vv * in_dim + (size_t)g * kGroup);
#pragma unroll
        for (int c = 0; c < kGroup / 4; ++c) {
            const float4 q = __ldg(x4 + c);
            xr[4 * c] = q.x; xr[4 * c + 1] = q.y; xr[4 * c + 2] = q.z; xr[4 * c + 3] = q.w;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) gsum = __fadd_rn(gsum, __fadd_rn(xr[2 * j], xr[2 * j + 1]));
        for (uint32_t r = 0; r < nr; ++r) {
            const uint32_t row = row0 + r;
            const uint4* wq = reinterpret_cast<const uint4*>(w + (size_t)row * (in_dim / 2) + (size_t)g * 32);
            const uint4 q0 = __ldg(wq), q1 = __ldg(wq + 1);
            const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            float dot = 0.0f;
#pragma unroll
            for (int j = 0; j < 32; ++j) {   // byte j holds elements 2j (low) and 2j + 1 (high)
                const uint32_t byte = (words[j >> 2] >> (8 * (j & 3))) & 0xFFu;
                dot = __fadd_rn(dot, __fmul_rn((float)(byte & 0x0Fu), xr[2 * j]));
                dot = __fadd_rn(dot, __fmul_rn((float)(byte >> 4), xr[2 * j + 1]));
            }
            const size_t si = (size_t)row * groups + g;
            terms[((size_t)r * GV + v) * groups + g] =
                __fadd_rn(__fmul_rn(bf16f(__ldg(s + si)), dot), __fmul_rn(bf16f(__ldg(b + si)), gsum));
        }
    }
    __syncthreads();
    if (t < GR * GV) {   // (row, vector): the group terms in group order
        const uint32_t r = t / GV, v2 = t - r * GV, vo = blockIdx.y * GV + v2;
        if (r < nr && vo < n) {
            const float* tp = terms + ((size_t)r * GV + v2) * groups;
            float acc = 0.0f;
#pragma unroll 4
            for (uint32_t gg = 0; gg < groups; ++gg) acc = __fadd_rn(acc, tp[gg]);
            out[(size_t)vo * rows + row0 + r] = acc;
        }
    }
}

// Grids for in_dim / 64 groups with GV x groups <= 1024 threads and GR x GV x groups floats of
// shared memory <= 48 KB (in_dim <= 12288); the caller takes gemv_exact_kernel otherwise.
bool k_gemv_exact_rows4(uint32_t rows, uint32_t in_dim, uint32_t n, const void* w, const uint16_t* s, const uint16_t* b,
                        const float* x, float* out, cudaStream_t st) {
    const uint32_t groups = in_dim / kGroup;
    const size_t smem = sizeof(float) * (size_t)GR * GV * groups;
    if (GV * groups > 1024 || smem > 48 * 1024) return false;
    const dim3 grid((rows + GR - 1) / GR, (n + GV - 1) / GV);
    gemv_exact_rows4_kernel<<<grid, GV * groups, smem, st>>>(in_dim, n, (const uint8_t*)w, s, b, x, out, rows);
    return true;
}

void k_gemv_exact(int bits, uint32_t rows, uint32_t in_dim, const void* w, const uint16_t* s, const uint16_t* b,
                  const float* x, float* out, uint32_t row_begin, uint32_t row_end, cudaStream_t st, uint32_t nvec) {
    const uint32_t groups = in_dim / kGroup;
    const uint32_t threads = groups >= 256 ? groups : (256 / groups) * groups;
    const uint32_t rpb = threads / groups;
    const uint32_t n = row_end - row_begin;
    const dim3 grid((n + rpb - 1) / rpb, nvec);
    const size_t smem = sizeof(float) * threads;
    if (bits == 4)
        gemv_exact_kernel<4><<<grid, threads, smem, st>>>(in_dim, (const uint8_t*)w, s, b, x, out, row_begin, row_end,
                                                          rows);
    else
        gemv_exact_kernel<8><<<grid, threads, smem, st>>>(in_dim, (const uint8_t*)w, s, b, x, out, row_begin, row_end,
                                                          rows);
}

// ---- RouterTopK -------------------------------------------------------------------------------
// One warp: k rounds of a (value desc, index asc) arg-max over the lanes' logits, then the
// softmax over the k selected times per_expert_scale (src/cpu_reference.cpp:447-480).
__global__ void router_topk_kernel(uint32_t n, uint32_t k, const float* __restrict__ logits,
                                   const uint16_t* __restrict__ pes, uint32_t* __restrict__ idx,
                                   float* __restrict__ wout) {
    const int lane = threadIdx.x;
    constexpr int kPer = 32;                   // up to 1024 experts
    float v[kPer];
    uint32_t taken = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const uint32_t e = lane + 32u * j;
        v[j] = e < n ? logits[e] : 0.0f;
    }
    __shared__ float sel[32];
    __shared__ uint32_t seli[32];
    const uint32_t kNone = 0xFFFFFFFFu;
    for (uint32_t r = 0; r < k; ++r) {
        float bv = 0.0f;
        uint32_t bi = kNone;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const uint32_t e = lane + 32u * j;
            if (e < n && !(taken & (1u << j)) && (bi == kNone || v[j] > bv || (v[j] == bv && e < bi))) { bv = v[j]; bi = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != kNone && (bi == kNone || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
        }
        if ((bi & 31u) == (uint32_t)lane) taken |= 1u << (bi >> 5);
        if (lane == 0) { sel[r] = bv; seli[r] = bi; }
    }
    __syncwarp();
    if (lane == 0) {
        float e[32], sum = 0.0f;
        for (uint32_t r = 0; r < k; ++r) { e[r] = expf(__fsub_rn(sel[r], sel[0])); sum = __fadd_rn(sum, e[r]); }
        for (uint32_t r = 0; r < k; ++r) {
            idx[r] = seli[r];
            wout[r] = __fmul_rn(__fdiv_rn(e[r], sum), bf16f(pes[seli[r]]));
        }
    }
}

void k_router_topk(uint32_t n, uint32_t k, const float* logits, const uint16_t* pes, uint32_t* idx, float* w,
                   cudaStream_t st) {
    router_topk_kernel<<<1, 32, 0, st>>>(n, k, logits, pes, idx, w);
}

// ---- elementwise ------------------------------------------------------------------------------
__device__ __forceinline__ float gelu_tanh_ref(float x) {
    // 0.5f * x * (1 + tanh(k0 * (x + k1 * x * x * x))), evaluated left to right as written
    const float inner = __fmul_rn(0.7978845608028654f, __fadd_rn(x, __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

__global__ void geglu_kernel(uint32_t n, const float* g, const float* u, float* out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __fmul_rn(gelu_tanh_ref(g[i]), u[i]);
}
void k_geglu(uint32_t n, const float* g, const float* u, float* out, cudaStream_t st) {
    geglu_kernel<<<(n + 255) / 256, 256, 0, st>>>(n, g, u, out);
}

__global__ void scale_accum_kernel(uint32_t n, const float* in, const float* w, uint32_t wi, int acc, float* out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = __fmul_rn(w[wi], in[i]);
    out[i] = acc ? __fadd_rn(out[i], v) : v;
}
void k_scale_accum(uint32_t n, const float* in, const float* w, uint32_t wi, int acc, float* out, cudaStream_t st) {
    scale_accum_kernel<<<(n + 255) / 256, 256, 0, st>>>(n, in, w, wi, acc, out);
}

__global__ void mul_bf16_kernel(uint32_t n, const float* in, const uint16_t* w, float scale, float* out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __fmul_rn(__fmul_rn(in[i], bf16f(w[i])), scale);
}
void k_mul_bf16(uint32_t n, const float* in, const uint16_t* w, float scale, float* out, cudaStream_t st) {
    mul_bf16_kernel<<<(n + 255) / 256, 256, 0, st>>>(n, in, w, scale, out);
}

// ---- RMSNormK / PostAttn / LayerTail: one CTA, vector staged in shared memory ------------------
constexpr int kNormThreads = 1024;

__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(uint32_t n, const float* x, const uint16_t* w, float eps,
                                                               float* out) {
    extern __shared__ float sx[];
    __shared__ double red[40];
    x += (size_t)blockIdx.x * n;     // row blockIdx.x
    out += (size_t)blockIdx.x * n;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) sx[i] = x[i];
    __syncthreads();
    const float inv = exact_rms_inv(sx, (int)n, eps, red);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = __fmul_rn(sx[i], inv);
        out[i] = w ? __fmul_rn(v, bf16f(w[i])) : v;
    }
}
void k_rmsnorm(uint32_t n, const float* x, const uint16_t* w, float eps, float* out, cudaStream_t st, uint32_t rows) {
    rmsnorm_kernel<<<rows, kNormThreads, sizeof(float) * n, st>>>(n, x, w, eps, out);
}

// src/cpu_reference.cpp:423-434 (the reference's PostAttn shader fuses the same steps).
__global__ void __launch_bounds__(kNormThreads) post_attn_kernel(uint32_t d, const float* attn, const float* hidden,
                                                                 const uint16_t* wpost, const uint16_t* wpre,
                                                                 const uint16_t* wpre2, float eps, float* hout,
                                                                 float* dense, float* routed, float* router) {
    extern __shared__ float sm[];
    float* sa = sm;
    float* sh = sm + d;
    __shared__ double red[40];
    const size_t r = (size_t)blockIdx.x * d;   // row blockIdx.x of every vector
    attn += r;
    hidden += r;
    hout += r;
    if (dense) dense += r;
    if (routed) routed += r;
    if (router) router += r;
    for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) { sa[i] = attn[i]; sh[i] = hidden[i]; }
    __syncthreads();
    const float ainv = exact_rms_inv(sa, (int)d, eps, red);
    for (uint32_t i = threadIdx.x; i < d; i += blockDim.x)
        sh[i] = __fadd_rn(sh[i], __fmul_rn(__fmul_rn(sa[i], ainv), bf16f(wpost[i])));
    __syncthreads();
    const float hinv = exact_rms_inv(sh, (int)d, eps, red);
    for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) {
        const float h = __fmul_rn(sh[i], hinv);
        hout[i] = sh[i];
        if (dense) dense[i] = __fmul_rn(h, bf16f(wpre[i]));
        if (routed) routed[i] = __fmul_rn(h, bf16f(wpre2[i]));
        if (router) router[i] = h;
    }
}
void k_post_attn(uint32_t d, const float* attn, const float* hidden, const uint16_t* wpost, const uint16_t* wpre,
                 const uint16_t* wpre2, float eps, float* hout, float* dense, float* routed, float* router,
                 cudaStream_t st, uint32_t rows) {
    post_attn_kernel<<<rows, kNormThreads, 2 * sizeof(float) * d, st>>>(d, attn, hidden, wpost, wpre, wpre2, eps, hout,
                                                                        dense, routed, router);
}

// src/cpu_reference.cpp:512-520.
__global__ void __launch_bounds__(kNormThreads) layer_tail_kernel(uint32_t d, const float* h2, const float* h1,
                                                                  const float* hidden, const uint16_t* wpf2,
                                                                  const uint16_t* wpf, float eps, float ls, float* hout) {
    extern __shared__ float sm[];
    float* s2 = sm;
    float* st = sm + d;
    __shared__ double red[40];
    for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) s2[i] = h2[i];
    __syncthreads();
    const float i2 = exact_rms_inv(s2, (int)d, eps, red);
    for (uint32_t i = threadIdx.x; i < d; i += blockDim.x)
        st[i] = __fadd_rn(__fmul_rn(__fmul_rn(s2[i], i2), bf16f(wpf2[i])), h1[i]);
    __syncthreads();
    const float i12 = exact_rms_inv(st, (int)d, eps, red);
    for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) {
        const float t2 = __fmul_rn(__fmul_rn(st[i], i12), bf16f(wpf[i]));
        hout[i] = __fmul_rn(__fadd_rn(hidden[i], t2), ls);
    }
}
void k_layer_tail(uint32_t d, const float* h2, const float* h1, const float* hidden, const uint16_t* wpf2,
                  const uint16_t* wpf, float eps, float ls, float* hout, cudaStream_t st) {
    layer_tail_kernel<<<1, kNormThreads, 2 * sizeof(float) * d, st>>>(d, h2, h1, hidden, wpf2, wpf, eps, ls, hout);
}

}  // namespace gtm

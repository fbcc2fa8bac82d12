// Batch-1 decode around the MoE block (include/gtmoe_attention.h): embedding lookup, the per-head
// q/k/v epilogue, and attention over the FP32 ring KV cache.
//
// Attention is split over positions (flash-decoding): att_partial runs one CTA per (kv head,
// position chunk); the CTA keeps the q rows of the kv head's query group in shared memory,
// scores its positions one warp per position (float4 K reads), and writes, per query head, the
// chunk's max score, its sum of exp(score - max) and its exp-weighted V sum. att_combine merges
// the chunks of each query head. Both read K and V once, so the kernel is bound by HBM: per
// token and layer 2 * (n_pos - first) * kv_heads * head_dim * 4 bytes.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "gtm_internal.h"
#include "gtmoe_attention.h"

namespace gtm {
namespace {

constexpr int kAttThreads = 256;
constexpr int kMaxGroup = 8;        // query heads per kv head
constexpr int kMaxHeadDim = 512;
constexpr int kMaxChunk = 256;      // positions per att_partial CTA
constexpr int kTargetCtas = 296;    // two per SM on 148 SMs

__device__ __forceinline__ float bf16f(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }

// ---- EmbedLookup ------------------------------------------------------------------------------
__device__ __forceinline__ float embed_elem(const uint8_t* __restrict__ w, const uint16_t* __restrict__ s,
                                            const uint16_t* __restrict__ b, uint32_t in_dim, uint32_t token, uint32_t c,
                                            float scale) {
    const uint32_t groups = in_dim / 64;
    const uint8_t byte = w[static_cast<size_t>(token) * (in_dim / 2) + (c >> 1)];
    const uint32_t q = (c & 1u) ? static_cast<uint32_t>(byte >> 4) : static_cast<uint32_t>(byte & 15u);
    const size_t g = static_cast<size_t>(token) * groups + c / 64;
    // (q * s + b) * scale with one rounding per operation, as the CPU reference evaluates it
    return __fmul_rn(__fadd_rn(__fmul_rn(static_cast<float>(q), bf16f(s[g])), bf16f(b[g])), scale);
}

__global__ void att_embed(const uint8_t* __restrict__ w, const uint16_t* __restrict__ s, const uint16_t* __restrict__ b,
                          uint32_t in_dim, uint32_t token, float scale, float* __restrict__ out) {
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c < in_dim) out[c] = embed_elem(w, s, b, in_dim, token, c, scale);
}

// Per-row values of a *_rows launch, passed by value (no host-to-device copy, checked on the host).
struct RowVals {
    uint32_t v[kMaxBatchRows];
};

// Row blockIdx.y: token tok.v[y] into out row y.
__global__ void att_embed_rows(const uint8_t* __restrict__ w, const uint16_t* __restrict__ s,
                               const uint16_t* __restrict__ b, uint32_t in_dim, float scale, float* __restrict__ out,
                               const __grid_constant__ RowVals tok) {
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c < in_dim) out[(size_t)blockIdx.y * in_dim + c] = embed_elem(w, s, b, in_dim, tok.v[blockIdx.y], c, scale);
}

// ---- QKVEpilogue: one CTA per head ------------------------------------------------------------
// `in` and `out` may be the same buffer (no __restrict__): every read of a head's input happens
// before the CTA's first barrier, every write after it.
__device__ __forceinline__ void epilogue_head(const float* src, const uint16_t* __restrict__ w, uint32_t head_dim,
                                              float eps, uint32_t pairs, float position, float theta, float* dst) {
    __shared__ float x[kMaxHeadDim];
    __shared__ double red[kAttThreads / 32];
    double a = 0.0;
    for (uint32_t i = threadIdx.x; i < head_dim; i += blockDim.x) {
        const float v = src[i];
        x[i] = v;
        a += static_cast<double>(v) * static_cast<double>(v);
    }
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
    __syncthreads();   // also publishes x: in and out may alias, so every read of src is done
    double acc = 0.0;
    for (int i = 0; i < kAttThreads / 32; ++i) acc += red[i];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(acc / static_cast<double>(head_dim)), eps)));
    for (uint32_t i = threadIdx.x; i < head_dim; i += blockDim.x) {
        const float v = __fmul_rn(x[i], inv);
        x[i] = w ? __fmul_rn(v, bf16f(w[i])) : v;
    }
    __syncthreads();
    const uint32_t half = head_dim / 2;
    for (uint32_t i = threadIdx.x; i < half; i += blockDim.x) {
        float y0 = x[i], y1 = x[i + half];
        if (i < pairs) {
            const float freq = powf(theta, __fdiv_rn(-static_cast<float>(2 * i), static_cast<float>(head_dim)));
            const float ang = __fmul_rn(position, freq);
            const float cs = cosf(ang), sn = sinf(ang);
            const float r0 = __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
            const float r1 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, cs));
            y0 = r0;
            y1 = r1;
        }
        dst[i] = y0;
        dst[i + half] = y1;
    }
}

__global__ void __launch_bounds__(kAttThreads) att_epilogue(const float* in, const uint16_t* __restrict__ w,
                                                            uint32_t head_dim, float eps, uint32_t pairs,
                                                            float position, float theta, float* out) {
    epilogue_head(in + static_cast<size_t>(blockIdx.x) * head_dim, w, head_dim, eps, pairs, position, theta,
                  out + static_cast<size_t>(blockIdx.x) * head_dim);
}

// Head blockIdx.x of row blockIdx.y at position pos.v[y]: the input row is in + y * heads *
// head_dim; the output row is the same place of `out` when capacity is 0, else ring row
// pos % capacity of sequence seq.v[y]'s cache, which starts at out + seq * capacity * heads * head_dim.
__global__ void __launch_bounds__(kAttThreads) att_epilogue_rows(const float* in, const uint16_t* __restrict__ w,
                                                                 uint32_t head_dim, float eps, uint32_t pairs,
                                                                 float theta, float* out, uint32_t capacity,
                                                                 const __grid_constant__ RowVals pos,
                                                                 const __grid_constant__ RowVals seq) {
    const size_t row = static_cast<size_t>(gridDim.x) * head_dim;
    const uint32_t y = blockIdx.y, p = pos.v[y];
    const size_t out_row = capacity ? (static_cast<size_t>(seq.v[y]) * capacity + p % capacity) : y;
    epilogue_head(in + y * row + static_cast<size_t>(blockIdx.x) * head_dim, w, head_dim, eps, pairs,
                  static_cast<float>(p), theta, out + out_row * row + static_cast<size_t>(blockIdx.x) * head_dim);
}

// ---- Attention, split over positions ----------------------------------------------------------
struct AttArgs {
    const float* q;
    const float* kc;
    const float* vc;
    float* part;       // [q_heads][splits][head_dim + 2]: o, then m, then l
    uint32_t q_heads, kv_heads, head_dim, n_pos, first, capacity, chunk, splits;
    uint32_t window;   // rows launches: attended positions (0 = all)
};

// Positions [first, n_pos) split into chunks of `chunk`, about kTargetCtas CTAs over the kv heads.
struct Plan {
    uint32_t chunk, splits;
};
__host__ __device__ __forceinline__ Plan plan(uint32_t kv_heads, uint32_t window) {
    const uint32_t t = (kTargetCtas + kv_heads - 1) / kv_heads;
    const uint32_t target = t > 1 ? t : 1;
    uint32_t chunk = (window + target - 1) / target;
    chunk = chunk < 1 ? 1 : (chunk > static_cast<uint32_t>(kMaxChunk) ? kMaxChunk : chunk);
    return {chunk, (window + chunk - 1) / chunk};
}

// One CTA's chunk of positions for kv head kvh: q of the row's query heads, the row's caches, and
// its partials part [q_heads][splits][HD + 2].
template <int HD>
__device__ __forceinline__ void partial_chunk(const float* q, const float* kc, const float* vc, float* part,
                                              uint32_t q_heads, uint32_t kv_heads, uint32_t capacity, uint32_t chunk,
                                              uint32_t splits, uint32_t n_pos, uint32_t first, uint32_t kvh,
                                              uint32_t split) {
    constexpr int V4 = HD / 128;   // float4s per lane in a K row
    __shared__ __align__(16) float qs[kMaxGroup * HD];
    __shared__ float sc[kMaxGroup * kMaxChunk];
    __shared__ float mx_s[kMaxGroup], sum_s[kMaxGroup];
    struct {
        const float *q, *kc, *vc;
        float* part;
        uint32_t capacity, splits;
    } a{q, kc, vc, part, capacity, splits};
    const int grp = static_cast<int>(q_heads / kv_heads);
    const uint32_t row = kv_heads * HD;
    const uint32_t t0 = first + split * chunk;
    const uint32_t t1 = min(n_pos, t0 + chunk);
    const int n = t1 > t0 ? static_cast<int>(t1 - t0) : 0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    for (int i = threadIdx.x; i < grp * HD; i += blockDim.x) qs[i] = a.q[static_cast<size_t>(kvh) * grp * HD + i];
    __syncthreads();

    // scores: one warp per position
    for (int j = warp; j < n; j += kAttThreads / 32) {
        const uint32_t slot = (t0 + j) % a.capacity;
        const float4* k4 = reinterpret_cast<const float4*>(a.kc + static_cast<size_t>(slot) * row + kvh * HD);
        float4 kv[V4];
#pragma unroll
        for (int u = 0; u < V4; ++u) kv[u] = __ldg(k4 + lane + 32 * u);
        for (int g = 0; g < grp; ++g) {
            const float4* q4 = reinterpret_cast<const float4*>(qs + g * HD);
            float d = 0.0f;
#pragma unroll
            for (int u = 0; u < V4; ++u) {
                const float4 qq = q4[lane + 32 * u];
                d += qq.x * kv[u].x + qq.y * kv[u].y + qq.z * kv[u].z + qq.w * kv[u].w;
            }
            for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            if (lane == 0) sc[g * kMaxChunk + j] = d;
        }
    }
    __syncthreads();
    // per query head: the chunk's max and exp weights (warp g handles head g)
    if (warp < grp) {
        const int g = warp;
        float m = -INFINITY;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[g * kMaxChunk + j]);
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int j = lane; j < n; j += 32) {
            const float e = expf(sc[g * kMaxChunk + j] - m);
            sc[g * kMaxChunk + j] = e;
            l += e;
        }
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) {
            mx_s[g] = m;
            sum_s[g] = l;
        }
    }
    __syncthreads();
    // weighted V: each thread owns dims d and d + 256 (coalesced V rows)
    float acc[kMaxGroup][2];
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) acc[g][0] = acc[g][1] = 0.0f;
    for (int j = 0; j < n; ++j) {
        const uint32_t slot = (t0 + j) % a.capacity;
        const float* vr = a.vc + static_cast<size_t>(slot) * row + kvh * HD;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int d = threadIdx.x + r * kAttThreads;
            if (d < HD) {
                const float v = __ldg(vr + d);
#pragma unroll
                for (int g = 0; g < kMaxGroup; ++g)
                    if (g < grp) acc[g][r] += sc[g * kMaxChunk + j] * v;
            }
        }
    }
    const size_t stride = HD + 2;
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
        if (g >= grp) break;
        float* p = a.part + (static_cast<size_t>(kvh * grp + g) * a.splits + split) * stride;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int d = threadIdx.x + r * kAttThreads;
            if (d < HD) p[d] = acc[g][r];
        }
        if (threadIdx.x == 0) {
            p[HD] = mx_s[g];
            p[HD + 1] = sum_s[g];
        }
    }
}

template <int HD>
__global__ void __launch_bounds__(kAttThreads) att_partial(AttArgs a) {
    partial_chunk<HD>(a.q, a.kc, a.vc, a.part, a.q_heads, a.kv_heads, a.capacity, a.chunk, a.splits, a.n_pos, a.first,
                      blockIdx.x, blockIdx.y);
}

// Row blockIdx.z: sequence seq.v[z] at position pos.v[z] attends [first, pos] of its own caches
// (kc + seq * capacity * kv_heads * HD), with the chunking a single call on that row would use,
// so each row's result is bit-identical to gtm_attention_decode on it. a.splits is the largest
// row's count (the grid); a row's surplus CTAs return at once.
__host__ __device__ __forceinline__ uint32_t row_first(uint32_t n_pos, uint32_t window) {
    return window && n_pos > window ? n_pos - window : 0;
}
template <int HD>
__global__ void __launch_bounds__(kAttThreads) att_partial_rows(AttArgs a, const __grid_constant__ RowVals seq,
                                                                const __grid_constant__ RowVals pos) {
    const uint32_t z = blockIdx.z;
    const uint32_t n_pos = pos.v[z] + 1, first = row_first(n_pos, a.window);
    const Plan pl = plan(a.kv_heads, n_pos - first);
    if (blockIdx.y >= pl.splits) return;
    const size_t cache = static_cast<size_t>(seq.v[z]) * a.capacity * a.kv_heads * HD;
    partial_chunk<HD>(a.q + static_cast<size_t>(z) * a.q_heads * HD, a.kc + cache, a.vc + cache,
                      a.part + static_cast<size_t>(z) * a.q_heads * a.splits * (HD + 2), a.q_heads, a.kv_heads,
                      a.capacity, pl.chunk, a.splits, n_pos, first, blockIdx.x, blockIdx.y);
}

// One CTA per query head (and row blockIdx.y of a rows launch): merge the chunks' (max, sum,
// weighted V). `splits` is the row's own chunk count, `stride_splits` the partials' layout.
__device__ __forceinline__ void combine_head(const float* p, uint32_t splits, uint32_t hd, float* out) {
    const size_t stride = hd + 2;
    float m = -INFINITY;
    for (uint32_t s = 0; s < splits; ++s) m = fmaxf(m, p[s * stride + hd]);
    float l = 0.0f, o = 0.0f;
    const uint32_t d = threadIdx.x;
    for (uint32_t s = 0; s < splits; ++s) {
        const float ms = p[s * stride + hd];
        if (ms == -INFINITY) continue;   // an empty chunk
        const float f = expf(ms - m);
        l += p[s * stride + hd + 1] * f;
        if (d < hd) o += p[s * stride + d] * f;
    }
    if (d < hd) out[d] = o / l;
}
__global__ void __launch_bounds__(kMaxHeadDim) att_combine(AttArgs a, float* __restrict__ ctx) {
    const uint32_t h = blockIdx.x, hd = a.head_dim;
    combine_head(a.part + static_cast<size_t>(h) * a.splits * (hd + 2), a.splits, hd, ctx + static_cast<size_t>(h) * hd);
}
__global__ void __launch_bounds__(kMaxHeadDim) att_combine_rows(AttArgs a, float* __restrict__ ctx,
                                                                const __grid_constant__ RowVals pos) {
    const uint32_t h = blockIdx.x, y = blockIdx.y, hd = a.head_dim;
    const uint32_t n_pos = pos.v[y] + 1;
    const Plan pl = plan(a.kv_heads, n_pos - row_first(n_pos, a.window));
    const float* p = a.part + (static_cast<size_t>(y) * a.q_heads + h) * a.splits * (hd + 2);
    combine_head(p, pl.splits, hd, ctx + (static_cast<size_t>(y) * a.q_heads + h) * hd);
}
uint32_t max_splits(uint32_t window) {
    return std::max<uint32_t>(kTargetCtas, (window + kMaxChunk - 1) / kMaxChunk);
}
bool aligned_to(const void* p, size_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

}  // namespace
}  // namespace gtm

using namespace gtm;

extern "C" {

GTM_API int gtm_embed_lookup(uint32_t rows, uint32_t in_dim, const void* w, const uint16_t* s, const uint16_t* b,
                             uint32_t token, float scale, float* out, void* stream) {
    const char* fn = "gtm_embed_lookup";
    if (!w || !s || !b || !out) return set_error(GTM_ERR_INVALID, "%s: null pointer", fn);
    if (in_dim == 0 || in_dim % 64 != 0) return set_error(GTM_ERR_INVALID, "%s: in_dim %u (multiple of 64)", fn, in_dim);
    if (token >= rows)   // cpu_reference.cpp:324-326
        return set_error(GTM_ERR_INVALID, "%s: token id %u out of vocabulary (%u rows)", fn, token, rows);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    att_embed<<<(in_dim + 255) / 256, 256, 0, st>>>(static_cast<const uint8_t*>(w), s, b, in_dim, token, scale, out);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(fn, e);
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_qkv_epilogue(uint32_t heads, uint32_t head_dim, const float* in, const uint16_t* w, float eps,
                             uint32_t rotated_pairs, uint32_t position, float theta, float* out, void* stream) {
    const char* fn = "gtm_qkv_epilogue";
    if (!in || !out) return set_error(GTM_ERR_INVALID, "%s: null pointer", fn);
    if (heads == 0 || (head_dim != 128 && head_dim != 256 && head_dim != 512))
        return set_error(GTM_ERR_UNSUPPORTED, "%s: heads=%u head_dim=%u (head_dim 128, 256 or 512)", fn, heads, head_dim);
    if (rotated_pairs > head_dim / 2)
        return set_error(GTM_ERR_INVALID, "%s: rotated_pairs %u > head_dim / 2", fn, rotated_pairs);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    att_epilogue<<<heads, kAttThreads, 0, st>>>(in, w, head_dim, eps, rotated_pairs, static_cast<float>(position), theta,
                                                out);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(fn, e);
    clear_error();
    return GTM_OK;
}

GTM_API size_t gtm_attention_workspace_bytes(uint32_t q_heads, uint32_t head_dim, uint32_t max_window) {
    if (q_heads == 0 || head_dim == 0 || head_dim > static_cast<uint32_t>(kMaxHeadDim) || max_window == 0) return 0;
    return static_cast<size_t>(q_heads) * max_splits(max_window) * (head_dim + 2) * sizeof(float);
}

GTM_API int gtm_attention_decode(uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim, uint32_t n_pos, uint32_t first,
                                 uint32_t capacity, const float* q, const float* kc, const float* vc, float* ctx, void* ws,
                                 size_t ws_bytes, void* stream) {
    const char* fn = "gtm_attention_decode";
    if (!q || !kc || !vc || !ctx) return set_error(GTM_ERR_INVALID, "%s: null pointer", fn);
    if (kv_heads == 0 || q_heads % kv_heads != 0 || q_heads / kv_heads > static_cast<uint32_t>(kMaxGroup))
        return set_error(GTM_ERR_UNSUPPORTED, "%s: q_heads %u / kv_heads %u (a group of 1..%d)", fn, q_heads, kv_heads,
                         kMaxGroup);
    if (head_dim != 128 && head_dim != 256 && head_dim != 512)
        return set_error(GTM_ERR_UNSUPPORTED, "%s: head_dim %u (128, 256 or 512)", fn, head_dim);
    if (first >= n_pos || capacity == 0 || n_pos - first > capacity)
        return set_error(GTM_ERR_INVALID, "%s: positions [%u, %u) do not fit a ring of %u rows", fn, first, n_pos,
                         capacity);
    if (!aligned_to(q, 16) || !aligned_to(kc, 16) || !aligned_to(vc, 16) || !aligned_to(ws, 16))
        return set_error(GTM_ERR_MISALIGNED, "%s: q, caches and workspace need 16-byte alignment", fn);
    const uint32_t window = n_pos - first;
    const size_t need = gtm_attention_workspace_bytes(q_heads, head_dim, window);
    if (!ws || ws_bytes < need) return set_error(GTM_ERR_WORKSPACE, "%s: workspace needs %zu bytes", fn, need);
    const Plan pl = plan(kv_heads, window);
    AttArgs a;
    a.q = q;
    a.kc = kc;
    a.vc = vc;
    a.part = static_cast<float*>(ws);
    a.q_heads = q_heads;
    a.kv_heads = kv_heads;
    a.head_dim = head_dim;
    a.n_pos = n_pos;
    a.first = first;
    a.capacity = capacity;
    a.chunk = pl.chunk;
    a.splits = pl.splits;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const dim3 grid(kv_heads, pl.splits);
    if (head_dim == 128)
        att_partial<128><<<grid, kAttThreads, 0, st>>>(a);
    else if (head_dim == 256)
        att_partial<256><<<grid, kAttThreads, 0, st>>>(a);
    else
        att_partial<512><<<grid, kAttThreads, 0, st>>>(a);
    att_combine<<<q_heads, kMaxHeadDim, 0, st>>>(a, ctx);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(fn, e);
    clear_error();
    return GTM_OK;
}

// ---- the same entries over many sequences at once (batched decode) ------------------------------

static int rows_common(const char* fn, uint32_t n) {
    if (n > kMaxBatchRows) return set_error(GTM_ERR_INVALID, "%s: n=%u rows (at most %u)", fn, n, kMaxBatchRows);
    return GTM_OK;
}

GTM_API int gtm_embed_lookup_rows(uint32_t rows, uint32_t in_dim, const void* w, const uint16_t* s, const uint16_t* b,
                                  const uint32_t* tokens, uint32_t n, float scale, float* out, void* stream) {
    const char* fn = "gtm_embed_lookup_rows";
    if (n == 0) { clear_error(); return GTM_OK; }
    int rc = rows_common(fn, n);
    if (rc) return rc;
    if (!w || !s || !b || !out || !tokens) return set_error(GTM_ERR_INVALID, "%s: null pointer", fn);
    if (in_dim == 0 || in_dim % 64 != 0) return set_error(GTM_ERR_INVALID, "%s: in_dim %u (multiple of 64)", fn, in_dim);
    RowVals tok;
    for (uint32_t i = 0; i < n; ++i) {
        if (tokens[i] >= rows)   // cpu_reference.cpp:324-326
            return set_error(GTM_ERR_INVALID, "%s: token id %u of row %u out of vocabulary (%u rows)", fn, tokens[i], i,
                             rows);
        tok.v[i] = tokens[i];
    }
    att_embed_rows<<<dim3((in_dim + 255) / 256, n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(w), s, b, in_dim, scale, out, tok);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(fn, e);
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_qkv_epilogue_rows(uint32_t heads, uint32_t head_dim, uint32_t n, const float* in, const uint16_t* w,
                                  float eps, uint32_t rotated_pairs, const uint32_t* positions, float theta, float* out,
                                  const uint32_t* seqs, uint32_t num_seqs, uint32_t capacity, void* stream) {
    const char* fn = "gtm_qkv_epilogue_rows";
    if (n == 0) { clear_error(); return GTM_OK; }
    int rc = rows_common(fn, n);
    if (rc) return rc;
    if (!in || !out || !positions || (capacity && !seqs)) return set_error(GTM_ERR_INVALID, "%s: null pointer", fn);
    if (heads == 0 || (head_dim != 128 && head_dim != 256 && head_dim != 512))
        return set_error(GTM_ERR_UNSUPPORTED, "%s: heads=%u head_dim=%u (head_dim 128, 256 or 512)", fn, heads, head_dim);
    if (rotated_pairs > head_dim / 2)
        return set_error(GTM_ERR_INVALID, "%s: rotated_pairs %u > head_dim / 2", fn, rotated_pairs);
    RowVals pos, seq;
    for (uint32_t i = 0; i < n; ++i) {
        pos.v[i] = positions[i];
        seq.v[i] = capacity ? seqs[i] : 0;
        if (capacity && seqs[i] >= num_seqs)
            return set_error(GTM_ERR_INVALID, "%s: row %u names sequence %u of %u", fn, i, seqs[i], num_seqs);
    }
    att_epilogue_rows<<<dim3(heads, n), kAttThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        in, w, head_dim, eps, rotated_pairs, theta, out, capacity, pos, seq);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(fn, e);
    clear_error();
    return GTM_OK;
}

GTM_API size_t gtm_attention_rows_workspace_bytes(uint32_t q_heads, uint32_t head_dim, uint32_t max_window, uint32_t n) {
    if (n == 0 || n > kMaxBatchRows) return 0;
    return static_cast<size_t>(n) * gtm_attention_workspace_bytes(q_heads, head_dim, max_window);
}

GTM_API int gtm_attention_decode_rows(uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim, uint32_t n,
                                      uint32_t window, uint32_t capacity, const float* q, const float* kc,
                                      const float* vc, const uint32_t* seqs, uint32_t num_seqs,
                                      const uint32_t* positions, float* ctx, void* ws, size_t ws_bytes, void* stream) {
    const char* fn = "gtm_attention_decode_rows";
    if (n == 0) { clear_error(); return GTM_OK; }
    int rc = rows_common(fn, n);
    if (rc) return rc;
    if (!q || !kc || !vc || !ctx || !seqs || !positions) return set_error(GTM_ERR_INVALID, "%s: null pointer", fn);
    if (kv_heads == 0 || q_heads % kv_heads != 0 || q_heads / kv_heads > static_cast<uint32_t>(kMaxGroup))
        return set_error(GTM_ERR_UNSUPPORTED, "%s: q_heads %u / kv_heads %u (a group of 1..%d)", fn, q_heads, kv_heads,
                         kMaxGroup);
    if (head_dim != 128 && head_dim != 256 && head_dim != 512)
        return set_error(GTM_ERR_UNSUPPORTED, "%s: head_dim %u (128, 256 or 512)", fn, head_dim);
    if (!aligned_to(q, 16) || !aligned_to(kc, 16) || !aligned_to(vc, 16) || !aligned_to(ws, 16))
        return set_error(GTM_ERR_MISALIGNED, "%s: q, caches and workspace need 16-byte alignment", fn);
    RowVals seq, pos;
    uint32_t wmax = 1, splits = 1;
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t n_pos = positions[i] + 1, first = row_first(n_pos, window);
        if (capacity == 0 || n_pos - first > capacity || seqs[i] >= num_seqs || positions[i] == 0xFFFFFFFFu)
            return set_error(GTM_ERR_INVALID, "%s: row %u (sequence %u of %u, position %u) does not fit a ring of %u rows",
                             fn, i, seqs[i], num_seqs, positions[i], capacity);
        seq.v[i] = seqs[i];
        pos.v[i] = positions[i];
        wmax = std::max(wmax, n_pos - first);
        splits = std::max(splits, plan(kv_heads, n_pos - first).splits);   // not monotonic in the window
    }
    const size_t need = gtm_attention_rows_workspace_bytes(q_heads, head_dim, wmax, n);
    if (!ws || ws_bytes < need) return set_error(GTM_ERR_WORKSPACE, "%s: workspace needs %zu bytes", fn, need);
    AttArgs a;
    a.q = q;
    a.kc = kc;
    a.vc = vc;
    a.part = static_cast<float*>(ws);
    a.q_heads = q_heads;
    a.kv_heads = kv_heads;
    a.head_dim = head_dim;
    a.n_pos = 0;
    a.first = 0;
    a.capacity = capacity;
    a.chunk = 0;
    a.splits = splits;   // the partials' layout: the most chunks any row has (<= max_splits(wmax))
    a.window = window;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const dim3 grid(kv_heads, a.splits, n);
    if (head_dim == 128)
        att_partial_rows<128><<<grid, kAttThreads, 0, st>>>(a, seq, pos);
    else if (head_dim == 256)
        att_partial_rows<256><<<grid, kAttThreads, 0, st>>>(a, seq, pos);
    else
        att_partial_rows<512><<<grid, kAttThreads, 0, st>>>(a, seq, pos);
    att_combine_rows<<<dim3(q_heads, n), kMaxHeadDim, 0, st>>>(a, ctx, pos);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(fn, e);
    clear_error();
    return GTM_OK;
}

}  // extern "C"

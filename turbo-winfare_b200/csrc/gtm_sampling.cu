// Token sampling on the device (include/gtmoe_sampling.h): the reference's src/sampling.cpp with
// the logits left in HBM.
//
// sample_token runs as two launches over the fp32 logits:
//   smp_scan    one CTA per slice of at most kSliceMax ids: the slice's max logit, its sum of
//               exp(l - slice max) in double, and its best kList candidates, sorted, as 64-bit
//               keys (orderable logit << 32 | ~id: larger key = larger logit, then lower id,
//               which is the reference's candidate order, sampling.cpp:128-131);
//   smp_finish  one CTA: global max; greedy takes the best list head; otherwise the full
//               denominator from the slice sums, a radix select of the n-th best key over the
//               slices' lists, the sorted shortlist, and then the reference's sequential steps
//               (nucleus cut, top-k cut, temperature weights, one xorshift64* draw) on one thread.
// The repetition penalty is two launches over the history (count per id, then apply the count
// in one read-modify-write per id).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>

#include "gtm_internal.h"
#include "gtmoe_sampling.h"

namespace gtm {
namespace {

constexpr int kScanThreads = 512;
constexpr int kFinishThreads = 1024;
constexpr int kSliceMax = 4096;   // ids per scan CTA (keys sorted in shared memory)
constexpr int kList = 256;        // candidates kept per slice = the largest shortlist
constexpr int kMaxGrid = 1024;    // slices a workspace is sized for
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ULL;

__device__ __forceinline__ uint64_t cand_key(float v, uint32_t id) {
    const uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);   // -0 and +0 compare equal
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (static_cast<uint64_t>(ord) << 32) | static_cast<uint32_t>(~id);
}
__device__ __forceinline__ uint32_t key_id(uint64_t k) { return ~static_cast<uint32_t>(k); }

// Sorts n keys (n a power of two, >= 2) in shared memory into descending order.
__device__ void bitonic_desc(uint64_t* a, int n) {
    for (int size = 2; size <= n; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
                const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
                const bool desc = (lo & size) == 0;
                const uint64_t x = a[lo], y = a[hi];
                if ((x < y) == desc) {
                    a[lo] = y;
                    a[hi] = x;
                }
            }
        }
    __syncthreads();
}

// Block-wide reductions (blockDim a multiple of 32, at most 1024); every thread gets the result.
__device__ float block_max_f(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float r = red[0];
    for (int i = 1; i < nw; ++i) r = fmaxf(r, red[i]);
    return r;
}
__device__ double block_sum_d(double v, double* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    double r = 0.0;
    for (int i = 0; i < nw; ++i) r += red[i];
    return r;
}
__device__ uint64_t block_max_u64(uint64_t v, uint64_t* red) {
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t t = __shfl_xor_sync(0xffffffffu, v, o);
        v = t > v ? t : v;
    }
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    uint64_t r = red[0];
    for (int i = 1; i < nw; ++i) r = red[i] > r ? red[i] : r;
    return r;
}

// One slice [b0, b0 + chunk) of the logits per CTA; p2 = keys sorted (power of two >= kList).
__global__ void __launch_bounds__(kScanThreads) smp_scan(const float* __restrict__ logits, uint32_t vocab,
                                                         uint32_t chunk, int p2, int need_sum,
                                                         uint64_t* __restrict__ keys, float* __restrict__ mxs,
                                                         double* __restrict__ sums) {
    __shared__ uint64_t sk[kSliceMax];
    __shared__ float redf[32];
    __shared__ double redd[32];
    const uint32_t b0 = blockIdx.x * chunk;
    const uint32_t b1 = min(vocab, b0 + chunk);
    const int n = b1 > b0 ? static_cast<int>(b1 - b0) : 0;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < p2; i += blockDim.x) {
        uint64_t k = 0;   // below every real key: the smallest real key is -inf's, 0x007FFFFF << 32
        if (i < n) {
            const float v = logits[b0 + i];
            k = cand_key(v, b0 + i);
            m = fmaxf(m, v);
        }
        sk[i] = k;
    }
    const float mx = block_max_f(m, redf);
    double s = 0.0;
    if (need_sum) {
        double part = 0.0;
        if (isfinite(mx))
            for (int i = threadIdx.x; i < n; i += blockDim.x)
                part += exp(__dsub_rn(static_cast<double>(logits[b0 + i]), static_cast<double>(mx)));
        s = block_sum_d(part, redd);
    }
    bitonic_desc(sk, p2);
    for (int i = threadIdx.x; i < kList; i += blockDim.x) keys[static_cast<size_t>(blockIdx.x) * kList + i] = sk[i];
    if (threadIdx.x == 0) {
        mxs[blockIdx.x] = mx;
        sums[blockIdx.x] = s;
    }
}

struct FinishArgs {
    const float* logits;
    uint32_t vocab;
    int slices;
    int want;   // shortlist length: min(top_k or 256, vocab)
    float temperature, top_p;
    int top_k;
    uint64_t seed;
    const uint64_t* keys;
    const float* mxs;
    const double* sums;
    uint32_t* token;
    uint32_t* status;
};

__global__ void __launch_bounds__(kFinishThreads) smp_finish(FinishArgs a) {
    __shared__ float redf[32];
    __shared__ uint64_t redk[32];
    __shared__ unsigned hist[256];
    __shared__ uint64_t s_prefix;
    __shared__ int s_k, s_cnt;
    __shared__ double s_total;
    __shared__ uint64_t sl[kList];
    __shared__ double ev[kList], qv[kList];
    const int tid = threadIdx.x;

    float m = -INFINITY;
    for (int c = tid; c < a.slices; c += blockDim.x) m = fmaxf(m, a.mxs[c]);
    const float mx = block_max_f(m, redf);

    if (!(a.temperature > 0.0f)) {   // greedy, sampling.cpp:96-104: the best key overall
        uint64_t best = 0;
        for (int c = tid; c < a.slices; c += blockDim.x) {
            const uint64_t k = a.keys[static_cast<size_t>(c) * kList];
            best = k > best ? k : best;
        }
        best = block_max_u64(best, redk);
        if (tid == 0) {
            *a.token = key_id(best);
            *a.status = 0;
        }
        return;
    }
    if (!isfinite(mx)) {   // exp(inf - inf) is NaN in the reference: its "degenerate" error
        if (tid == 0) {
            *a.token = 0xFFFFFFFFu;
            *a.status = GTM_SAMPLE_DEGENERATE;
        }
        return;
    }
    const double dmx = static_cast<double>(mx);
    if (tid == 0) {   // full-vocabulary denominator from the slice sums, in slice order
        double t = 0.0;
        for (int c = 0; c < a.slices; ++c) {
            const float mc = a.mxs[c];
            if (mc != -INFINITY) t += a.sums[c] * exp(__dsub_rn(static_cast<double>(mc), dmx));
        }
        s_total = t;
        s_prefix = 0;
        s_k = a.want;
        s_cnt = 0;
    }

    // radix select (8 bits per pass, high to low) of the want-th best key among the first
    // `want` keys of every slice's sorted list; keys are unique, so it is exact
    const int per = a.want;
    const int total_keys = a.slices * per;
    for (int pass = 0; pass < 8; ++pass) {
        const int shift = 56 - 8 * pass;
        for (int b = tid; b < 256; b += blockDim.x) hist[b] = 0;
        __syncthreads();
        const uint64_t prefix = s_prefix;
        const uint64_t hmask = pass == 0 ? 0ull : (~0ull << (shift + 8));
        for (int j = tid; j < total_keys; j += blockDim.x) {
            const uint64_t k = a.keys[static_cast<size_t>(j / per) * kList + (j % per)];
            if ((k & hmask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            const unsigned need = static_cast<unsigned>(s_k);
            unsigned above = 0;
            for (int b = 255; b >= 0; --b) {
                if (above + hist[b] >= need) {
                    s_prefix = prefix | (static_cast<uint64_t>(b) << shift);
                    s_k = static_cast<int>(need - above);
                    break;
                }
                above += hist[b];
            }
        }
        __syncthreads();
    }
    const uint64_t thr = s_prefix;
    for (int i = tid; i < kList; i += blockDim.x) sl[i] = 0;
    __syncthreads();
    for (int j = tid; j < total_keys; j += blockDim.x) {
        const uint64_t k = a.keys[static_cast<size_t>(j / per) * kList + (j % per)];
        if (k >= thr) {
            const int slot = atomicAdd(&s_cnt, 1);
            if (slot < kList) sl[slot] = k;
        }
    }
    bitonic_desc(sl, kList);

    // per-candidate exps in parallel; the sums below run in the reference's order on one thread
    const double temp = static_cast<double>(a.temperature);
    for (int i = tid; i < per; i += blockDim.x) {
        const uint32_t id = key_id(sl[i]);   // a real id: `per` keys >= thr exist (a pad would decode to ~0)
        const float l = id < a.vocab ? a.logits[id] : -INFINITY;
        const double d = __dsub_rn(static_cast<double>(l), dmx);
        ev[i] = exp(d);
        qv[i] = exp(__ddiv_rn(d, temp));
    }
    __syncthreads();
    if (tid != 0) return;

    uint32_t st = 0;
    int cut = per;
    if (a.top_p < 1.0f) {   // sampling.cpp:141-148, against the full denominator
        const double tp = static_cast<double>(a.top_p);
        const double tol = static_cast<double>(a.vocab + 4u * static_cast<uint32_t>(per)) * 0x1p-52 * tp;
        const double total = s_total;
        double run = 0.0;
        for (int i = 0; i < per; ++i) {
            run = __dadd_rn(run, __ddiv_rn(ev[i], total));
            if (fabs(run - tp) <= tol) st |= GTM_SAMPLE_NEAR_CUT;
            if (run >= tp) {
                cut = i + 1;
                break;
            }
        }
    }
    if (a.top_k > 0 && cut > a.top_k) cut = a.top_k;   // sampling.cpp:150-151
    if (cut < 1) cut = 1;
    double denom = 0.0;   // sampling.cpp:154-159
    for (int i = 0; i < cut; ++i) denom = __dadd_rn(denom, qv[i]);
    uint64_t s = a.seed;   // xorshift64*, sampling.cpp:17-28
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    const uint64_t r64 = s * 0x2545F4914F6CDD1DULL;
    const float u = __fmul_rn(static_cast<float>((r64 >> 40) & 0xFFFFFFu), 0x1p-24f);   // exact: / 2^24
    const double r = __dmul_rn(static_cast<double>(u), denom);
    const double tol2 = 4.0 * static_cast<double>(cut + 2) * 0x1p-52 * denom;
    uint32_t tok = key_id(sl[cut - 1]);   // reachable only through rounding, as in the reference
    double acc = 0.0;
    for (int i = 0; i < cut; ++i) {   // sampling.cpp:161-167
        acc = __dadd_rn(acc, qv[i]);
        if (fabs(acc - r) <= tol2) st |= GTM_SAMPLE_NEAR_DRAW;
        if (acc >= r) {
            tok = key_id(sl[i]);
            break;
        }
    }
    *a.token = tok;
    *a.status = st;
}

__global__ void smp_penalty_count(const uint32_t* __restrict__ hist, uint32_t n, uint32_t vocab,
                                  uint32_t* __restrict__ cnt) {
    const uint32_t h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h < n) {
        const uint32_t id = hist[h];
        if (id < vocab) atomicAdd(cnt + id, 1u);
    }
}

// The first thread to reach an id takes its count (and leaves 0) and applies the step that many
// times: every application is the same function, so this equals the reference's in-order loop.
__global__ void smp_penalty_apply(float* __restrict__ logits, const uint32_t* __restrict__ hist, uint32_t n,
                                  uint32_t vocab, uint32_t* __restrict__ cnt, float penalty, float limit) {
    const uint32_t h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h >= n) return;
    const uint32_t id = hist[h];
    if (id >= vocab) return;
    const uint32_t c = atomicExch(cnt + id, 0u);
    if (c == 0) return;
    float v = logits[id];
    if (v != v) {
        // NaN: the reference's `v * penalty` on the host returns the NaN operand quieted (x86 SSE
        // propagates its payload) and its clamp keeps it; the device multiply would return the
        // canonical NaN instead
        logits[id] = __uint_as_float(__float_as_uint(v) | 0x00400000u);
        return;
    }
    for (uint32_t j = 0; j < c; ++j) {
        v = v > 0.0f ? __fdiv_rn(v, penalty) : __fmul_rn(v, penalty);
        if (limit > 0.0f) v = v < -limit ? -limit : (limit < v ? limit : v);
    }
    logits[id] = v;
}

// in and out may alias: each element is read once, then written by the same thread
__global__ void smp_softcap(const float* in, uint32_t n, float cap, float* out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __fmul_rn(cap, tanhf(__fdiv_rn(in[i], cap)));
}

size_t up256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

int grid_slices(uint32_t vocab) {
    return static_cast<int>(std::max<uint64_t>((vocab + kSliceMax - 1) / kSliceMax,
                                               std::min<uint64_t>(kMaxGrid, (vocab + kList - 1) / kList)));
}

struct WsLayout {
    size_t cnt, keys, mxs, sums, total;
};
WsLayout ws_layout(uint32_t vocab) {
    const size_t g = static_cast<size_t>(grid_slices(vocab));
    WsLayout w;
    w.cnt = 0;
    w.keys = up256(static_cast<size_t>(vocab) * 4);
    w.mxs = w.keys + up256(g * kList * 8);
    w.sums = w.mxs + up256(g * 4);
    w.total = w.sums + up256(g * 8);
    return w;
}

// The reference's messages (sampling.cpp:32-54).
int validate(const GtmSampling* p, const char* fn) {
    if (!std::isfinite(p->temperature) || p->temperature < 0.0f)
        return set_error(GTM_ERR_INVALID, "%s: temperature must be finite and >= 0 (0 = greedy)", fn);
    if (!std::isfinite(p->top_p) || p->top_p <= 0.0f || p->top_p > 1.0f)
        return set_error(GTM_ERR_INVALID, "%s: top_p must be in (0, 1]", fn);
    if (p->top_k < 0 || p->top_k > GTM_SAMPLE_MAX_TOP_K)
        return set_error(GTM_ERR_INVALID, "%s: top_k must be in 0..%d (0 disables it)", fn, GTM_SAMPLE_MAX_TOP_K);
    if (!std::isfinite(p->repetition_penalty) || p->repetition_penalty <= 0.0f)
        return set_error(GTM_ERR_INVALID, "%s: repetition_penalty must be finite and > 0 (1 = disabled)", fn);
    if (p->temperature > 0.0f && p->top_p < 1.0f && p->top_k == 0)
        return set_error(GTM_ERR_INVALID,
                         "%s: top_p < 1 with temperature > 0 requires top_k in 1..%d; full-vocabulary nucleus "
                         "sampling is not implemented", fn, GTM_SAMPLE_MAX_TOP_K);
    return GTM_OK;
}

uint64_t splitmix(uint64_t x) {
    uint64_t z = x + kGolden;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

int device_sms(const char* fn, int* sms) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return set_cuda_error(fn, e);
    return GTM_OK;
}

bool aligned_to(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace
}  // namespace gtm

using namespace gtm;

extern "C" {

GTM_API int gtm_sampling_validate(const GtmSampling* p) {
    if (!p) return set_error(GTM_ERR_INVALID, "gtm_sampling_validate: null parameters");
    const int rc = validate(p, "gtm_sampling_validate");
    if (rc == GTM_OK) clear_error();
    return rc;
}

GTM_API uint64_t gtm_sampling_splitmix64(uint64_t x) { return splitmix(x); }

GTM_API uint64_t gtm_sampling_seed_for(const GtmSampling* p, int position) {
    const uint64_t pos = static_cast<uint64_t>(static_cast<int64_t>(position));
    const uint64_t base = (p && p->has_seed) ? p->seed + pos : (kGolden ^ (pos * 0xD1B54A32D192ED03ULL));
    const uint64_t s = splitmix(base);
    return s != 0 ? s : kGolden;
}

GTM_API int gtm_softcap(uint32_t n, const float* in, float cap, float* out, void* stream) {
    const char* fn = "gtm_softcap";
    if (n == 0) {
        clear_error();
        return GTM_OK;
    }
    if (!in || !out) return set_error(GTM_ERR_INVALID, "%s: null pointer", fn);
    if (!(cap > 0.0f) || !std::isfinite(cap)) return set_error(GTM_ERR_INVALID, "%s: cap must be finite and > 0", fn);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    smp_softcap<<<(n + 255) / 256, 256, 0, st>>>(in, n, cap, out);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(fn, e);
    clear_error();
    return GTM_OK;
}

GTM_API size_t gtm_sample_workspace_bytes(uint32_t vocab) {
    if (vocab == 0 || vocab > GTM_SAMPLE_MAX_VOCAB) return 0;
    return ws_layout(vocab).total;
}

GTM_API int gtm_repetition_penalty(float* logits, uint32_t vocab, const uint32_t* history, uint32_t n_history,
                                   float penalty, float softcap, void* ws, size_t ws_bytes, void* stream) {
    const char* fn = "gtm_repetition_penalty";
    if (!logits || (n_history > 0 && !history)) return set_error(GTM_ERR_INVALID, "%s: null pointer", fn);
    if (vocab == 0 || vocab > GTM_SAMPLE_MAX_VOCAB)
        return set_error(GTM_ERR_INVALID, "%s: vocab=%u (1..%u)", fn, vocab, GTM_SAMPLE_MAX_VOCAB);
    if (!std::isfinite(penalty) || penalty <= 0.0f)
        return set_error(GTM_ERR_INVALID, "%s: repetition_penalty must be finite and > 0 (1 = disabled)", fn);
    if (!aligned_to(logits, 4) || !aligned_to(history, 4)) return set_error(GTM_ERR_MISALIGNED, "%s: 4-byte alignment", fn);
    if (penalty == 1.0f || n_history == 0) {   // sampling.cpp:77
        clear_error();
        return GTM_OK;
    }
    const WsLayout L = ws_layout(vocab);
    if (!ws || ws_bytes < L.total || !aligned_to(ws, 256))
        return set_error(GTM_ERR_WORKSPACE, "%s: workspace needs %zu bytes, 256-byte aligned", fn, L.total);
    const float limit = softcap > 0.0f ? softcap * 0.9999f : 0.0f;   // sampling.cpp:79
    uint32_t* cnt = reinterpret_cast<uint32_t*>(static_cast<char*>(ws) + L.cnt);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(cnt, 0, static_cast<size_t>(vocab) * 4, st);
    if (e != cudaSuccess) return set_cuda_error(fn, e);
    const uint32_t blocks = (n_history + 255) / 256;
    smp_penalty_count<<<blocks, 256, 0, st>>>(history, n_history, vocab, cnt);
    smp_penalty_apply<<<blocks, 256, 0, st>>>(logits, history, n_history, vocab, cnt, penalty, limit);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(fn, e);
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_sample_token(const float* logits, uint32_t vocab, const GtmSampling* p, uint64_t seed,
                             uint32_t* token, uint32_t* status, void* ws, size_t ws_bytes, void* stream) {
    const char* fn = "gtm_sample_token";
    if (!logits || !p || !token || !status) return set_error(GTM_ERR_INVALID, "%s: null pointer", fn);
    if (vocab == 0) return set_error(GTM_ERR_INVALID, "%s: empty vocabulary", fn);   // sampling.cpp:94
    if (vocab > GTM_SAMPLE_MAX_VOCAB) return set_error(GTM_ERR_UNSUPPORTED, "%s: vocab %u > %u", fn, vocab, GTM_SAMPLE_MAX_VOCAB);
    int rc = validate(p, fn);
    if (rc) return rc;
    if (!aligned_to(logits, 4) || !aligned_to(token, 4) || !aligned_to(status, 4))
        return set_error(GTM_ERR_MISALIGNED, "%s: 4-byte alignment", fn);
    const WsLayout L = ws_layout(vocab);
    if (!ws || ws_bytes < L.total || !aligned_to(ws, 256))
        return set_error(GTM_ERR_WORKSPACE, "%s: workspace needs %zu bytes, 256-byte aligned", fn, L.total);
    int sms = 0;
    rc = device_sms(fn, &sms);
    if (rc) return rc;
    // about one slice per SM, at most kSliceMax ids each
    const uint64_t g0 = std::max<uint64_t>(1, std::min<uint64_t>(sms, (vocab + kList - 1) / kList));
    uint32_t chunk = static_cast<uint32_t>((vocab + g0 - 1) / g0);
    if (chunk > static_cast<uint32_t>(kSliceMax)) chunk = kSliceMax;
    const int slices = static_cast<int>((vocab + chunk - 1) / chunk);
    if (slices > grid_slices(vocab)) return set_error(GTM_ERR_UNSUPPORTED, "%s: %d SMs exceed the workspace plan", fn, sms);
    int p2 = kList;
    while (p2 < static_cast<int>(chunk)) p2 <<= 1;
    char* base = static_cast<char*>(ws);
    uint64_t* keys = reinterpret_cast<uint64_t*>(base + L.keys);
    float* mxs = reinterpret_cast<float*>(base + L.mxs);
    double* sums = reinterpret_cast<double*>(base + L.sums);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool greedy = !(p->temperature > 0.0f);
    smp_scan<<<slices, kScanThreads, 0, st>>>(logits, vocab, chunk, p2, greedy ? 0 : 1, keys, mxs, sums);
    FinishArgs a;
    a.logits = logits;
    a.vocab = vocab;
    a.slices = slices;
    const uint32_t cap = p->top_k > 0 ? static_cast<uint32_t>(p->top_k) : static_cast<uint32_t>(kList);
    a.want = static_cast<int>(cap < vocab ? cap : vocab);
    a.temperature = p->temperature;
    a.top_p = p->top_p;
    a.top_k = p->top_k;
    a.seed = seed;
    a.keys = keys;
    a.mxs = mxs;
    a.sums = sums;
    a.token = token;
    a.status = status;
    smp_finish<<<1, kFinishThreads, 0, st>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(fn, e);
    clear_error();
    return GTM_OK;
}

}  // extern "C"

// C ABI of libgtmoe (include/gtmoe.h): argument validation, error reporting and launches.
// Errors never escape as exceptions; they become a gtm_status plus a thread-local message,
// as src/c_api.cpp:29-34 does for the reference's C API.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <cuda_runtime.h>

#include "gtm_internal.h"

namespace gtm {

constexpr uint32_t kGroup = 64;

static thread_local char g_err[512] = "";

int set_error(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return status;
}
int set_cuda_error(const char* what, cudaError_t e) {
    return set_error(GTM_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}
void clear_error() { g_err[0] = '\0'; }

static int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(what, e);
    clear_error();
    return GTM_OK;
}

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace gtm

using namespace gtm;

extern "C" {

GTM_API const char* gtm_last_error(void) { return g_err; }
GTM_API const char* gtm_version(void) { return "gtmoe 0.1 (sm_100a)"; }

static int gemv_common(int bits, uint32_t rows, uint32_t in_dim, const void* w, const uint16_t* s, const uint16_t* b,
                       const float* x, float* out, uint32_t row_begin, uint32_t row_end, void* stream,
                       const char* name) {
    if (!w || !s || !b || !x || !out) return set_error(GTM_ERR_INVALID, "%s: null pointer", name);
    if (rows == 0 || in_dim == 0 || in_dim % kGroup != 0)
        return set_error(GTM_ERR_INVALID, "%s: rows=%u in_dim=%u (in_dim must be a positive multiple of 64)", name,
                         rows, in_dim);
    if (in_dim / kGroup > 1024) return set_error(GTM_ERR_UNSUPPORTED, "%s: in_dim %u > 65536", name, in_dim);
    if (!aligned(w, 16) || !aligned(s, 2) || !aligned(b, 2) || !aligned(x, 4) || !aligned(out, 4))
        return set_error(GTM_ERR_MISALIGNED, "%s: weights need 16-byte alignment", name);
    if (row_begin >= row_end) { clear_error(); return GTM_OK; }
    k_gemv_exact(bits, rows, in_dim, w, s, b, x, out, row_begin, row_end, (cudaStream_t)stream);
    return check_launch(name);
}

GTM_API int gtm_gemv_q4(uint32_t rows, uint32_t in_dim, const void* w, const uint16_t* s, const uint16_t* b,
                        const float* x, float* out, void* stream) {
    return gemv_common(4, rows, in_dim, w, s, b, x, out, 0, rows, stream, "gtm_gemv_q4");
}
GTM_API int gtm_gemv_q8(uint32_t rows, uint32_t in_dim, const void* w, const uint16_t* s, const uint16_t* b,
                        const float* x, float* out, void* stream) {
    return gemv_common(8, rows, in_dim, w, s, b, x, out, 0, rows, stream, "gtm_gemv_q8");
}

GTM_API int gtm_gemv_q4_rows(uint32_t rows, uint32_t in_dim, uint32_t n, const void* w, const uint16_t* s,
                             const uint16_t* b, const float* x, float* out, void* stream) {
    if (n == 0) { clear_error(); return GTM_OK; }
    if (n > kMaxBatchRows)
        return set_error(GTM_ERR_INVALID, "gtm_gemv_q4_rows: n=%u vectors (1..%u)", n, kMaxBatchRows);
    if (!w || !s || !b || !x || !out) return set_error(GTM_ERR_INVALID, "gtm_gemv_q4_rows: null pointer");
    if (rows == 0 || in_dim == 0 || in_dim % kGroup != 0 || in_dim / kGroup > 1024)
        return set_error(GTM_ERR_INVALID, "gtm_gemv_q4_rows: rows=%u in_dim=%u (a multiple of 64, at most 65536)", rows,
                         in_dim);
    if (!aligned(w, 16) || !aligned(s, 2) || !aligned(b, 2) || !aligned(x, 4) || !aligned(out, 4))
        return set_error(GTM_ERR_MISALIGNED, "gtm_gemv_q4_rows: weights need 16-byte alignment");
    if (n == 1 || !aligned(x, 16) || !k_gemv_exact_rows4(rows, in_dim, n, w, s, b, x, out, (cudaStream_t)stream))
        k_gemv_exact(4, rows, in_dim, w, s, b, x, out, 0, rows, (cudaStream_t)stream, n);
    return check_launch("gtm_gemv_q4_rows");
}

GTM_API int gtm_router_topk(uint32_t n, uint32_t k, const float* logits, const uint16_t* pes, uint32_t* idx,
                            float* w, void* stream) {
    if (!logits || !pes || !idx || !w) return set_error(GTM_ERR_INVALID, "gtm_router_topk: null pointer");
    if (n == 0 || n > 1024 || k == 0 || k > 32 || k > n)
        return set_error(GTM_ERR_INVALID, "gtm_router_topk: num_experts=%u k=%u (need 1 <= k <= min(32, n), n <= 1024)",
                         n, k);
    k_router_topk(n, k, logits, pes, idx, w, (cudaStream_t)stream);
    return check_launch("gtm_router_topk");
}

GTM_API int gtm_geglu(uint32_t n, const float* g, const float* u, float* out, void* stream) {
    if (!g || !u || !out) return set_error(GTM_ERR_INVALID, "gtm_geglu: null pointer");
    if (n == 0) { clear_error(); return GTM_OK; }
    k_geglu(n, g, u, out, (cudaStream_t)stream);
    return check_launch("gtm_geglu");
}

GTM_API int gtm_scale_accum(uint32_t n, const float* in, const float* w, uint32_t wi, int acc, float* out,
                            void* stream) {
    if (!in || !w || !out) return set_error(GTM_ERR_INVALID, "gtm_scale_accum: null pointer");
    if (n == 0) { clear_error(); return GTM_OK; }
    k_scale_accum(n, in, w, wi, acc, out, (cudaStream_t)stream);
    return check_launch("gtm_scale_accum");
}

GTM_API int gtm_mul_bf16(uint32_t n, const float* in, const uint16_t* w, float scale, float* out, void* stream) {
    if (!in || !w || !out) return set_error(GTM_ERR_INVALID, "gtm_mul_bf16: null pointer");
    if (n == 0) { clear_error(); return GTM_OK; }
    k_mul_bf16(n, in, w, scale, out, (cudaStream_t)stream);
    return check_launch("gtm_mul_bf16");
}

GTM_API int gtm_rmsnorm(uint32_t n, const float* x, const uint16_t* w, float eps, float* out, void* stream) {
    if (!x || !out) return set_error(GTM_ERR_INVALID, "gtm_rmsnorm: null pointer");
    if (n == 0 || n > kMaxNormDim) return set_error(GTM_ERR_INVALID, "gtm_rmsnorm: n=%u (1..%u)", n, kMaxNormDim);
    k_rmsnorm(n, x, w, eps, out, (cudaStream_t)stream);
    return check_launch("gtm_rmsnorm");
}

GTM_API int gtm_rmsnorm_rows(uint32_t rows, uint32_t n, const float* x, const uint16_t* w, float eps, float* out,
                             void* stream) {
    if (rows == 0) { clear_error(); return GTM_OK; }
    if (!x || !out) return set_error(GTM_ERR_INVALID, "gtm_rmsnorm_rows: null pointer");
    if (n == 0 || n > kMaxNormDim || rows > kMaxBatchRows)
        return set_error(GTM_ERR_INVALID, "gtm_rmsnorm_rows: n=%u (1..%u), rows=%u (at most %u)", n, kMaxNormDim, rows,
                         kMaxBatchRows);
    k_rmsnorm(n, x, w, eps, out, (cudaStream_t)stream, rows);
    return check_launch("gtm_rmsnorm_rows");
}

GTM_API int gtm_post_attn_rows(uint32_t rows, uint32_t d, const float* attn, const float* hidden,
                               const uint16_t* wpost, const uint16_t* wpre, const uint16_t* wpre2, float eps,
                               float* hout, float* dense, float* routed, float* router, void* stream) {
    if (rows == 0) { clear_error(); return GTM_OK; }
    if (!attn || !hidden || !wpost || !hout || (dense && !wpre) || (routed && !wpre2))
        return set_error(GTM_ERR_INVALID, "gtm_post_attn_rows: null pointer");
    if (d == 0 || d > kMaxNormDim / 2 || rows > kMaxBatchRows)
        return set_error(GTM_ERR_INVALID, "gtm_post_attn_rows: d=%u (1..%u), rows=%u (at most %u)", d, kMaxNormDim / 2,
                         rows, kMaxBatchRows);
    k_post_attn(d, attn, hidden, wpost, wpre, wpre2, eps, hout, dense, routed, router, (cudaStream_t)stream, rows);
    return check_launch("gtm_post_attn_rows");
}

GTM_API int gtm_post_attn(uint32_t d, const float* attn, const float* hidden, const uint16_t* wpost,
                          const uint16_t* wpre, const uint16_t* wpre2, float eps, float* hout, float* dense,
                          float* routed, float* router, void* stream) {
    if (!attn || !hidden || !wpost || !wpre || !wpre2 || !hout || !dense || !routed || !router)
        return set_error(GTM_ERR_INVALID, "gtm_post_attn: null pointer");
    if (d == 0 || d > kMaxNormDim / 2) return set_error(GTM_ERR_INVALID, "gtm_post_attn: d=%u (1..%u)", d, kMaxNormDim / 2);
    k_post_attn(d, attn, hidden, wpost, wpre, wpre2, eps, hout, dense, routed, router, (cudaStream_t)stream);
    return check_launch("gtm_post_attn");
}

GTM_API int gtm_layer_tail(uint32_t d, const float* h2, const float* h1, const float* hidden, const uint16_t* wpf2,
                           const uint16_t* wpf, float eps, float ls, float* hout, void* stream) {
    if (!h2 || !h1 || !hidden || !wpf2 || !wpf || !hout) return set_error(GTM_ERR_INVALID, "gtm_layer_tail: null pointer");
    if (d == 0 || d > kMaxNormDim / 2) return set_error(GTM_ERR_INVALID, "gtm_layer_tail: d=%u (1..%u)", d, kMaxNormDim / 2);
    k_layer_tail(d, h2, h1, hidden, wpf2, wpf, eps, ls, hout, (cudaStream_t)stream);
    return check_launch("gtm_layer_tail");
}

// ---- gtm_dispatch: the reference's root-constant convention ------------------------------------
static float f_of(uint32_t bits) { float f; memcpy(&f, &bits, 4); return f; }

GTM_API int gtm_dispatch(int kernel, const void* const* srv, int n_srv, void* const* uav, int n_uav,
                         const uint32_t c[16], uint32_t grid_x, void* stream) {
    if (!c) return set_error(GTM_ERR_INVALID, "gtm_dispatch: constants are NULL");
    auto in = [&](int i, uint32_t off) -> const unsigned char* {
        return (i < n_srv && srv && srv[i]) ? static_cast<const unsigned char*>(srv[i]) + off : nullptr;
    };
    auto outp = [&](int i, uint32_t off) -> unsigned char* {
        return (i < n_uav && uav && uav[i]) ? static_cast<unsigned char*>(uav[i]) + off : nullptr;
    };
    switch (kernel) {
        case GTM_KERNEL_GEMV_INT4:
        case GTM_KERNEL_GEMV_INT8: {
            // gp0 = (rows, in_dim, w_off, s_off)  gp1 = (b_off, x_off, out_off, row_base)  (GemvInt4.hlsl:9-10)
            const uint32_t rows = c[0], in_dim = c[1], row_base = c[7];
            const uint32_t end = rows < row_base + grid_x ? rows : row_base + grid_x;
            const unsigned char* o = outp(0, c[6]);
            return gemv_common(kernel == GTM_KERNEL_GEMV_INT4 ? 4 : 8, rows, in_dim, in(0, c[2]),
                               reinterpret_cast<const uint16_t*>(in(1, c[3])), reinterpret_cast<const uint16_t*>(in(2, c[4])),
                               reinterpret_cast<const float*>(in(3, c[5])), (float*)o, row_base, end, stream,
                               "gtm_dispatch(GemvInt)");
        }
        case GTM_KERNEL_RMSNORMK:   // gp0 = (n, x_off, w_off, out_off)  gp1 = (has_weight, eps_bits)
            return gtm_rmsnorm(c[0], reinterpret_cast<const float*>(in(0, c[1])),
                               c[4] ? reinterpret_cast<const uint16_t*>(in(1, c[2])) : nullptr, f_of(c[5]),
                               reinterpret_cast<float*>(outp(0, c[3])), stream);
        case GTM_KERNEL_ROUTER_TOPK: {  // gp0 = (num_experts, K, logits_off, scale_off)  gp1 = (idx_off, wgt_off)
            const uint32_t k = c[1] < 8 ? c[1] : 8;   // the shader's MAX_TOPK
            return gtm_router_topk(c[0], k, reinterpret_cast<const float*>(in(0, c[2])),
                                   reinterpret_cast<const uint16_t*>(in(1, c[3])), reinterpret_cast<uint32_t*>(outp(0, c[4])),
                                   reinterpret_cast<float*>(outp(1, c[5])), stream);
        }
        case GTM_KERNEL_GEGLU:      // gp0 = (n, gate_off, up_off, out_off)
            return gtm_geglu(c[0], reinterpret_cast<const float*>(in(0, c[1])), reinterpret_cast<const float*>(in(1, c[2])),
                             reinterpret_cast<float*>(outp(0, c[3])), stream);
        case GTM_KERNEL_SCALE_ACCUM:  // gp0 = (n, in_off, out_off, w_off)  gp1 = (accumulate, weight_index)
            return gtm_scale_accum(c[0], reinterpret_cast<const float*>(in(0, c[1])),
                                   reinterpret_cast<const float*>(in(1, c[3])), c[5], c[4] != 0,
                                   reinterpret_cast<float*>(outp(0, c[2])), stream);
        case GTM_KERNEL_MUL_BF16:   // gp0 = (n, in_off, w_off, out_off)  gp1 = (scale_bits)
            return gtm_mul_bf16(c[0], reinterpret_cast<const float*>(in(0, c[1])),
                                reinterpret_cast<const uint16_t*>(in(1, c[2])), f_of(c[4]),
                                reinterpret_cast<float*>(outp(0, c[3])), stream);
        case GTM_KERNEL_POST_ATTN:  // gp0 = (D, attn, hidden, out_hidden) gp1 = (eps, w_post, w_pre, w_pre2) gp2 = (dense, routed, router)
            return gtm_post_attn(c[0], reinterpret_cast<const float*>(in(0, c[1])), reinterpret_cast<const float*>(in(1, c[2])),
                                 reinterpret_cast<const uint16_t*>(in(2, c[5])), reinterpret_cast<const uint16_t*>(in(3, c[6])),
                                 reinterpret_cast<const uint16_t*>(in(4, c[7])), f_of(c[4]),
                                 reinterpret_cast<float*>(outp(0, c[3])), reinterpret_cast<float*>(outp(1, c[8])),
                                 reinterpret_cast<float*>(outp(2, c[9])), reinterpret_cast<float*>(outp(3, c[10])), stream);
        case GTM_KERNEL_LAYER_TAIL:  // gp0 = (D, h2, h1, hidden) gp1 = (eps, w_pf2, w_pf, out) gp2 = (layer_scalar_bits, scratch)
            return gtm_layer_tail(c[0], reinterpret_cast<const float*>(in(0, c[1])), reinterpret_cast<const float*>(in(1, c[2])),
                                  reinterpret_cast<const float*>(in(2, c[3])), reinterpret_cast<const uint16_t*>(in(3, c[5])),
                                  reinterpret_cast<const uint16_t*>(in(4, c[6])), f_of(c[4]), f_of(c[8]),
                                  reinterpret_cast<float*>(outp(0, c[7])), stream);
        default:
            return set_error(GTM_ERR_UNSUPPORTED, "gtm_dispatch: kernel %d is not on the MoE path", kernel);
    }
}

// ---- fused decode ---------------------------------------------------------------------------------
static bool dims_supported(const GtmDims* d) {
    return d->hidden == 2816 && d->moe_inter == 704 && d->ffn_inter == 2112 && d->num_experts == 128 && d->top_k == 8;
}

GTM_API size_t gtm_moe_decode_workspace_bytes(const GtmDims* dims) {
    if (!dims || !dims_supported(dims)) return 0;
    return decode_workspace_bytes();
}

GTM_API int gtm_moe_decode(const GtmDims* dims, const GtmLayer* layers, int num_layers, const GtmDecodeIO* io,
                           void* ws, size_t ws_bytes, void* stream) {
    if (!dims || !layers || !io) return set_error(GTM_ERR_INVALID, "gtm_moe_decode: null argument");
    if (!dims_supported(dims))
        return set_error(GTM_ERR_UNSUPPORTED,
                         "gtm_moe_decode: built for hidden 2816, moe 704, ffn 2112, 128 experts, top-8 (got %u/%u/%u/%u/%u)",
                         dims->hidden, dims->moe_inter, dims->ffn_inter, dims->num_experts, dims->top_k);
    if (num_layers < 1 || num_layers > GTM_MAX_LAYERS)
        return set_error(GTM_ERR_INVALID, "gtm_moe_decode: num_layers=%d (1..%d)", num_layers, GTM_MAX_LAYERS);
    if (!io->hidden_in_dev || !io->hidden_out_dev) return set_error(GTM_ERR_INVALID, "gtm_moe_decode: hidden in/out NULL");
    if (!ws || ws_bytes < decode_workspace_bytes() || !aligned(ws, 256))
        return set_error(GTM_ERR_WORKSPACE, "gtm_moe_decode: workspace needs %zu bytes, 256-byte aligned",
                         decode_workspace_bytes());
    for (int l = 0; l < num_layers; ++l) {
        const GtmLayer& L = layers[l];
        if (!L.resident_dev || !L.experts_dev || L.expert_stride == 0)
            return set_error(GTM_ERR_INVALID, "gtm_moe_decode: layer %d has a null base or zero stride", l);
        // weight rows, scales and biases move by 16-byte bulk copies; norm vectors by 16-byte cp.async
        const uint64_t offs16[] = {L.router.weight, L.expert_stride, L.expert_gate.weight, L.expert_up.weight,
                                   L.expert_down.weight, L.shared_gate.weight, L.shared_up.weight, L.shared_down.weight,
                                   L.expert_gate.scales, L.expert_gate.biases, L.expert_up.scales, L.expert_up.biases,
                                   L.expert_down.scales, L.expert_down.biases, L.shared_gate.scales,
                                   L.shared_gate.biases, L.shared_up.scales, L.shared_up.biases, L.shared_down.scales,
                                   L.shared_down.biases, L.per_expert_scale, L.pre_ffn_norm, L.pre_ffn_norm_2,
                                   L.router_scale, L.post_ffn_norm_1, L.post_ffn_norm_2, L.post_ffn_norm};
        if (!aligned(L.resident_dev, 16) || !aligned(L.experts_dev, 16))
            return set_error(GTM_ERR_MISALIGNED, "gtm_moe_decode: layer %d base pointers must be 16-byte aligned", l);
        for (uint64_t o : offs16)
            if (o % 16) return set_error(GTM_ERR_MISALIGNED, "gtm_moe_decode: layer %d weight offset %llu not 16-byte aligned",
                                         l, (unsigned long long)o);
    }
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return set_cuda_error("gtm_moe_decode: device query", e);
    // at most 176 CTAs: the per-CTA down chunks are sized for 120..176 CTAs
    const int ctas = sms < 176 ? sms : 176;
    if (ctas < kDecodeMinCtas)
        return set_error(GTM_ERR_UNSUPPORTED, "gtm_moe_decode: needs >= %d SMs (device has %d)", kDecodeMinCtas, sms);
    int rc = launch_decode(*dims, layers, num_layers, *io, ws, ws_bytes, (cudaStream_t)stream, ctas);
    if (rc == GTM_OK) clear_error();
    return rc;
}

GTM_API int gtm_moe_decode_check(void* ws, void* stream) {
    if (!ws) return set_error(GTM_ERR_INVALID, "gtm_moe_decode_check: null workspace");
    int flag = 0;
    char* sticky = static_cast<char*>(ws) + decode_sticky_offset();
    cudaError_t e = cudaMemcpyAsync(&flag, sticky, sizeof(int), cudaMemcpyDeviceToHost,
                                    (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) return set_cuda_error("gtm_moe_decode_check", e);
    if (flag != 0) {
        int zero = 0;
        cudaMemcpy(sticky, &zero, sizeof(int), cudaMemcpyHostToDevice);
        return set_error(GTM_ERR_TIMEOUT, "gtm_moe_decode: a grid barrier wait timed out (device flag %d)", flag);
    }
    clear_error();
    return GTM_OK;
}

// ---- T > 1 tokens -------------------------------------------------------------------------------
static constexpr uint32_t kMaxTokens = 65536;

static int check_layer(const char* fn, const GtmLayer& L) {
    if (!L.resident_dev || !L.experts_dev || L.expert_stride == 0)
        return set_error(GTM_ERR_INVALID, "%s: null base or zero expert stride", fn);
    if (!aligned(L.resident_dev, 16) || !aligned(L.experts_dev, 16))
        return set_error(GTM_ERR_MISALIGNED, "%s: base pointers must be 16-byte aligned", fn);
    // packed weights load by TMA and the expert/shared scale and bias rows by bulk copy: both want
    // 16-byte aligned sources
    const uint64_t offs16[] = {L.router.weight, L.expert_stride, L.expert_gate.weight, L.expert_up.weight,
                               L.expert_down.weight, L.shared_gate.weight, L.shared_up.weight, L.shared_down.weight,
                               L.shared_gate.scales, L.shared_gate.biases, L.shared_up.scales, L.shared_up.biases,
                               L.shared_down.scales, L.shared_down.biases, L.expert_gate.scales, L.expert_gate.biases,
                               L.expert_up.scales, L.expert_up.biases, L.expert_down.scales, L.expert_down.biases};
    for (uint64_t o : offs16)
        if (o % 16) return set_error(GTM_ERR_MISALIGNED, "%s: weight/scale/bias offset %llu not 16-byte aligned", fn,
                                     (unsigned long long)o);
    const uint64_t offs2[] = {L.router.scales, L.router.biases, L.router_scale, L.per_expert_scale,
                              L.pre_ffn_norm, L.pre_ffn_norm_2, L.post_ffn_norm_1, L.post_ffn_norm_2,
                              L.post_ffn_norm, L.layer_scalar};
    for (uint64_t o : offs2)
        if (o % 2) return set_error(GTM_ERR_MISALIGNED, "%s: bf16 offset %llu is odd", fn, (unsigned long long)o);
    return GTM_OK;
}

GTM_API size_t gtm_moe_tokens_workspace_bytes(const GtmDims* dims, uint32_t max_tokens) {
    if (!dims || !dims_supported(dims) || max_tokens == 0 || max_tokens > kMaxTokens) return 0;
    return tokens_workspace_bytes(max_tokens);
}

GTM_API int gtm_moe_tokens(const GtmDims* dims, const GtmLayer* layer, const GtmTokensIO* io, void* ws,
                           size_t ws_bytes, void* stream) {
    if (!dims || !layer || !io) return set_error(GTM_ERR_INVALID, "gtm_moe_tokens: null argument");
    if (!dims_supported(dims))
        return set_error(GTM_ERR_UNSUPPORTED,
                         "gtm_moe_tokens: built for hidden 2816, moe 704, ffn 2112, 128 experts, top-8 (got %u/%u/%u/%u/%u)",
                         dims->hidden, dims->moe_inter, dims->ffn_inter, dims->num_experts, dims->top_k);
    const uint32_t T = io->num_tokens;
    if (T == 0 || T > kMaxTokens)
        return set_error(GTM_ERR_INVALID, "gtm_moe_tokens: num_tokens=%u (1..%u)", T, kMaxTokens);
    if ((io->x_dev == nullptr) == (io->x_bf16_dev == nullptr))
        return set_error(GTM_ERR_INVALID, "gtm_moe_tokens: give exactly one of x_dev and x_bf16_dev");
    if (!io->hidden_out_dev) return set_error(GTM_ERR_INVALID, "gtm_moe_tokens: hidden_out_dev is NULL");
    if (!aligned(io->x_dev, 4) || !aligned(io->x_bf16_dev, 2) || !aligned(io->hidden_out_dev, 4) ||
        !aligned(io->h1_dev, 4) || !aligned(io->h2_dev, 4) || !aligned(io->logits_dev, 4) ||
        !aligned(io->topk_idx_dev, 4) || !aligned(io->topk_w_dev, 4) || !aligned(io->logit_bias_dev, 4) ||
        !aligned(io->route_logits_dev, 4))
        return set_error(GTM_ERR_MISALIGNED, "gtm_moe_tokens: an io pointer is not aligned to its element size");
    const size_t need = tokens_workspace_bytes(T);
    if (!ws || ws_bytes < need || !aligned(ws, 256))
        return set_error(GTM_ERR_WORKSPACE, "gtm_moe_tokens: workspace needs %zu bytes, 256-byte aligned", need);
    int rc = check_layer("gtm_moe_tokens", *layer);
    if (rc) return rc;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return set_cuda_error("gtm_moe_tokens: device query", e);
    rc = launch_tokens(*dims, *layer, *io, ws, ws_bytes, (cudaStream_t)stream, sms);
    if (rc == GTM_OK) clear_error();
    return rc;
}

GTM_API int gtm_moe_tokens_check(void* ws, void* stream) {
    if (!ws) return set_error(GTM_ERR_INVALID, "gtm_moe_tokens_check: null workspace");
    const int rc = tokens_check(ws, (cudaStream_t)stream);
    if (rc == GTM_OK) clear_error();
    return rc;
}

GTM_API int gtm_set_phase_events(void* const* events, int n) {
    const int rc = set_phase_events(events, n);
    if (rc == GTM_OK) clear_error();
    return rc;
}

// ---- tied LM head, greedy --------------------------------------------------------------------------
static int sm_count(const char* fn, int* sms);

GTM_API size_t gtm_lm_head_workspace_bytes(uint32_t rows) {
    return rows == 0 ? 0 : lm_head_workspace_bytes(rows);
}

GTM_API int gtm_lm_head_greedy(uint32_t rows, uint32_t in_dim, const void* w, const uint16_t* s, const uint16_t* b,
                               const float* x, uint32_t* token, float* logit, void* ws, size_t ws_bytes, void* stream) {
    const char* fn = "gtm_lm_head_greedy";
    if (rows == 0 || !w || !s || !b || !x || !token) return set_error(GTM_ERR_INVALID, "%s: null pointer or zero rows", fn);
    if (in_dim != 2816) return set_error(GTM_ERR_UNSUPPORTED, "%s: built for in_dim 2816 (got %u)", fn, in_dim);
    if (!aligned(w, 16) || !aligned(s, 2) || !aligned(b, 2) || !aligned(x, 16) || !aligned(token, 4) || !aligned(logit, 4))
        return set_error(GTM_ERR_MISALIGNED, "%s: weights and x must be 16-byte aligned", fn);
    const size_t need = lm_head_workspace_bytes(rows);
    if (!ws || ws_bytes < need || !aligned(ws, 256))
        return set_error(GTM_ERR_WORKSPACE, "%s: workspace needs %zu bytes, 256-byte aligned", fn, need);
    int sms = 0;
    int rc = sm_count(fn, &sms);
    if (rc) return rc;
    rc = launch_lm_head(rows, w, s, b, x, token, logit, ws, (cudaStream_t)stream, sms);
    if (rc == GTM_OK) clear_error();
    return rc;
}

GTM_API int gtm_lm_head_candidates(void* ws, void* stream, int32_t* count) {
    if (!ws || !count) return set_error(GTM_ERR_INVALID, "gtm_lm_head_candidates: null argument");
    int n = 0;
    const int rc = lm_head_candidates(ws, (cudaStream_t)stream, &n);
    if (rc) return rc;
    *count = n;
    clear_error();
    return GTM_OK;
}

// ---- expert parallelism -------------------------------------------------------------------------
static bool ep_config_ok(const GtmEpConfig* ep) {
    return ep && ep->world >= 1 && ep->world <= GTM_EP_MAX_WORLD && 128 % ep->world == 0 && ep->rank < ep->world &&
           ep->max_tokens >= 1 && ep->max_tokens <= kMaxTokens && ep->max_recv_rows >= 1 &&
           ep->max_recv_rows <= kMaxTokens * 8u;
}

static int ep_common(const char* fn, const GtmDims* dims, const GtmLayer* layer, const GtmEpConfig* ep, void* ws,
                     size_t ws_bytes) {
    if (!dims || !layer || !ep) return set_error(GTM_ERR_INVALID, "%s: null argument", fn);
    if (!dims_supported(dims))
        return set_error(GTM_ERR_UNSUPPORTED, "%s: built for hidden 2816, moe 704, ffn 2112, 128 experts, top-8", fn);
    if (!ep_config_ok(ep))
        return set_error(GTM_ERR_INVALID, "%s: bad EP config (world %u must divide 128, rank %u < world, sizes %u/%u)",
                         fn, ep->world, ep->rank, ep->max_tokens, ep->max_recv_rows);
    const size_t need = ep_workspace_bytes(ep->max_tokens, ep->max_recv_rows);
    if (!ws || ws_bytes < need || !aligned(ws, 256))
        return set_error(GTM_ERR_WORKSPACE, "%s: workspace needs %zu bytes, 256-byte aligned", fn, need);
    return check_layer(fn, *layer);
}

// allow_empty: a rank with no tokens in this call still takes part (peer-memory phases)
static int ep_io(const char* fn, const GtmTokensIO* io, const GtmEpConfig* ep, bool need_out, bool allow_empty = false) {
    if (!io) return set_error(GTM_ERR_INVALID, "%s: null io", fn);
    if (allow_empty && io->num_tokens == 0) return GTM_OK;
    if (io->num_tokens == 0 || io->num_tokens > ep->max_tokens)
        return set_error(GTM_ERR_INVALID, "%s: num_tokens=%u (1..max_tokens %u)", fn, io->num_tokens, ep->max_tokens);
    if ((io->x_dev == nullptr) == (io->x_bf16_dev == nullptr))
        return set_error(GTM_ERR_INVALID, "%s: give exactly one of x_dev and x_bf16_dev", fn);
    if (need_out && !io->hidden_out_dev) return set_error(GTM_ERR_INVALID, "%s: hidden_out_dev is NULL", fn);
    return GTM_OK;
}

static int sm_count(const char* fn, int* sms) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return set_cuda_error(fn, e);
    return GTM_OK;
}

GTM_API size_t gtm_moe_ep_workspace_bytes(const GtmDims* dims, const GtmEpConfig* ep) {
    if (!dims || !dims_supported(dims) || !ep_config_ok(ep)) return 0;
    return ep_workspace_bytes(ep->max_tokens, ep->max_recv_rows);
}

GTM_API int gtm_moe_ep_dispatch(const GtmDims* dims, const GtmLayer* layer, const GtmTokensIO* io,
                                const GtmEpConfig* ep, float* send_rows, GtmEpMeta* send_meta, int32_t* send_counts,
                                void* ws, size_t ws_bytes, void* stream) {
    const char* fn = "gtm_moe_ep_dispatch";
    int rc = ep_common(fn, dims, layer, ep, ws, ws_bytes);
    if (!rc) rc = ep_io(fn, io, ep, false);
    if (rc) return rc;
    if (!send_rows || !send_meta || !send_counts) return set_error(GTM_ERR_INVALID, "%s: null send buffer", fn);
    if (!aligned(send_rows, 16) || !aligned(send_meta, 8) || !aligned(send_counts, 4))
        return set_error(GTM_ERR_MISALIGNED, "%s: send_rows must be 16-byte aligned", fn);
    rc = launch_ep_dispatch(*dims, *layer, *io, *ep, send_rows, send_meta, send_counts, ws, (cudaStream_t)stream);
    if (rc == GTM_OK) clear_error();
    return rc;
}

GTM_API int gtm_moe_ep_shared(const GtmDims* dims, const GtmLayer* layer, const GtmTokensIO* io,
                              const GtmEpConfig* ep, void* ws, size_t ws_bytes, void* stream) {
    const char* fn = "gtm_moe_ep_shared";
    int rc = ep_common(fn, dims, layer, ep, ws, ws_bytes);
    if (!rc) rc = ep_io(fn, io, ep, false);
    int sms = 0;
    if (!rc) rc = sm_count(fn, &sms);
    if (rc) return rc;
    rc = launch_ep_shared(*layer, *io, *ep, ws, (cudaStream_t)stream, sms, false);
    if (rc == GTM_OK) clear_error();
    return rc;
}

GTM_API int gtm_moe_ep_experts(const GtmDims* dims, const GtmLayer* layer, const GtmEpConfig* ep,
                               const float* recv_rows, const GtmEpMeta* recv_meta, uint32_t n_recv, float* ret_rows,
                               void* ws, size_t ws_bytes, void* stream) {
    const char* fn = "gtm_moe_ep_experts";
    int rc = ep_common(fn, dims, layer, ep, ws, ws_bytes);
    if (rc) return rc;
    if (n_recv > ep->max_recv_rows)
        return set_error(GTM_ERR_WORKSPACE, "%s: %u rows > max_recv_rows %u", fn, n_recv, ep->max_recv_rows);
    if (n_recv > 0 && (!recv_rows || !recv_meta || !ret_rows)) return set_error(GTM_ERR_INVALID, "%s: null row buffer", fn);
    if (!aligned(recv_rows, 16) || !aligned(recv_meta, 8) || !aligned(ret_rows, 16))
        return set_error(GTM_ERR_MISALIGNED, "%s: row buffers must be 16-byte aligned", fn);
    int sms = 0;
    if ((rc = sm_count(fn, &sms))) return rc;
    rc = launch_ep_experts(*layer, *ep, recv_rows, recv_meta, n_recv, ret_rows, ws, (cudaStream_t)stream, sms);
    if (rc == GTM_OK) clear_error();
    return rc;
}

GTM_API int gtm_moe_ep_combine(const GtmDims* dims, const GtmLayer* layer, const GtmTokensIO* io,
                               const GtmEpConfig* ep, const float* ret_rows, void* ws, size_t ws_bytes, void* stream) {
    const char* fn = "gtm_moe_ep_combine";
    int rc = ep_common(fn, dims, layer, ep, ws, ws_bytes);
    if (!rc) rc = ep_io(fn, io, ep, true);
    if (rc) return rc;
    if (!ret_rows) return set_error(GTM_ERR_INVALID, "%s: null ret_rows", fn);
    rc = launch_ep_combine(*dims, *layer, *io, *ep, ret_rows, ws, (cudaStream_t)stream);
    if (rc == GTM_OK) clear_error();
    return rc;
}

GTM_API int gtm_moe_ep_check(void* ws, void* stream) {
    if (!ws) return set_error(GTM_ERR_INVALID, "gtm_moe_ep_check: null workspace");
    const int rc = tokens_check(ws, (cudaStream_t)stream);
    if (rc == GTM_OK) clear_error();
    return rc;
}

// ---- expert parallelism over peer memory --------------------------------------------------------
static bool peer_config_ok(const GtmEpConfig* ep) {
    return ep && ep->world >= 1 && ep->world <= GTM_EP_PEER_MAX_WORLD && 128 % ep->world == 0 &&
           ep->rank < ep->world && ep->max_tokens >= 1 && (uint64_t)ep->world * ep->max_tokens <= kMaxTokens;
}

static int peer_common(const char* fn, const GtmDims* dims, const GtmLayer* layer, const GtmEpConfig* ep,
                       const void* ws, size_t ws_bytes) {
    if (!dims || !layer || !ep) return set_error(GTM_ERR_INVALID, "%s: null argument", fn);
    if (!dims_supported(dims))
        return set_error(GTM_ERR_UNSUPPORTED, "%s: built for hidden 2816, moe 704, ffn 2112, 128 experts, top-8", fn);
    if (!peer_config_ok(ep))
        return set_error(GTM_ERR_INVALID,
                         "%s: bad EP config (world %u divides 128 and is at most %d, rank %u < world, "
                         "world x max_tokens %u at most %u)", fn, ep->world, GTM_EP_PEER_MAX_WORLD, ep->rank,
                         ep->max_tokens, kMaxTokens);
    const size_t need = ep_peer_workspace_bytes(ep->world, ep->max_tokens);
    if (!ws || ws_bytes < need || !aligned(ws, 256))
        return set_error(GTM_ERR_WORKSPACE, "%s: workspace needs %zu bytes, 256-byte aligned", fn, need);
    return check_layer(fn, *layer);
}

GTM_API size_t gtm_moe_ep_peer_workspace_bytes(const GtmDims* dims, const GtmEpConfig* ep) {
    if (!dims || !dims_supported(dims) || !peer_config_ok(ep)) return 0;
    return ep_peer_workspace_bytes(ep->world, ep->max_tokens);
}

static int peers_ok(const char* fn, const GtmEpConfig* ep, const GtmEpPeers* peers) {
    for (uint32_t s = 0; s < ep->world; ++s)
        if (!peers->workspace_dev[s] || !aligned(peers->workspace_dev[s], 256))
            return set_error(GTM_ERR_INVALID, "%s: workspace of rank %u is null or not 256-byte aligned", fn, s);
    return GTM_OK;
}

GTM_API int gtm_moe_ep_peer_dispatch(const GtmDims* dims, const GtmLayer* layer, const GtmTokensIO* io,
                                     const GtmEpConfig* ep, const GtmEpPeers* peers, size_t ws_bytes, void* stream) {
    const char* fn = "gtm_moe_ep_peer_dispatch";
    if (!peers || !ep) return set_error(GTM_ERR_INVALID, "%s: null argument", fn);
    int rc = peer_common(fn, dims, layer, ep, ep->rank < GTM_EP_PEER_MAX_WORLD ? peers->workspace_dev[ep->rank] : nullptr,
                         ws_bytes);
    if (!rc) rc = peers_ok(fn, ep, peers);
    if (!rc) rc = ep_io(fn, io, ep, false, true);
    if (rc) return rc;
    rc = launch_ep_peer_dispatch(*dims, *layer, *io, *ep, peers->workspace_dev, (cudaStream_t)stream);
    if (rc == GTM_OK) clear_error();
    return rc;
}

GTM_API int gtm_moe_ep_peer_shared(const GtmDims* dims, const GtmLayer* layer, const GtmTokensIO* io,
                                   const GtmEpConfig* ep, void* ws, size_t ws_bytes, void* stream) {
    const char* fn = "gtm_moe_ep_peer_shared";
    int rc = peer_common(fn, dims, layer, ep, ws, ws_bytes);
    if (!rc) rc = ep_io(fn, io, ep, false, true);
    int sms = 0;
    if (!rc) rc = sm_count(fn, &sms);
    if (rc) return rc;
    if (io->num_tokens == 0) { clear_error(); return GTM_OK; }
    rc = launch_ep_shared(*layer, *io, *ep, ws, (cudaStream_t)stream, sms, true);
    if (rc == GTM_OK) clear_error();
    return rc;
}

GTM_API int gtm_moe_ep_peer_experts(const GtmDims* dims, const GtmLayer* layer, const GtmEpConfig* ep,
                                    const GtmEpPeers* peers, size_t ws_bytes, void* stream) {
    const char* fn = "gtm_moe_ep_peer_experts";
    if (!peers || !ep) return set_error(GTM_ERR_INVALID, "%s: null argument", fn);
    int rc = peer_common(fn, dims, layer, ep, ep->rank < GTM_EP_PEER_MAX_WORLD ? peers->workspace_dev[ep->rank] : nullptr,
                         ws_bytes);
    if (!rc) rc = peers_ok(fn, ep, peers);
    if (rc) return rc;
    int sms = 0;
    if ((rc = sm_count(fn, &sms))) return rc;
    rc = launch_ep_peer_experts(*layer, *ep, peers->workspace_dev, (cudaStream_t)stream, sms);
    if (rc == GTM_OK) clear_error();
    return rc;
}

GTM_API int gtm_moe_ep_peer_combine(const GtmDims* dims, const GtmLayer* layer, const GtmTokensIO* io,
                                    const GtmEpConfig* ep, void* ws, size_t ws_bytes, void* stream) {
    const char* fn = "gtm_moe_ep_peer_combine";
    int rc = peer_common(fn, dims, layer, ep, ws, ws_bytes);
    if (!rc) rc = ep_io(fn, io, ep, true, true);
    if (rc) return rc;
    if (io->num_tokens == 0) { clear_error(); return GTM_OK; }
    rc = launch_ep_peer_combine(*dims, *layer, *io, *ep, ws, (cudaStream_t)stream);
    if (rc == GTM_OK) clear_error();
    return rc;
}

// ---- device memory shared between processes (CUDA IPC) ------------------------------------------
static_assert(sizeof(cudaIpcMemHandle_t) == GTM_IPC_HANDLE_BYTES, "IPC handle size");

GTM_API int gtm_ipc_alloc(size_t bytes, void** dev_ptr, uint8_t handle_out[GTM_IPC_HANDLE_BYTES]) {
    if (!dev_ptr || !handle_out || bytes == 0) return set_error(GTM_ERR_INVALID, "gtm_ipc_alloc: bad argument");
    *dev_ptr = nullptr;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        return set_cuda_error("gtm_ipc_alloc", e);
    }
    memcpy(handle_out, &h, sizeof(h));
    *dev_ptr = p;
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_ipc_open(const uint8_t handle[GTM_IPC_HANDLE_BYTES], void** dev_ptr) {
    if (!handle || !dev_ptr) return set_error(GTM_ERR_INVALID, "gtm_ipc_open: null argument");
    *dev_ptr = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return set_cuda_error("gtm_ipc_open", e);
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_ipc_close(void* dev_ptr) {
    if (!dev_ptr) return set_error(GTM_ERR_INVALID, "gtm_ipc_close: null pointer");
    const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
    if (e != cudaSuccess) return set_cuda_error("gtm_ipc_close", e);
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_ipc_free(void* dev_ptr) {
    if (!dev_ptr) return set_error(GTM_ERR_INVALID, "gtm_ipc_free: null pointer");
    const cudaError_t e = cudaFree(dev_ptr);
    if (e != cudaSuccess) return set_cuda_error("gtm_ipc_free", e);
    clear_error();
    return GTM_OK;
}

}  // extern "C"

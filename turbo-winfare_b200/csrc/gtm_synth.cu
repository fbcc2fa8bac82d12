// On-device synthetic weights (include/gtmoe_synth.h), using the same element generators as
// the CPU oracle (gtm_synth.h), so both sides hold identical bytes.
#include <cstdint>
#include <cstring>
#include <cuda_runtime.h>

#include "gtmoe_synth.h"
#include "gtm_internal.h"
#include "gtm_synth.h"

namespace gtm {

// Fills a quantised matrix (packed words, scales, biases) for experts [e0, e0 + gridDim.y).
__global__ void synth_quant_kernel(uint64_t seed, uint32_t layer, uint32_t kind_w, uint32_t kind_s, uint32_t e0,
                                   uint64_t stride, uint8_t* base, uint64_t w_off, uint64_t s_off, uint64_t b_off,
                                   uint64_t words, uint64_t nscale, float zero_point) {
    const uint32_t e = e0 + blockIdx.y;
    uint8_t* blk = base + (uint64_t)blockIdx.y * stride;
    const uint64_t sw = gtm_stream(seed, layer, kind_w, e);
    const uint64_t ss = gtm_stream(seed, layer, kind_s, e);
    uint32_t* w = reinterpret_cast<uint32_t*>(blk + w_off);
    uint16_t* s = reinterpret_cast<uint16_t*>(blk + s_off);
    uint16_t* b = reinterpret_cast<uint16_t*>(blk + b_off);
    const uint64_t step = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < words; i += step) w[i] = gtm_qword(sw, i);
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nscale; i += step) {
        const uint16_t sc = gtm_scale_bits(ss, i);
        s[i] = sc;
        b[i] = gtm_bias_bits(sc, zero_point);
    }
}

// A standalone int4 matrix (zero point 8) into three separate arrays.
__global__ void synth_matrix_kernel(uint64_t seed, uint32_t layer, uint32_t kind_w, uint32_t kind_s, uint32_t* w,
                                    uint16_t* s, uint16_t* b, uint64_t words, uint64_t nscale) {
    const uint64_t sw = gtm_stream(seed, layer, kind_w, 0);
    const uint64_t ss = gtm_stream(seed, layer, kind_s, 0);
    const uint64_t step = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < words; i += step) w[i] = gtm_qword(sw, i);
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nscale; i += step) {
        const uint16_t sc = gtm_scale_bits(ss, i);
        s[i] = sc;
        b[i] = gtm_bias_bits(sc, 8.0f);
    }
}

__global__ void synth_zero_kernel(uint8_t* base, uint64_t stride, uint64_t from, uint64_t to) {
    uint8_t* blk = base + (uint64_t)blockIdx.y * stride;
    for (uint64_t i = from + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < to; i += (uint64_t)gridDim.x * blockDim.x)
        blk[i] = 0;
}

__global__ void synth_vec_kernel(uint64_t seed, uint32_t layer, uint32_t kind, uint32_t n, int mode, uint16_t* dst) {
    const uint64_t st = gtm_stream(seed, layer, kind, 0);
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        dst[i] = mode == 0 ? gtm_norm_weight_bits(st, i) : gtm_per_expert_scale_bits(st, i);
}

__global__ void synth_scalar_kernel(uint16_t* dst) { *dst = GTM_LAYER_SCALAR_BITS; }

__global__ void synth_x_kernel(uint64_t seed, uint32_t token0, uint32_t hidden, float* dst) {
    const uint32_t t = token0 + blockIdx.y;
    const uint64_t st = gtm_stream(seed, 0xFFFFu, GTM_K_X, t);
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x)
        dst[(uint64_t)blockIdx.y * hidden + i] = gtm_normal(st, i);
}

static void quant(uint64_t seed, uint32_t layer, uint32_t kw, uint32_t ks, uint32_t e0, uint32_t count, uint64_t stride,
                  uint8_t* base, uint64_t wo, uint64_t so, uint64_t bo, uint32_t rows, uint32_t in_dim, int bits,
                  cudaStream_t st) {
    const uint64_t words = (uint64_t)rows * in_dim * bits / 32;
    const uint64_t nsc = (uint64_t)rows * (in_dim / 64);
    dim3 grid(256, count);
    synth_quant_kernel<<<grid, 256, 0, st>>>(seed, layer, kw, ks, e0, stride, base, wo, so, bo, words, nsc,
                                             bits == 4 ? 8.0f : 128.0f);
}

}  // namespace gtm

using namespace gtm;

extern "C" {

GTM_API int gtm_synth_expert_layout(uint32_t hidden, uint32_t inter, uint64_t offsets[9], uint64_t* stride) {
    if (!offsets || !stride || hidden % 64 || inter % 64 || !hidden || !inter)
        return set_error(GTM_ERR_INVALID, "gtm_synth_expert_layout: bad arguments");
    GtmExpertBlockLayout L = gtm_expert_block_layout(hidden, inter);
    memcpy(offsets, L.offset, sizeof(L.offset));
    *stride = L.stride;
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_synth_resident_layout(uint32_t hidden, uint32_t ffn, uint32_t experts, uint64_t offsets[20],
                                      uint64_t* total) {
    if (!offsets || !total || hidden % 64 || ffn % 64 || !hidden || !ffn || !experts)
        return set_error(GTM_ERR_INVALID, "gtm_synth_resident_layout: bad arguments");
    GtmResidentLayout R = gtm_resident_layout(hidden, ffn, experts);
    memcpy(offsets, R.offset, sizeof(R.offset));
    *total = R.total;
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_synth_experts(uint64_t seed, uint32_t layer, uint32_t hidden, uint32_t inter, uint32_t first,
                              uint32_t count, void* dst, void* stream) {
    if (!dst || !count || hidden % 64 || inter % 64) return set_error(GTM_ERR_INVALID, "gtm_synth_experts: bad arguments");
    cudaStream_t st = (cudaStream_t)stream;
    GtmExpertBlockLayout B = gtm_expert_block_layout(hidden, inter);
    uint8_t* base = static_cast<uint8_t*>(dst);
    quant(seed, layer, GTM_K_EXP_GATE_W, GTM_K_EXP_GATE_S, first, count, B.stride, base, B.offset[0], B.offset[1],
          B.offset[2], inter, hidden, 4, st);
    quant(seed, layer, GTM_K_EXP_UP_W, GTM_K_EXP_UP_S, first, count, B.stride, base, B.offset[3], B.offset[4],
          B.offset[5], inter, hidden, 4, st);
    quant(seed, layer, GTM_K_EXP_DOWN_W, GTM_K_EXP_DOWN_S, first, count, B.stride, base, B.offset[6], B.offset[7],
          B.offset[8], hidden, inter, 4, st);
    if (B.stride > B.used) synth_zero_kernel<<<dim3(16, count), 256, 0, st>>>(base, B.stride, B.used, B.stride);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("gtm_synth_experts", e);
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_synth_resident(uint64_t seed, uint32_t layer, uint32_t hidden, uint32_t ffn, uint32_t experts,
                               void* dst, void* stream) {
    if (!dst || hidden % 64 || ffn % 64 || !experts) return set_error(GTM_ERR_INVALID, "gtm_synth_resident: bad arguments");
    cudaStream_t st = (cudaStream_t)stream;
    GtmResidentLayout R = gtm_resident_layout(hidden, ffn, experts);
    uint8_t* o = static_cast<uint8_t*>(dst);
    cudaError_t e = cudaMemsetAsync(o, 0, R.total, st);
    if (e != cudaSuccess) return set_cuda_error("gtm_synth_resident: memset", e);
    quant(seed, layer, GTM_K_ROUTER_W, GTM_K_ROUTER_S, 0, 1, 0, o, R.offset[GTM_R_ROUTER_W], R.offset[GTM_R_ROUTER_S],
          R.offset[GTM_R_ROUTER_B], experts, hidden, 8, st);
    quant(seed, layer, GTM_K_SH_GATE_W, GTM_K_SH_GATE_S, 0, 1, 0, o, R.offset[GTM_R_SH_GATE_W], R.offset[GTM_R_SH_GATE_S],
          R.offset[GTM_R_SH_GATE_B], ffn, hidden, 4, st);
    quant(seed, layer, GTM_K_SH_UP_W, GTM_K_SH_UP_S, 0, 1, 0, o, R.offset[GTM_R_SH_UP_W], R.offset[GTM_R_SH_UP_S],
          R.offset[GTM_R_SH_UP_B], ffn, hidden, 4, st);
    quant(seed, layer, GTM_K_SH_DOWN_W, GTM_K_SH_DOWN_S, 0, 1, 0, o, R.offset[GTM_R_SH_DOWN_W], R.offset[GTM_R_SH_DOWN_S],
          R.offset[GTM_R_SH_DOWN_B], hidden, ffn, 4, st);
    const uint32_t kinds[6] = {GTM_K_ROUTER_SCALE, GTM_K_W_PRE, GTM_K_W_PRE2, GTM_K_W_PF1, GTM_K_W_PF2, GTM_K_W_PF};
    const int regions[6] = {GTM_R_ROUTER_SCALE, GTM_R_W_PRE, GTM_R_W_PRE2, GTM_R_W_PF1, GTM_R_W_PF2, GTM_R_W_PF};
    for (int k = 0; k < 6; ++k)
        synth_vec_kernel<<<8, 256, 0, st>>>(seed, layer, kinds[k], hidden, 0,
                                            reinterpret_cast<uint16_t*>(o + R.offset[regions[k]]));
    synth_vec_kernel<<<1, 256, 0, st>>>(seed, layer, GTM_K_PER_EXPERT_SCALE, experts, 1,
                                        reinterpret_cast<uint16_t*>(o + R.offset[GTM_R_PER_EXPERT_SCALE]));
    synth_scalar_kernel<<<1, 1, 0, st>>>(reinterpret_cast<uint16_t*>(o + R.offset[GTM_R_LAYER_SCALAR]));
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("gtm_synth_resident", e);
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_synth_x(uint64_t seed, uint32_t token0, uint32_t count, uint32_t hidden, float* dst, void* stream) {
    if (!dst || !count || !hidden) return set_error(GTM_ERR_INVALID, "gtm_synth_x: bad arguments");
    synth_x_kernel<<<dim3((hidden + 255) / 256, count), 256, 0, (cudaStream_t)stream>>>(seed, token0, hidden, dst);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("gtm_synth_x", e);
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_synth_quant(uint64_t seed, uint32_t layer, uint32_t kind_w, uint32_t kind_s, uint32_t rows,
                            uint32_t in_dim, void* w_dev, uint16_t* s_dev, uint16_t* b_dev, void* stream) {
    if (!w_dev || !s_dev || !b_dev || rows == 0 || in_dim == 0 || in_dim % 64 != 0)
        return set_error(GTM_ERR_INVALID, "gtm_synth_quant: null pointer or in_dim %u not a multiple of 64", in_dim);
    synth_matrix_kernel<<<512, 256, 0, (cudaStream_t)stream>>>(seed, layer, kind_w, kind_s, static_cast<uint32_t*>(w_dev),
                                                               s_dev, b_dev, (uint64_t)rows * in_dim / 8,
                                                               (uint64_t)rows * (in_dim / 64));
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("gtm_synth_quant", e);
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_synth_norm(uint64_t seed, uint32_t layer, uint32_t kind, uint32_t n, uint16_t* dst_dev, void* stream) {
    if (!dst_dev || n == 0) return set_error(GTM_ERR_INVALID, "gtm_synth_norm: null pointer or n = 0");
    synth_vec_kernel<<<(n + 255) / 256 < 64 ? (n + 255) / 256 : 64, 256, 0, (cudaStream_t)stream>>>(seed, layer, kind, n,
                                                                                                   0, dst_dev);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("gtm_synth_norm", e);
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_synth_layer_desc(uint32_t hidden, uint32_t moe_inter, uint32_t ffn, uint32_t experts,
                                 const void* resident_dev, const void* experts_dev, GtmLayer* out) {
    if (!out || !resident_dev || !experts_dev) return set_error(GTM_ERR_INVALID, "gtm_synth_layer_desc: null argument");
    GtmResidentLayout R = gtm_resident_layout(hidden, ffn, experts);
    GtmExpertBlockLayout B = gtm_expert_block_layout(hidden, moe_inter);
    GtmLayer L;
    memset(&L, 0, sizeof(L));
    L.resident_dev = resident_dev;
    L.router = {R.offset[GTM_R_ROUTER_W], R.offset[GTM_R_ROUTER_S], R.offset[GTM_R_ROUTER_B]};
    L.router_scale = R.offset[GTM_R_ROUTER_SCALE];
    L.per_expert_scale = R.offset[GTM_R_PER_EXPERT_SCALE];
    L.shared_gate = {R.offset[GTM_R_SH_GATE_W], R.offset[GTM_R_SH_GATE_S], R.offset[GTM_R_SH_GATE_B]};
    L.shared_up = {R.offset[GTM_R_SH_UP_W], R.offset[GTM_R_SH_UP_S], R.offset[GTM_R_SH_UP_B]};
    L.shared_down = {R.offset[GTM_R_SH_DOWN_W], R.offset[GTM_R_SH_DOWN_S], R.offset[GTM_R_SH_DOWN_B]};
    L.pre_ffn_norm = R.offset[GTM_R_W_PRE];
    L.pre_ffn_norm_2 = R.offset[GTM_R_W_PRE2];
    L.post_ffn_norm_1 = R.offset[GTM_R_W_PF1];
    L.post_ffn_norm_2 = R.offset[GTM_R_W_PF2];
    L.post_ffn_norm = R.offset[GTM_R_W_PF];
    L.layer_scalar = R.offset[GTM_R_LAYER_SCALAR];
    L.experts_dev = experts_dev;
    L.expert_stride = B.stride;
    L.expert_gate = {B.offset[0], B.offset[1], B.offset[2]};
    L.expert_up = {B.offset[3], B.offset[4], B.offset[5]};
    L.expert_down = {B.offset[6], B.offset[7], B.offset[8]};
    *out = L;
    clear_error();
    return GTM_OK;
}

}  // extern "C"

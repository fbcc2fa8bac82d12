/*
 * Deterministic synthetic MoE weights and activations, shared by the CUDA generator kernels
 * and the CPU oracle so that both sides hold byte-identical tensors.
 *
 * Every value is a pure function of (seed, layer, tensor kind, expert, element index): a
 * splitmix64-style counter hash, then integer arithmetic and single IEEE-754 float
 * multiplies/adds (no transcendental functions, no fused multiply-add), so the host compiler
 * and nvcc produce the same bits. Normal deviates use an Irwin-Hall(4) sum of four 16-bit
 * uniforms scaled to unit variance (bounded at +-3.46 sigma); that stands in for N(0, 1).
 *
 * Distributions follow the benchmark configuration of the reference MoE layer
 * (Gemma-4-26B-A4B shapes, MLX affine quantisation, group 64):
 *   expert / shared-expert int4:  q ~ U{0..15}, scale = bf16|0.02 n|, bias = -8 * scale
 *   router int8 (unsigned bytes): q ~ U{0..255}, scale = bf16|0.02 n|, bias = -128 * scale
 *   RMSNorm weights, router.scale: bf16(1 + 0.1 n);  per_expert_scale: bf16 U(0.5, 1.5)
 *   layer_scalar: bf16(1.0);  activations: fp32 n.
 *
 * The expert block byte layout is the .gturbo converter order (gate, up, down; weight,
 * scales, biases each), packed tight and padded to a 16 KB stride
 * (tools/convert_hf_to_gturbo.py:93-98 and :379-419, include/gturbo/packed_experts.hpp:34-59).
 */
#ifndef GTM_SYNTH_H
#define GTM_SYNTH_H

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define GTM_HD __host__ __device__ __forceinline__
#else
#define GTM_HD static inline
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- tensor kinds (stream ids) ---------------------------------------------------------- */
enum {
    GTM_K_X = 0,            /* block input activation (per token)            */
    GTM_K_EXP_GATE_W = 1, GTM_K_EXP_GATE_S = 2,
    GTM_K_EXP_UP_W = 3,   GTM_K_EXP_UP_S = 4,
    GTM_K_EXP_DOWN_W = 5, GTM_K_EXP_DOWN_S = 6,
    GTM_K_SH_GATE_W = 7,  GTM_K_SH_GATE_S = 8,
    GTM_K_SH_UP_W = 9,    GTM_K_SH_UP_S = 10,
    GTM_K_SH_DOWN_W = 11, GTM_K_SH_DOWN_S = 12,
    GTM_K_ROUTER_W = 13,  GTM_K_ROUTER_S = 14,
    GTM_K_ROUTER_SCALE = 15, GTM_K_PER_EXPERT_SCALE = 16,
    GTM_K_W_PRE = 17, GTM_K_W_PRE2 = 18, GTM_K_W_PF1 = 19, GTM_K_W_PF2 = 20, GTM_K_W_PF = 21,
    GTM_K_ROUTE_LOGITS = 22 /* uniform-random routing logits (prefill configuration) */
};

/* ---- float helpers with explicit single rounding ---------------------------------------- */
GTM_HD float gtm_u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
GTM_HD uint32_t gtm_f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

GTM_HD float gtm_fmul(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fmul_rn(a, b);
#else
    return a * b;   /* host TUs are built with -ffp-contract=off */
#endif
}
GTM_HD float gtm_fadd(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fadd_rn(a, b);
#else
    return a + b;
#endif
}

/* float -> bf16 bits, round to nearest even (NaN is not produced by this generator). */
GTM_HD uint16_t gtm_bf16_rne(float f) {
    uint32_t w = gtm_f2u(f);
    uint32_t rounding = 0x7FFFu + ((w >> 16) & 1u);
    return (uint16_t)((w + rounding) >> 16);
}
GTM_HD float gtm_bf16f(uint16_t b) { return gtm_u2f((uint32_t)b << 16); }

/* ---- counter hash --------------------------------------------------------------------- */
GTM_HD uint64_t gtm_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
/* Stream key for one tensor. `layer` is 0..N-1, `expert` is 0 for non-expert tensors. */
GTM_HD uint64_t gtm_stream(uint64_t seed, uint32_t layer, uint32_t kind, uint32_t expert) {
    uint64_t s = gtm_mix64(seed + 0x5851F42D4C957F2Dull);
    s = gtm_mix64(s ^ ((uint64_t)layer << 20) ^ (uint64_t)kind);
    return gtm_mix64(s + ((uint64_t)expert << 8));
}
GTM_HD uint64_t gtm_hash(uint64_t stream, uint64_t idx) { return gtm_mix64(stream + idx * 0xD1B54A32D192ED03ull); }

/* Irwin-Hall(4) deviate with unit variance. 1/sigma = 0x375db3d7 (sigma = 75674.454). */
GTM_HD float gtm_normal(uint64_t stream, uint64_t idx) {
    uint64_t h = gtm_hash(stream, idx);
    int32_t s = 2 * (int32_t)((h & 0xFFFFu) + ((h >> 16) & 0xFFFFu) + ((h >> 32) & 0xFFFFu) + (h >> 48))
                - 4 * 65535;
    return gtm_fmul((float)s, gtm_u2f(0x375db3d7u));
}
/* Uniform in [0, 1) with 24 random bits. */
GTM_HD float gtm_uniform(uint64_t stream, uint64_t idx) {
    uint64_t h = gtm_hash(stream, idx);
    return gtm_fmul((float)(uint32_t)(h >> 40), gtm_u2f(0x33800000u)); /* * 2^-24 */
}

/* Packed quantised word `w` of a tensor: eight int4 nibbles or four uint8 bytes. */
GTM_HD uint32_t gtm_qword(uint64_t stream, uint64_t w) { return (uint32_t)(gtm_hash(stream, w) >> 16); }
/* Group scale bf16|0.02 n| and the matching affine bias (-zero_point * scale). */
GTM_HD uint16_t gtm_scale_bits(uint64_t stream, uint64_t i) {
    float s = gtm_fmul(0.02f, gtm_normal(stream, i));
    return gtm_bf16_rne(s < 0.0f ? -s : s);
}
GTM_HD uint16_t gtm_bias_bits(uint16_t scale_bits, float zero_point) {
    return gtm_bf16_rne(gtm_fmul(-zero_point, gtm_bf16f(scale_bits)));  /* exact: power-of-two * bf16 */
}
GTM_HD uint16_t gtm_norm_weight_bits(uint64_t stream, uint64_t i) {
    return gtm_bf16_rne(gtm_fadd(1.0f, gtm_fmul(0.1f, gtm_normal(stream, i))));
}
GTM_HD uint16_t gtm_per_expert_scale_bits(uint64_t stream, uint64_t i) {
    return gtm_bf16_rne(gtm_fadd(0.5f, gtm_uniform(stream, i)));
}
#define GTM_LAYER_SCALAR_BITS ((uint16_t)0x3F80u) /* bf16(1.0) */

/* ---- byte layouts ----------------------------------------------------------------------- */
#define GTM_ALIGN 16384ull
GTM_HD uint64_t gtm_align_up(uint64_t n) { return (n + GTM_ALIGN - 1) / GTM_ALIGN * GTM_ALIGN; }

/* One routed-expert block: sub-tensor offsets in converter order.
 * idx: 0 gate.weight 1 gate.scales 2 gate.biases 3 up.weight ... 8 down.biases */
typedef struct GtmExpertBlockLayout {
    uint64_t offset[9];
    uint64_t size[9];
    uint64_t used;     /* bytes before padding */
    uint64_t stride;   /* padded to 16 KB */
} GtmExpertBlockLayout;

GTM_HD GtmExpertBlockLayout gtm_expert_block_layout(uint32_t hidden, uint32_t inter) {
    GtmExpertBlockLayout L;
    uint64_t wsz = (uint64_t)inter * hidden / 2;          /* [inter][hidden] int4, same for down */
    uint64_t gu_s = (uint64_t)inter * (hidden / 64) * 2;  /* gate/up scales */
    uint64_t dn_s = (uint64_t)hidden * (inter / 64) * 2;  /* down scales */
    uint64_t sz[9] = {wsz, gu_s, gu_s, wsz, gu_s, gu_s, wsz, dn_s, dn_s};
    uint64_t cur = 0;
    for (int i = 0; i < 9; ++i) { L.offset[i] = cur; L.size[i] = sz[i]; cur += sz[i]; }
    L.used = cur;
    L.stride = gtm_align_up(cur);
    return L;
}

/* One layer's resident (non-expert) tensors, each region on a 16 KB boundary like resident.bin. */
enum {
    GTM_R_ROUTER_W = 0, GTM_R_ROUTER_S, GTM_R_ROUTER_B, GTM_R_ROUTER_SCALE, GTM_R_PER_EXPERT_SCALE,
    GTM_R_SH_GATE_W, GTM_R_SH_GATE_S, GTM_R_SH_GATE_B,
    GTM_R_SH_UP_W, GTM_R_SH_UP_S, GTM_R_SH_UP_B,
    GTM_R_SH_DOWN_W, GTM_R_SH_DOWN_S, GTM_R_SH_DOWN_B,
    GTM_R_W_PRE, GTM_R_W_PRE2, GTM_R_W_PF1, GTM_R_W_PF2, GTM_R_W_PF, GTM_R_LAYER_SCALAR,
    GTM_R_COUNT
};
typedef struct GtmResidentLayout {
    uint64_t offset[GTM_R_COUNT];
    uint64_t size[GTM_R_COUNT];
    uint64_t total;
} GtmResidentLayout;

GTM_HD GtmResidentLayout gtm_resident_layout(uint32_t hidden, uint32_t ffn, uint32_t experts) {
    GtmResidentLayout L;
    uint64_t H = hidden, F = ffn, E = experts;
    uint64_t sz[GTM_R_COUNT] = {
        E * H, E * (H / 64) * 2, E * (H / 64) * 2, H * 2, E * 2,
        F * H / 2, F * (H / 64) * 2, F * (H / 64) * 2,
        F * H / 2, F * (H / 64) * 2, F * (H / 64) * 2,
        H * F / 2, H * (F / 64) * 2, H * (F / 64) * 2,
        H * 2, H * 2, H * 2, H * 2, H * 2, 2};
    uint64_t cur = 0;
    for (int i = 0; i < GTM_R_COUNT; ++i) { L.offset[i] = cur; L.size[i] = sz[i]; cur = gtm_align_up(cur + sz[i]); }
    L.total = cur;
    return L;
}

/* ---- element generators (one call per 32-bit word / per bf16) ----------------------------
 * These produce the contents of the regions above. For a quantised matrix with `rows` rows and
 * `in_dim` inputs, word w of the packed weights and group entry i = row * groups + g of the
 * scales/biases are generated independently, so any subset can be produced on demand.      */
GTM_HD uint32_t gtm_gen_weight_word(uint64_t seed, uint32_t layer, uint32_t kind, uint32_t expert, uint64_t w) {
    return gtm_qword(gtm_stream(seed, layer, kind, expert), w);
}
GTM_HD uint16_t gtm_gen_scale(uint64_t seed, uint32_t layer, uint32_t kind, uint32_t expert, uint64_t i) {
    return gtm_scale_bits(gtm_stream(seed, layer, kind, expert), i);
}

#ifdef __cplusplus
}
#endif
#endif /* GTM_SYNTH_H */

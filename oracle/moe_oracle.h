/*
 * TEST INFRASTRUCTURE ONLY. CPU restatement of the reference MoE block, used by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker. Nothing on the
 * product path links or calls this code.
 *
 * Follows the reference's scalar FP32 forward (src/cpu_reference.cpp) operation by
 * operation so that results are bit-identical with it; each function names the lines it
 * restates. Build with -O2 -ffp-contract=off (no FMA contraction, no fast-math).
 */
#ifndef GTM_MOE_ORACLE_H
#define GTM_MOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* An affine-quantised matrix view (cpu_reference.hpp:42-53 QuantTensor). */
typedef struct orc_qt {
    const uint8_t* data;      /* packed: 4-bit low nibble first, or one byte per element  */
    const uint16_t* scales;   /* bf16 [rows][in_dim/64] */
    const uint16_t* biases;   /* bf16 [rows][in_dim/64] */
    uint32_t rows, in_dim;
    int bits;                 /* 4 or 8 */
} orc_qt;

typedef struct orc_layer {
    uint32_t hidden, moe_inter, ffn_inter, num_experts, top_k;
    float eps;
    orc_qt router;                              /* router.proj (8-bit)              */
    const uint16_t* router_scale;               /* router.scale bf16[hidden]        */
    const uint16_t* per_expert_scale;           /* router.per_expert_scale bf16[E]  */
    orc_qt sh_gate, sh_up, sh_down;             /* mlp.{gate,up,down}_proj          */
    const uint16_t *w_pre, *w_pre2, *w_pf1, *w_pf2, *w_pf;   /* the five RMSNorm weights */
    uint16_t layer_scalar;                      /* bf16 */
    /* Routed experts: expert e's block starts at experts + e * expert_stride, its nine
     * sub-tensors at the layout.expertBlock offsets (gate w/s/b, up w/s/b, down w/s/b). */
    const uint8_t* experts;
    uint64_t expert_stride;
    uint64_t sub_off[9];
} orc_layer;

/* Per-token outputs of one MoE block. */
typedef struct orc_block_out {
    float* hidden_out;        /* [hidden] new residual stream        */
    float* h1;                /* [hidden] normed shared-expert output */
    float* h2;                /* [hidden] weighted routed-expert sum  */
    float* logits;            /* [E] router logits (nullable)         */
    uint32_t* top_idx;        /* [K] (nullable)                       */
    float* top_w;             /* [K] (nullable)                       */
} orc_block_out;

float orc_bf16(uint16_t bits);
uint16_t orc_bf16_rne(float f);
float orc_gelu_tanh(float x);
void orc_rms_norm(const float* x, const uint16_t* w, size_t n, float eps, float* out);
void orc_matvec(const orc_qt* t, const float* x, float* out);
void orc_topk(const float* logits, uint32_t n, uint32_t k, const uint16_t* per_expert_scale,
              uint32_t* idx, float* w);
/* One MoE block for one token. `logit_bias` (nullable, [E]) is added to the router logits
 * before selection; `route_logits` (nullable, [E]) replaces the router GEMV outright. */
int orc_moe_block(const orc_layer* L, const float* hidden_in, const float* logit_bias,
                  const float* route_logits, const orc_block_out* out);

/* ---- synthetic model (same generator as the CUDA side) -------------------------------- */
/* Fills a whole layer's resident image (layout from gtm_resident_layout) on the host. */
void orc_synth_resident(uint64_t seed, uint32_t layer, uint32_t hidden, uint32_t ffn,
                        uint32_t experts, uint8_t* image);
/* Fills one routed expert's block (layout from gtm_expert_block_layout). */
void orc_synth_expert(uint64_t seed, uint32_t layer, uint32_t expert, uint32_t hidden,
                      uint32_t inter, uint8_t* block);
/* Block input activation x ~ N(0,1) for token `token`. */
void orc_synth_x(uint64_t seed, uint32_t token, uint32_t hidden, float* x);
/* Builds an orc_layer view over a resident image and an expert-set base pointer. */
void orc_layer_view(orc_layer* L, const uint8_t* resident, const uint8_t* experts,
                    uint32_t hidden, uint32_t moe_inter, uint32_t ffn, uint32_t experts_n,
                    uint32_t top_k, float eps);

/* A lazily generated synthetic layer: experts are materialised on first use. */
typedef struct orc_synth_layer orc_synth_layer;
orc_synth_layer* orc_synth_layer_create(uint64_t seed, uint32_t layer, uint32_t hidden,
                                        uint32_t moe_inter, uint32_t ffn, uint32_t experts,
                                        uint32_t top_k, float eps);
void orc_synth_layer_destroy(orc_synth_layer* s);
/* The layer's weight view, and on-demand generation of the given experts. */
const orc_layer* orc_synth_layer_view(const orc_synth_layer* s);
void orc_synth_layer_ensure(orc_synth_layer* s, const uint32_t* experts, uint32_t n);
/* Views, router and top-k only; generates the selected experts. idx_out may be NULL. */
void orc_synth_layer_route(orc_synth_layer* s, const float* hidden_in, const float* logit_bias,
                           const float* route_logits, uint32_t* idx_out);
/* Runs the block; generates the selected experts first. */
int orc_synth_layer_block(orc_synth_layer* s, const float* hidden_in, const float* logit_bias,
                          const float* route_logits, const orc_block_out* out);
/* A stack of `n` synthetic layers with a weightless RMSNorm after every layer but the last.
 * Per-layer outputs are written at [l * hidden] / [l * top_k] when non-null. */
int orc_synth_stack(orc_synth_layer** layers, uint32_t n, const float* hidden_in,
                    float* hidden_out, float* hidden_per_layer, uint32_t* idx_per_layer,
                    float* w_per_layer);

#ifdef __cplusplus
}
#endif
#endif

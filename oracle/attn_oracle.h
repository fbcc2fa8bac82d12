/*
 * TEST INFRASTRUCTURE ONLY. CPU restatement of the reference's decoder remainder around the MoE
 * block: the embedding lookup and one layer's attention step with its KV cache
 * (src/cpu_reference.cpp:108-140, 322-420). It is the checker for a device attention path;
 * nothing on the product path links or calls it.
 *
 * Pinned against the same steps assembled from the reference's own compiled helpers
 * (oracle/_ref/libgtref.so) and the fixtures of tests/golden/attn.npz. Build with -O2
 * -ffp-contract=off; the float transcendentals (powf, cosf, sinf, expf) are the C library's,
 * the routines the reference's std:: float overloads call on this host.
 */
#ifndef GTM_ATTN_ORACLE_H
#define GTM_ATTN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#include "moe_oracle.h"

#ifdef __cplusplus
extern "C" {
#endif

/* The per-layer attention shape (cpu_reference.cpp:333-341, include/gturbo/manifest.hpp:22-49). */
typedef struct orc_attn_shape {
    uint32_t hidden;          /* 2816 */
    uint32_t num_heads;       /* 16 */
    uint32_t head_dim;        /* 256 sliding-window layers, 512 full-attention layers */
    uint32_t kv_heads;        /* 8 sliding, 2 full */
    uint32_t rotated_pairs;   /* head_dim / 2 sliding; head_dim * 0.25 / 2 full */
    float theta;              /* 1e4 sliding, 1e6 full */
    int32_t sliding_window;   /* 1024; 0 = full attention (attend to every position) */
    int32_t k_eq_v;           /* full layers: V is the raw k_proj output (no v_proj) */
    float eps;
} orc_attn_shape;

/* One layer's attention weights; v is ignored when k_eq_v. */
typedef struct orc_attn_layer {
    orc_qt q, k, v, o;
    const uint16_t* input_norm;   /* [hidden] bf16 */
    const uint16_t* q_norm;       /* [head_dim] bf16 */
    const uint16_t* k_norm;       /* [head_dim] bf16 */
} orc_attn_layer;

/* dequant_row then * sqrt(hidden) (cpu_reference.cpp:322-330). embed: [vocab][hidden] int4. */
void orc_embed(const orc_qt* embed, uint32_t token, float* out);
/* rope_neox (cpu_reference.cpp:126-140), in place. */
void orc_rope_neox(float* vec, uint32_t head_dim, uint32_t rotated_pairs, float position, float theta);
/* Per head: RMS norm with weight w (NULL = no scale), then NeoX RoPE of rotated_pairs pairs at
 * `position` (cpu_reference.cpp:360-376; the QKVEpilogue kernel's contract), in place. */
void orc_qkv_epilogue(float* vec, uint32_t heads, uint32_t head_dim, const uint16_t* w, float eps,
                      uint32_t rotated_pairs, float position, float theta);
/* The attention core (cpu_reference.cpp:382-414): for every query head, scores q.k (scale 1.0)
 * over positions [first, n_pos), a float softmax, and the weighted V sum into ctx [heads *
 * head_dim]. Position t lives in cache row t % capacity (the reference's ring KV,
 * kv_cache.cpp:36-50); capacity >= n_pos is a linear cache. */
void orc_attention_core(const float* q, const float* k_cache, const float* v_cache, uint32_t q_heads,
                        uint32_t kv_heads, uint32_t head_dim, int n_pos, int first, uint32_t capacity, float* ctx);
/* One attention step at position `pos` (cpu_reference.cpp:345-417). k_cache / v_cache hold
 * pos + 1 rows of kv_heads * head_dim floats (row t = position t); rows 0..pos-1 come from
 * earlier steps and this call writes row pos. attn_out [hidden] is o_proj's output; q_out
 * [num_heads * head_dim], k_out and v_out [kv_heads * head_dim] (nullable) receive the
 * post-norm, post-RoPE vectors. Returns 0. */
int orc_attention_step(const orc_attn_shape* s, const orc_attn_layer* L, int pos, const float* hidden,
                       float* k_cache, float* v_cache, float* attn_out, float* q_out, float* k_out, float* v_out);

#ifdef __cplusplus
}
#endif
#endif

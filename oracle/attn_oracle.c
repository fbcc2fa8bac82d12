/*
 * TEST INFRASTRUCTURE ONLY. CPU restatement of the reference's embedding lookup and attention
 * step; see attn_oracle.h. Each function names the lines of src/cpu_reference.cpp it follows.
 */
#include "attn_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* cpu_reference.cpp:108-124 (dequant_row: q * scale + bias per element, low nibble first) and
 * :322-330 (times sqrt(hidden) as a float). */
void orc_embed(const orc_qt* t, uint32_t token, float* out) {
    const uint32_t d = t->in_dim, groups = d / 64;
    const uint8_t* w = t->data + (size_t)token * (d / 2);
    const uint16_t* sc = t->scales + (size_t)token * groups;
    const uint16_t* bi = t->biases + (size_t)token * groups;
    for (uint32_t g = 0; g < groups; ++g) {
        const float s = orc_bf16(sc[g]), b = orc_bf16(bi[g]);
        for (uint32_t j = 0; j < 64; ++j) {
            const uint32_t c = g * 64 + j;
            const uint8_t byte = w[c >> 1];
            const uint32_t q = (c & 1u) ? (uint32_t)(byte >> 4) : (uint32_t)(byte & 15u);
            out[c] = (float)q * s + b;
        }
    }
    const float scale = sqrtf((float)d);
    for (uint32_t c = 0; c < d; ++c) out[c] *= scale;
}

/* cpu_reference.cpp:126-140: pairs (i, i + head_dim/2), angle = position * theta^(-2i/head_dim),
 * all in float. */
void orc_rope_neox(float* vec, uint32_t head_dim, uint32_t rotated_pairs, float position, float theta) {
    const uint32_t half = head_dim / 2;
    for (uint32_t i = 0; i < rotated_pairs; ++i) {
        const float freq = powf(theta, -(float)(2 * i) / (float)head_dim);
        const float angle = position * freq;
        const float c = cosf(angle), s = sinf(angle);
        const float x0 = vec[i], x1 = vec[i + half];
        vec[i] = x0 * c - x1 * s;
        vec[i + half] = x0 * s + x1 * c;
    }
}

void orc_qkv_epilogue(float* vec, uint32_t heads, uint32_t head_dim, const uint16_t* w, float eps,
                      uint32_t rotated_pairs, float position, float theta) {
    float* scratch = malloc(head_dim * sizeof(float));
    for (uint32_t h = 0; h < heads; ++h) {
        orc_rms_norm(vec + (size_t)h * head_dim, w, head_dim, eps, scratch);
        memcpy(vec + (size_t)h * head_dim, scratch, head_dim * sizeof(float));
        if (rotated_pairs) orc_rope_neox(vec + (size_t)h * head_dim, head_dim, rotated_pairs, position, theta);
    }
    free(scratch);
}

void orc_attention_core(const float* q, const float* k_cache, const float* v_cache, uint32_t q_heads,
                        uint32_t kv_heads, uint32_t head_dim, int n_pos, int first, uint32_t capacity, float* ctx) {
    const size_t row = (size_t)kv_heads * head_dim;
    const uint32_t gqa = q_heads / kv_heads;
    float* scores = malloc((size_t)(n_pos > 0 ? n_pos : 1) * sizeof(float));
    memset(ctx, 0, (size_t)q_heads * head_dim * sizeof(float));
    for (uint32_t h = 0; h < q_heads; ++h) {
        const uint32_t kvh = h / gqa;
        const float* qh = q + (size_t)h * head_dim;
        float best = -1e30f;
        for (int t = first; t < n_pos; ++t) {
            const float* kt = k_cache + (size_t)((uint32_t)t % capacity) * row + kvh * head_dim;
            float dot = 0.0f;
            for (uint32_t d = 0; d < head_dim; ++d) dot += qh[d] * kt[d];
            scores[t] = dot;
            best = best < dot ? dot : best;   /* std::max(best, dot) */
        }
        float sum = 0.0f;
        for (int t = first; t < n_pos; ++t) {
            const float e = expf(scores[t] - best);
            scores[t] = e;
            sum += e;
        }
        float* out = ctx + (size_t)h * head_dim;
        for (int t = first; t < n_pos; ++t) {
            const float wgt = scores[t] / sum;
            const float* vt = v_cache + (size_t)((uint32_t)t % capacity) * row + kvh * head_dim;
            for (uint32_t d = 0; d < head_dim; ++d) out[d] += wgt * vt[d];
        }
    }
    free(scores);
}

/* cpu_reference.cpp:345-417. */
int orc_attention_step(const orc_attn_shape* s, const orc_attn_layer* L, int pos, const float* hidden,
                       float* k_cache, float* v_cache, float* attn_out, float* q_out, float* k_out, float* v_out) {
    const uint32_t D = s->hidden, hd = s->head_dim, H = s->num_heads, KV = s->kv_heads;
    const size_t qn = (size_t)H * hd, kn = (size_t)KV * hd;
    float* normed = malloc(D * sizeof(float));
    float* q = malloc(qn * sizeof(float));
    float* k = malloc(kn * sizeof(float));
    float* v = malloc(kn * sizeof(float));
    float* ctx = malloc(qn * sizeof(float));

    /* input norm, projections (full layers: V is the raw k_proj output, :349-358) */
    orc_rms_norm(hidden, L->input_norm, D, s->eps, normed);
    orc_matvec(&L->q, normed, q);
    orc_matvec(&L->k, normed, k);
    if (s->k_eq_v)
        memcpy(v, k, kn * sizeof(float));
    else
        orc_matvec(&L->v, normed, v);

    /* per-head q/k norms then RoPE; V: no-scale norm, no rotation (:360-376). The reference
     * interleaves k and v per head; each head's values depend only on that head, so the order
     * of the two loops does not change a bit. */
    orc_qkv_epilogue(q, H, hd, L->q_norm, s->eps, s->rotated_pairs, (float)pos, s->theta);
    orc_qkv_epilogue(k, KV, hd, L->k_norm, s->eps, s->rotated_pairs, (float)pos, s->theta);
    orc_qkv_epilogue(v, KV, hd, NULL, s->eps, 0, 0.0f, 0.0f);
    memcpy(k_cache + (size_t)pos * kn, k, kn * sizeof(float));   /* the cache row of this position */
    memcpy(v_cache + (size_t)pos * kn, v, kn * sizeof(float));

    /* scores with scale 1.0 over the window, softmax in float, weighted V sum (:382-414) */
    const int n_pos = pos + 1;
    const int first = s->sliding_window > 0 ? (n_pos - s->sliding_window > 0 ? n_pos - s->sliding_window : 0) : 0;
    orc_attention_core(q, k_cache, v_cache, H, KV, hd, n_pos, first, (uint32_t)n_pos, ctx);
    orc_matvec(&L->o, ctx, attn_out);

    if (q_out) memcpy(q_out, q, qn * sizeof(float));
    if (k_out) memcpy(k_out, k, kn * sizeof(float));
    if (v_out) memcpy(v_out, v, kn * sizeof(float));
    free(normed);
    free(q);
    free(k);
    free(v);
    free(ctx);
    return 0;
}

/*
 * TEST INFRASTRUCTURE ONLY -- the CPU checker for the CUDA MoE path (see moe_oracle.h).
 *
 * Parity: every function below restates src/cpu_reference.cpp of the reference with the same
 * floating-point operation order, and tests/test_oracle.py proves it bit-identical against the
 * reference's own primitives compiled from its sources (oracle/_ref).
 */
#include "moe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "../turbo-winfare_b200/csrc/gtm_synth.h"

#define GROUP 64u

float orc_bf16(uint16_t bits) {
    uint32_t w = (uint32_t)bits << 16;
    float f;
    memcpy(&f, &w, 4);
    return f;
}

uint16_t orc_bf16_rne(float f) { return gtm_bf16_rne(f); }

/* gelu_pytorch_tanh, cpu_reference.cpp:34-38. */
float orc_gelu_tanh(float x) {
    const float k0 = 0.7978845608028654f;
    const float k1 = 0.044715f;
    return 0.5f * x * (1.0f + tanhf(k0 * (x + k1 * x * x * x)));
}

/* cpu_reference.cpp:43-52: double sum of squares, float rsqrt by 1/sqrtf. */
void orc_rms_norm(const float* x, const uint16_t* w, size_t n, float eps, float* out) {
    double acc = 0.0;
    for (size_t i = 0; i < n; ++i) acc += (double)x[i] * x[i];
    const float inv = 1.0f / sqrtf((float)(acc / (double)n) + eps);
    if (w) {
        for (size_t i = 0; i < n; ++i) out[i] = x[i] * inv * orc_bf16(w[i]);
    } else {
        for (size_t i = 0; i < n; ++i) out[i] = x[i] * inv;
    }
}

/* cpu_reference.cpp:55-106: per row, groups in order; inside a group the products are
 * accumulated one element at a time (4-bit: low nibble then high nibble of each byte,
 * and the group's x-sum by pairs), then acc += s*dot + b*sum. */
void orc_matvec(const orc_qt* t, const float* x, float* out) {
    const uint32_t groups = t->in_dim / GROUP;
    if (t->bits == 4) {
        const size_t row_bytes = t->in_dim / 2;
        for (uint32_t r = 0; r < t->rows; ++r) {
            const uint8_t* wrow = t->data + (size_t)r * row_bytes;
            const uint16_t* srow = t->scales + (size_t)r * groups;
            const uint16_t* brow = t->biases + (size_t)r * groups;
            float acc = 0.0f;
            for (uint32_t g = 0; g < groups; ++g) {
                const float s = orc_bf16(srow[g]);
                const float b = orc_bf16(brow[g]);
                const uint32_t base = g * GROUP;
                float dot = 0.0f, sum = 0.0f;
                for (uint32_t j = 0; j < GROUP; j += 2) {
                    const uint8_t byte = wrow[(base + j) / 2];
                    const float x0 = x[base + j];
                    const float x1 = x[base + j + 1];
                    dot += (float)(byte & 0x0F) * x0;
                    dot += (float)(byte >> 4) * x1;
                    sum += x0 + x1;
                }
                acc += s * dot + b * sum;
            }
            out[r] = acc;
        }
        return;
    }
    for (uint32_t r = 0; r < t->rows; ++r) {
        const uint8_t* wrow = t->data + (size_t)r * t->in_dim;
        const uint16_t* srow = t->scales + (size_t)r * groups;
        const uint16_t* brow = t->biases + (size_t)r * groups;
        float acc = 0.0f;
        for (uint32_t g = 0; g < groups; ++g) {
            const float s = orc_bf16(srow[g]);
            const float b = orc_bf16(brow[g]);
            const uint32_t base = g * GROUP;
            float dot = 0.0f, sum = 0.0f;
            for (uint32_t j = 0; j < GROUP; ++j) {
                const float xv = x[base + j];
                dot += (float)wrow[base + j] * xv;
                sum += xv;
            }
            acc += s * dot + b * sum;
        }
        out[r] = acc;
    }
}

/* Ordering used by the reference's partial_sort (cpu_reference.cpp:447-462): larger logit
 * first, equal logits by lower expert index. Returns nonzero when a ranks before b. */
static int ranks_before(const float* v, uint32_t a, uint32_t b) {
    if (v[a] != v[b]) return v[a] > v[b];
    return a < b;
}

/* Top-k selection, then softmax over the selected k only, times per_expert_scale
 * (cpu_reference.cpp:447-480). */
void orc_topk(const float* logits, uint32_t n, uint32_t k, const uint16_t* per_expert_scale,
              uint32_t* idx, float* w) {
    /* Selection by repeated extraction under the same strict weak order. */
    uint8_t* taken = (uint8_t*)calloc(n, 1);
    for (uint32_t i = 0; i < k; ++i) {
        uint32_t best = n;
        for (uint32_t e = 0; e < n; ++e) {
            if (taken[e]) continue;
            if (best == n || ranks_before(logits, e, best)) best = e;
        }
        taken[best] = 1;
        idx[i] = best;
    }
    free(taken);
    const float top = logits[idx[0]];
    float sum = 0.0f;
    for (uint32_t i = 0; i < k; ++i) {
        w[i] = expf(logits[idx[i]] - top);
        sum += w[i];
    }
    for (uint32_t i = 0; i < k; ++i) w[i] = w[i] / sum * orc_bf16(per_expert_scale[idx[i]]);
}

static orc_qt expert_qt(const orc_layer* L, const uint8_t* block, int role) {
    /* role 0 gate, 1 up, 2 down: sub-tensors 3*role + {0,1,2} */
    orc_qt t;
    t.data = block + L->sub_off[3 * role + 0];
    t.scales = (const uint16_t*)(block + L->sub_off[3 * role + 1]);
    t.biases = (const uint16_t*)(block + L->sub_off[3 * role + 2]);
    t.rows = role == 2 ? L->hidden : L->moe_inter;
    t.in_dim = role == 2 ? L->moe_inter : L->hidden;
    t.bits = 4;
    return t;
}

/* The MoE half of one decoder layer for one token, cpu_reference.cpp:422-520 with the block
 * input `hidden` standing in for the post-attention residual:
 *   views (:425-434), router (:436-480), shared expert (:482-494),
 *   routed experts (:496-510), layer tail (:512-520). */
int orc_moe_block(const orc_layer* L, const float* hidden_in, const float* logit_bias,
                  const float* route_logits, const orc_block_out* out) {
    const uint32_t D = L->hidden, E = L->num_experts, K = L->top_k;
    const float eps = L->eps;
    float* tmp = (float*)malloc(sizeof(float) * D);
    float* dense_x = (float*)malloc(sizeof(float) * D);
    float* routed_x = (float*)malloc(sizeof(float) * D);
    float* router_in = (float*)malloc(sizeof(float) * D);
    float* logits = (float*)malloc(sizeof(float) * E);
    uint32_t* top = (uint32_t*)malloc(sizeof(uint32_t) * K);
    float* wts = (float*)malloc(sizeof(float) * K);
    const uint32_t Fmax = L->ffn_inter > L->moe_inter ? L->ffn_inter : L->moe_inter;
    float* g = (float*)malloc(sizeof(float) * Fmax);
    float* u = (float*)malloc(sizeof(float) * Fmax);
    float* act = (float*)malloc(sizeof(float) * Fmax);
    float* outv = (float*)malloc(sizeof(float) * D);
    float* h2 = out->h2;
    float* h1 = out->h1;

    /* views: h = rmsnorm_no_scale(hidden); dense = h*w_pre; routed = h*w_pre2; router = h */
    orc_rms_norm(hidden_in, NULL, D, eps, tmp);
    for (uint32_t i = 0; i < D; ++i) {
        dense_x[i] = tmp[i] * orc_bf16(L->w_pre[i]);
        routed_x[i] = tmp[i] * orc_bf16(L->w_pre2[i]);
    }
    /* router input: router_x * bf16(router.scale) * (1/sqrt(D)), left to right */
    const float inv_sqrt_d = 1.0f / sqrtf((float)D);
    for (uint32_t i = 0; i < D; ++i) router_in[i] = tmp[i] * orc_bf16(L->router_scale[i]) * inv_sqrt_d;
    if (route_logits) {
        memcpy(logits, route_logits, sizeof(float) * E);
    } else {
        orc_matvec(&L->router, router_in, logits);
    }
    if (logit_bias) {
        for (uint32_t e = 0; e < E; ++e) logits[e] = logits[e] + logit_bias[e];
    }
    orc_topk(logits, E, K, L->per_expert_scale, top, wts);

    /* shared expert, no routing weight; post_feedforward_layernorm_1 -> h1 */
    orc_matvec(&L->sh_gate, dense_x, g);
    orc_matvec(&L->sh_up, dense_x, u);
    for (uint32_t i = 0; i < L->ffn_inter; ++i) act[i] = orc_gelu_tanh(g[i]) * u[i];
    orc_matvec(&L->sh_down, act, outv);
    orc_rms_norm(outv, L->w_pf1, D, eps, h1);

    /* routed experts in router order, h2 += w_k * out_k */
    for (uint32_t i = 0; i < D; ++i) h2[i] = 0.0f;
    for (uint32_t k = 0; k < K; ++k) {
        const uint8_t* block = L->experts + (uint64_t)top[k] * L->expert_stride;
        orc_qt eg = expert_qt(L, block, 0), eu = expert_qt(L, block, 1), ed = expert_qt(L, block, 2);
        orc_matvec(&eg, routed_x, g);
        orc_matvec(&eu, routed_x, u);
        for (uint32_t j = 0; j < L->moe_inter; ++j) act[j] = orc_gelu_tanh(g[j]) * u[j];
        orc_matvec(&ed, act, outv);
        const float wk = wts[k];
        for (uint32_t j = 0; j < D; ++j) h2[j] += wk * outv[j];
    }

    /* layer tail: t = rms(h2)*w_pf2 + h1; hidden = (hidden + rms(t)*w_pf) * layer_scalar */
    orc_rms_norm(h2, L->w_pf2, D, eps, tmp);
    for (uint32_t i = 0; i < D; ++i) tmp[i] += h1[i];
    orc_rms_norm(tmp, L->w_pf, D, eps, outv);
    const float ls = orc_bf16(L->layer_scalar);
    for (uint32_t i = 0; i < D; ++i) out->hidden_out[i] = (hidden_in[i] + outv[i]) * ls;

    if (out->logits) memcpy(out->logits, logits, sizeof(float) * E);
    if (out->top_idx) memcpy(out->top_idx, top, sizeof(uint32_t) * K);
    if (out->top_w) memcpy(out->top_w, wts, sizeof(float) * K);
    free(tmp); free(dense_x); free(routed_x); free(router_in); free(logits); free(top); free(wts);
    free(g); free(u); free(act); free(outv);
    return 0;
}

/* ---- synthetic model ------------------------------------------------------------------ */

static void fill_quant(uint64_t seed, uint32_t layer, uint32_t kind_w, uint32_t kind_s, uint32_t expert,
                       uint32_t rows, uint32_t in_dim, int bits, uint8_t* w, uint8_t* s, uint8_t* b) {
    const uint64_t words = (uint64_t)rows * in_dim * bits / 32;
    const uint64_t sw = gtm_stream(seed, layer, kind_w, expert);
    uint32_t* wp = (uint32_t*)w;
    for (uint64_t i = 0; i < words; ++i) wp[i] = gtm_qword(sw, i);
    const uint64_t nsc = (uint64_t)rows * (in_dim / GROUP);
    const uint64_t ss = gtm_stream(seed, layer, kind_s, expert);
    uint16_t* sp = (uint16_t*)s;
    uint16_t* bp = (uint16_t*)b;
    const float zp = bits == 4 ? 8.0f : 128.0f;
    for (uint64_t i = 0; i < nsc; ++i) {
        sp[i] = gtm_scale_bits(ss, i);
        bp[i] = gtm_bias_bits(sp[i], zp);
    }
}

void orc_synth_resident(uint64_t seed, uint32_t layer, uint32_t hidden, uint32_t ffn,
                        uint32_t experts, uint8_t* image) {
    GtmResidentLayout R = gtm_resident_layout(hidden, ffn, experts);
    memset(image, 0, R.total);
    uint8_t* o = image;
    fill_quant(seed, layer, GTM_K_ROUTER_W, GTM_K_ROUTER_S, 0, experts, hidden, 8,
               o + R.offset[GTM_R_ROUTER_W], o + R.offset[GTM_R_ROUTER_S], o + R.offset[GTM_R_ROUTER_B]);
    fill_quant(seed, layer, GTM_K_SH_GATE_W, GTM_K_SH_GATE_S, 0, ffn, hidden, 4,
               o + R.offset[GTM_R_SH_GATE_W], o + R.offset[GTM_R_SH_GATE_S], o + R.offset[GTM_R_SH_GATE_B]);
    fill_quant(seed, layer, GTM_K_SH_UP_W, GTM_K_SH_UP_S, 0, ffn, hidden, 4,
               o + R.offset[GTM_R_SH_UP_W], o + R.offset[GTM_R_SH_UP_S], o + R.offset[GTM_R_SH_UP_B]);
    fill_quant(seed, layer, GTM_K_SH_DOWN_W, GTM_K_SH_DOWN_S, 0, hidden, ffn, 4,
               o + R.offset[GTM_R_SH_DOWN_W], o + R.offset[GTM_R_SH_DOWN_S], o + R.offset[GTM_R_SH_DOWN_B]);
    const uint32_t norm_kinds[6] = {GTM_K_ROUTER_SCALE, GTM_K_W_PRE, GTM_K_W_PRE2, GTM_K_W_PF1, GTM_K_W_PF2, GTM_K_W_PF};
    const int norm_regions[6] = {GTM_R_ROUTER_SCALE, GTM_R_W_PRE, GTM_R_W_PRE2, GTM_R_W_PF1, GTM_R_W_PF2, GTM_R_W_PF};
    for (int k = 0; k < 6; ++k) {
        const uint64_t st = gtm_stream(seed, layer, norm_kinds[k], 0);
        uint16_t* p = (uint16_t*)(o + R.offset[norm_regions[k]]);
        for (uint32_t i = 0; i < hidden; ++i) p[i] = gtm_norm_weight_bits(st, i);
    }
    {
        const uint64_t st = gtm_stream(seed, layer, GTM_K_PER_EXPERT_SCALE, 0);
        uint16_t* p = (uint16_t*)(o + R.offset[GTM_R_PER_EXPERT_SCALE]);
        for (uint32_t e = 0; e < experts; ++e) p[e] = gtm_per_expert_scale_bits(st, e);
    }
    *(uint16_t*)(o + R.offset[GTM_R_LAYER_SCALAR]) = GTM_LAYER_SCALAR_BITS;
}

void orc_synth_expert(uint64_t seed, uint32_t layer, uint32_t expert, uint32_t hidden,
                      uint32_t inter, uint8_t* block) {
    GtmExpertBlockLayout B = gtm_expert_block_layout(hidden, inter);
    memset(block + B.used, 0, B.stride - B.used);
    fill_quant(seed, layer, GTM_K_EXP_GATE_W, GTM_K_EXP_GATE_S, expert, inter, hidden, 4,
               block + B.offset[0], block + B.offset[1], block + B.offset[2]);
    fill_quant(seed, layer, GTM_K_EXP_UP_W, GTM_K_EXP_UP_S, expert, inter, hidden, 4,
               block + B.offset[3], block + B.offset[4], block + B.offset[5]);
    fill_quant(seed, layer, GTM_K_EXP_DOWN_W, GTM_K_EXP_DOWN_S, expert, hidden, inter, 4,
               block + B.offset[6], block + B.offset[7], block + B.offset[8]);
}

void orc_synth_x(uint64_t seed, uint32_t token, uint32_t hidden, float* x) {
    const uint64_t st = gtm_stream(seed, 0xFFFFu, GTM_K_X, token);
    for (uint32_t i = 0; i < hidden; ++i) x[i] = gtm_normal(st, i);
}

void orc_layer_view(orc_layer* L, const uint8_t* resident, const uint8_t* experts,
                    uint32_t hidden, uint32_t moe_inter, uint32_t ffn, uint32_t experts_n,
                    uint32_t top_k, float eps) {
    GtmResidentLayout R = gtm_resident_layout(hidden, ffn, experts_n);
    GtmExpertBlockLayout B = gtm_expert_block_layout(hidden, moe_inter);
    const uint8_t* o = resident;
    memset(L, 0, sizeof(*L));
    L->hidden = hidden; L->moe_inter = moe_inter; L->ffn_inter = ffn;
    L->num_experts = experts_n; L->top_k = top_k; L->eps = eps;
    L->router.data = o + R.offset[GTM_R_ROUTER_W];
    L->router.scales = (const uint16_t*)(o + R.offset[GTM_R_ROUTER_S]);
    L->router.biases = (const uint16_t*)(o + R.offset[GTM_R_ROUTER_B]);
    L->router.rows = experts_n; L->router.in_dim = hidden; L->router.bits = 8;
    L->router_scale = (const uint16_t*)(o + R.offset[GTM_R_ROUTER_SCALE]);
    L->per_expert_scale = (const uint16_t*)(o + R.offset[GTM_R_PER_EXPERT_SCALE]);
    const int qw[3] = {GTM_R_SH_GATE_W, GTM_R_SH_UP_W, GTM_R_SH_DOWN_W};
    orc_qt* qs[3] = {&L->sh_gate, &L->sh_up, &L->sh_down};
    for (int i = 0; i < 3; ++i) {
        qs[i]->data = o + R.offset[qw[i]];
        qs[i]->scales = (const uint16_t*)(o + R.offset[qw[i] + 1]);
        qs[i]->biases = (const uint16_t*)(o + R.offset[qw[i] + 2]);
        qs[i]->rows = i == 2 ? hidden : ffn;
        qs[i]->in_dim = i == 2 ? ffn : hidden;
        qs[i]->bits = 4;
    }
    L->w_pre = (const uint16_t*)(o + R.offset[GTM_R_W_PRE]);
    L->w_pre2 = (const uint16_t*)(o + R.offset[GTM_R_W_PRE2]);
    L->w_pf1 = (const uint16_t*)(o + R.offset[GTM_R_W_PF1]);
    L->w_pf2 = (const uint16_t*)(o + R.offset[GTM_R_W_PF2]);
    L->w_pf = (const uint16_t*)(o + R.offset[GTM_R_W_PF]);
    L->layer_scalar = *(const uint16_t*)(o + R.offset[GTM_R_LAYER_SCALAR]);
    L->experts = experts;
    L->expert_stride = B.stride;
    for (int i = 0; i < 9; ++i) L->sub_off[i] = B.offset[i];
}

struct orc_synth_layer {
    uint64_t seed;
    uint32_t layer, hidden, moe_inter, ffn, experts, top_k;
    float eps;
    uint8_t* resident;
    uint8_t* expert_mem;      /* experts * stride bytes, filled lazily */
    uint8_t* have;            /* [experts] */
    orc_layer view;
};

orc_synth_layer* orc_synth_layer_create(uint64_t seed, uint32_t layer, uint32_t hidden,
                                        uint32_t moe_inter, uint32_t ffn, uint32_t experts,
                                        uint32_t top_k, float eps) {
    orc_synth_layer* s = (orc_synth_layer*)calloc(1, sizeof(*s));
    if (!s) return NULL;
    s->seed = seed; s->layer = layer; s->hidden = hidden; s->moe_inter = moe_inter;
    s->ffn = ffn; s->experts = experts; s->top_k = top_k; s->eps = eps;
    GtmResidentLayout R = gtm_resident_layout(hidden, ffn, experts);
    GtmExpertBlockLayout B = gtm_expert_block_layout(hidden, moe_inter);
    s->resident = (uint8_t*)malloc(R.total);
    s->expert_mem = (uint8_t*)malloc(B.stride * experts);
    s->have = (uint8_t*)calloc(experts, 1);
    if (!s->resident || !s->expert_mem || !s->have) { orc_synth_layer_destroy(s); return NULL; }
    orc_synth_resident(seed, layer, hidden, ffn, experts, s->resident);
    orc_layer_view(&s->view, s->resident, s->expert_mem, hidden, moe_inter, ffn, experts, top_k, eps);
    return s;
}

void orc_synth_layer_destroy(orc_synth_layer* s) {
    if (!s) return;
    free(s->resident); free(s->expert_mem); free(s->have); free(s);
}

const orc_layer* orc_synth_layer_view(const orc_synth_layer* s) { return &s->view; }

void orc_synth_layer_ensure(orc_synth_layer* s, const uint32_t* experts, uint32_t n) {
    GtmExpertBlockLayout B = gtm_expert_block_layout(s->hidden, s->moe_inter);
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t e = experts[i];
        if (e >= s->experts || s->have[e]) continue;
        orc_synth_expert(s->seed, s->layer, e, s->hidden, s->moe_inter, s->expert_mem + (uint64_t)e * B.stride);
        s->have[e] = 1;
    }
}

int orc_synth_layer_block(orc_synth_layer* s, const float* hidden_in, const float* logit_bias,
                          const float* route_logits, const orc_block_out* out) {
    orc_synth_layer_route(s, hidden_in, logit_bias, route_logits, NULL);
    return orc_moe_block(&s->view, hidden_in, logit_bias, route_logits, out);
}

/* Views, router and top-k only (no expert work); materialises the selected experts. */
void orc_synth_layer_route(orc_synth_layer* s, const float* hidden_in, const float* logit_bias,
                           const float* route_logits, uint32_t* idx_out) {
    const uint32_t D = s->hidden, E = s->experts, K = s->top_k;
    float* tmp = (float*)malloc(sizeof(float) * D);
    float* rin = (float*)malloc(sizeof(float) * D);
    float* logits = (float*)malloc(sizeof(float) * E);
    uint32_t* idx = (uint32_t*)malloc(sizeof(uint32_t) * K);
    float* w = (float*)malloc(sizeof(float) * K);
    orc_rms_norm(hidden_in, NULL, D, s->eps, tmp);
    const float inv_sqrt_d = 1.0f / sqrtf((float)D);
    for (uint32_t i = 0; i < D; ++i) rin[i] = tmp[i] * orc_bf16(s->view.router_scale[i]) * inv_sqrt_d;
    if (route_logits) memcpy(logits, route_logits, sizeof(float) * E);
    else orc_matvec(&s->view.router, rin, logits);
    if (logit_bias) for (uint32_t e = 0; e < E; ++e) logits[e] = logits[e] + logit_bias[e];
    orc_topk(logits, E, K, s->view.per_expert_scale, idx, w);
    orc_synth_layer_ensure(s, idx, K);
    if (idx_out) memcpy(idx_out, idx, sizeof(uint32_t) * K);
    free(tmp); free(rin); free(logits); free(idx); free(w);
}

int orc_synth_stack(orc_synth_layer** layers, uint32_t n, const float* hidden_in,
                    float* hidden_out, float* hidden_per_layer, uint32_t* idx_per_layer,
                    float* w_per_layer) {
    if (n == 0) return -1;
    const uint32_t D = layers[0]->hidden, K = layers[0]->top_k;
    float* cur = (float*)malloc(sizeof(float) * D);
    float* nxt = (float*)malloc(sizeof(float) * D);
    float* h1 = (float*)malloc(sizeof(float) * D);
    float* h2 = (float*)malloc(sizeof(float) * D);
    memcpy(cur, hidden_in, sizeof(float) * D);
    for (uint32_t l = 0; l < n; ++l) {
        orc_block_out o;
        o.hidden_out = nxt; o.h1 = h1; o.h2 = h2; o.logits = NULL;
        o.top_idx = idx_per_layer ? idx_per_layer + (size_t)l * K : NULL;
        o.top_w = w_per_layer ? w_per_layer + (size_t)l * K : NULL;
        orc_synth_layer_block(layers[l], cur, NULL, NULL, &o);
        if (l + 1 < n) orc_rms_norm(nxt, NULL, D, layers[l]->eps, cur);
        else memcpy(cur, nxt, sizeof(float) * D);
        if (hidden_per_layer) memcpy(hidden_per_layer + (size_t)l * D, cur, sizeof(float) * D);
    }
    memcpy(hidden_out, cur, sizeof(float) * D);
    free(cur); free(nxt); free(h1); free(h2);
    return 0;
}

/*
 * TEST INFRASTRUCTURE ONLY. Builds the reference's own scalar FP32 primitives into
 * oracle/_ref/libgtref.so so tests can pin the restated oracle against them and bench.py can
 * time the reference's CPU arithmetic as the CPU baseline.
 *
 * The reference source is compiled where it lies (the Makefile passes its path); nothing of
 * it is copied here. Its numeric helpers are file-static (src/cpu_reference.cpp:21-106), so
 * this translation unit includes that file and exposes the helpers through a C ABI. The MoE
 * block below composes those helpers in the order of CpuReference::forward
 * (src/cpu_reference.cpp:422-520); CpuReference::forward itself also runs attention and the
 * LM head, so the block is reassembled from its parts.
 */
#include GTREF_CPU_REFERENCE_CPP
#include "gturbo/sampling.hpp"

#include <cstdint>
#include <cstring>
#include <fstream>
#include <numeric>
#include <sstream>
#include <vector>

using gturbo::QuantTensor;

namespace {
QuantTensor view(const uint8_t* data, const uint16_t* s, const uint16_t* b, uint32_t rows,
                 uint32_t in_dim, int bits) {
    QuantTensor t;
    t.data = data;
    t.scales = s;
    t.biases = b;
    t.rows = rows;
    t.in_dim = in_dim;
    t.groups = in_dim / 64;
    t.bits = bits;
    t.quantized = true;
    return t;
}
}  // namespace

extern "C" {

struct gtref_qt {
    const uint8_t* data;
    const uint16_t* scales;
    const uint16_t* biases;
    uint32_t rows, in_dim;
    int bits;
};

/* Mirrors orc_layer in oracle/moe_oracle.h field for field. */
struct gtref_layer {
    uint32_t hidden, moe_inter, ffn_inter, num_experts, top_k;
    float eps;
    gtref_qt router;
    const uint16_t* router_scale;
    const uint16_t* per_expert_scale;
    gtref_qt sh_gate, sh_up, sh_down;
    const uint16_t *w_pre, *w_pre2, *w_pf1, *w_pf2, *w_pf;
    uint16_t layer_scalar;
    const uint8_t* experts;
    uint64_t expert_stride;
    uint64_t sub_off[9];
};

struct gtref_block_out {
    float* hidden_out;
    float* h1;
    float* h2;
    float* logits;
    uint32_t* top_idx;
    float* top_w;
};

__attribute__((visibility("default"))) float gtref_bf16(uint16_t bits) { return gturbo::bf16(bits); }
__attribute__((visibility("default"))) float gtref_gelu_tanh(float x) { return gturbo::gelu_tanh(x); }
__attribute__((visibility("default"))) void gtref_rms_norm(const float* x, const uint16_t* w, size_t n,
                                                           float eps, float* out) {
    gturbo::rms_norm(x, w, n, eps, out);
}
__attribute__((visibility("default"))) void gtref_matvec(const gtref_qt* t, const float* x, float* out) {
    gturbo::matvec(view(t->data, t->scales, t->biases, t->rows, t->in_dim, t->bits), x, out);
}

/* The MoE block of one token using only the reference's helpers, in its forward() order. */
__attribute__((visibility("default"))) int gtref_moe_block(const gtref_layer* L, const float* hidden_in,
                                                           const float* logit_bias, const float* route_logits,
                                                           const gtref_block_out* out) {
    const uint32_t D = L->hidden, E = L->num_experts, K = L->top_k;
    const float eps = L->eps;
    std::vector<float> tmp(D), dense_x(D), routed_x(D), router_in(D);
    gturbo::rms_norm(hidden_in, nullptr, D, eps, tmp.data());
    for (uint32_t i = 0; i < D; ++i) {
        dense_x[i] = tmp[i] * gturbo::bf16(L->w_pre[i]);
        routed_x[i] = tmp[i] * gturbo::bf16(L->w_pre2[i]);
    }
    const float inv_sqrt_d = 1.0f / std::sqrt(static_cast<float>(D));
    for (uint32_t i = 0; i < D; ++i) router_in[i] = tmp[i] * gturbo::bf16(L->router_scale[i]) * inv_sqrt_d;

    std::vector<float> logits(E);
    if (route_logits) {
        std::copy(route_logits, route_logits + E, logits.begin());
    } else {
        const gtref_qt& r = L->router;
        gturbo::matvec(view(r.data, r.scales, r.biases, r.rows, r.in_dim, r.bits), router_in.data(), logits.data());
    }
    if (logit_bias) for (uint32_t e = 0; e < E; ++e) logits[e] = logits[e] + logit_bias[e];

    std::vector<int> order(E);
    std::iota(order.begin(), order.end(), 0);
    std::partial_sort(order.begin(), order.begin() + K, order.end(), [&](int a, int b) {
        if (logits[a] != logits[b]) return logits[a] > logits[b];
        return a < b;
    });
    std::vector<float> w(K);
    {
        const float best = logits[order[0]];
        float sum = 0.0f;
        for (uint32_t i = 0; i < K; ++i) { w[i] = std::exp(logits[order[i]] - best); sum += w[i]; }
        for (uint32_t i = 0; i < K; ++i) w[i] = w[i] / sum * gturbo::bf16(L->per_expert_scale[order[i]]);
    }

    const uint32_t F = std::max(L->ffn_inter, L->moe_inter);
    std::vector<float> g(F), u(F), act(F), o(D);
    auto qt = [](const gtref_qt& q) { return view(q.data, q.scales, q.biases, q.rows, q.in_dim, q.bits); };
    gturbo::matvec(qt(L->sh_gate), dense_x.data(), g.data());
    gturbo::matvec(qt(L->sh_up), dense_x.data(), u.data());
    for (uint32_t i = 0; i < L->ffn_inter; ++i) act[i] = gturbo::gelu_tanh(g[i]) * u[i];
    gturbo::matvec(qt(L->sh_down), act.data(), o.data());
    gturbo::rms_norm(o.data(), L->w_pf1, D, eps, out->h1);

    float* h2 = out->h2;
    std::fill(h2, h2 + D, 0.0f);
    for (uint32_t k = 0; k < K; ++k) {
        const uint8_t* blk = L->experts + static_cast<uint64_t>(order[k]) * L->expert_stride;
        auto ex = [&](int role) {
            const bool down = role == 2;
            return view(blk + L->sub_off[3 * role], reinterpret_cast<const uint16_t*>(blk + L->sub_off[3 * role + 1]),
                        reinterpret_cast<const uint16_t*>(blk + L->sub_off[3 * role + 2]),
                        down ? D : L->moe_inter, down ? L->moe_inter : D, 4);
        };
        gturbo::matvec(ex(0), routed_x.data(), g.data());
        gturbo::matvec(ex(1), routed_x.data(), u.data());
        for (uint32_t j = 0; j < L->moe_inter; ++j) act[j] = gturbo::gelu_tanh(g[j]) * u[j];
        gturbo::matvec(ex(2), act.data(), o.data());
        const float wk = w[k];
        for (uint32_t j = 0; j < D; ++j) h2[j] += wk * o[j];
    }

    gturbo::rms_norm(h2, L->w_pf2, D, eps, tmp.data());
    for (uint32_t i = 0; i < D; ++i) tmp[i] += out->h1[i];
    gturbo::rms_norm(tmp.data(), L->w_pf, D, eps, o.data());
    const float ls = gturbo::bf16(L->layer_scalar);
    for (uint32_t i = 0; i < D; ++i) out->hidden_out[i] = (hidden_in[i] + o[i]) * ls;

    if (out->logits) std::copy(logits.begin(), logits.end(), out->logits);
    for (uint32_t k = 0; k < K; ++k) {
        if (out->top_idx) out->top_idx[k] = static_cast<uint32_t>(order[k]);
        if (out->top_w) out->top_w[k] = w[k];
    }
    return 0;
}

/* ---- embedding lookup and one attention step, from the reference's own helpers ---- */

/* Mirrors orc_attn_shape / orc_attn_layer in oracle/attn_oracle.h field for field. */
struct gtref_attn_shape {
    uint32_t hidden, num_heads, head_dim, kv_heads, rotated_pairs;
    float theta;
    int32_t sliding_window, k_eq_v;
    float eps;
};
struct gtref_attn_layer {
    gtref_qt q, k, v, o;
    const uint16_t *input_norm, *q_norm, *k_norm;
};

static QuantTensor qt_of(const gtref_qt& t) { return view(t.data, t.scales, t.biases, t.rows, t.in_dim, t.bits); }

/* cpu_reference.cpp:322-330: dequant_row, then * sqrt(hidden). */
void gtref_embed(const gtref_qt* embed, uint32_t token, float* out) {
    const QuantTensor t = qt_of(*embed);
    gturbo::dequant_row(t, token, out);
    const float embed_scale = std::sqrt(static_cast<float>(t.in_dim));
    for (uint32_t i = 0; i < t.in_dim; ++i) out[i] *= embed_scale;
}

void gtref_rope_neox(float* vec, uint32_t head_dim, uint32_t rotated_pairs, float position, float theta) {
    gturbo::rope_neox(vec, head_dim, rotated_pairs, position, theta);
}

/* The attention section of CpuReference::forward (cpu_reference.cpp:345-417) for one layer,
 * with the layer's KV rows in caller memory instead of LayerKV vectors. */
int gtref_attention_step(const gtref_attn_shape* s, const gtref_attn_layer* L, int pos, const float* hidden,
                         float* k_cache, float* v_cache, float* attn_out, float* q_out, float* k_out, float* v_out) {
    const uint32_t D = s->hidden, head_dim = s->head_dim, q_heads = s->num_heads, kv_heads = s->kv_heads;
    const float eps = s->eps;
    std::vector<float> normed(D);
    gturbo::rms_norm(hidden, L->input_norm, D, eps, normed.data());
    std::vector<float> q(q_heads * head_dim), k(kv_heads * head_dim), v(kv_heads * head_dim);
    gturbo::matvec(qt_of(L->q), normed.data(), q.data());
    gturbo::matvec(qt_of(L->k), normed.data(), k.data());
    if (s->k_eq_v) {
        v = k;
    } else {
        gturbo::matvec(qt_of(L->v), normed.data(), v.data());
    }
    std::vector<float> scratch(head_dim);
    for (uint32_t h = 0; h < q_heads; ++h) {
        gturbo::rms_norm(q.data() + h * head_dim, L->q_norm, head_dim, eps, scratch.data());
        std::copy(scratch.begin(), scratch.end(), q.begin() + h * head_dim);
        gturbo::rope_neox(q.data() + h * head_dim, head_dim, s->rotated_pairs, static_cast<float>(pos), s->theta);
    }
    for (uint32_t h = 0; h < kv_heads; ++h) {
        gturbo::rms_norm(k.data() + h * head_dim, L->k_norm, head_dim, eps, scratch.data());
        std::copy(scratch.begin(), scratch.end(), k.begin() + h * head_dim);
        gturbo::rope_neox(k.data() + h * head_dim, head_dim, s->rotated_pairs, static_cast<float>(pos), s->theta);
        gturbo::rms_norm(v.data() + h * head_dim, nullptr, head_dim, eps, scratch.data());
        std::copy(scratch.begin(), scratch.end(), v.begin() + h * head_dim);
    }
    const size_t row = static_cast<size_t>(kv_heads) * head_dim;
    std::copy(k.begin(), k.end(), k_cache + static_cast<size_t>(pos) * row);
    std::copy(v.begin(), v.end(), v_cache + static_cast<size_t>(pos) * row);

    const uint32_t gqa = q_heads / kv_heads;
    const int n_pos = pos + 1;
    const int first = s->sliding_window <= 0 ? 0 : std::max(0, n_pos - s->sliding_window);
    std::vector<float> ctx(q_heads * head_dim, 0.0f);
    std::vector<float> scores(static_cast<size_t>(n_pos));
    for (uint32_t h = 0; h < q_heads; ++h) {
        const uint32_t kvh = h / gqa;
        const float* qh = q.data() + h * head_dim;
        float best = -1e30f;
        for (int t = first; t < n_pos; ++t) {
            const float* kt = k_cache + static_cast<size_t>(t) * row + kvh * head_dim;
            float dot = 0.0f;
            for (uint32_t d = 0; d < head_dim; ++d) dot += qh[d] * kt[d];
            scores[static_cast<size_t>(t)] = dot;
            best = std::max(best, dot);
        }
        float sum = 0.0f;
        for (int t = first; t < n_pos; ++t) {
            float e = std::exp(scores[static_cast<size_t>(t)] - best);
            scores[static_cast<size_t>(t)] = e;
            sum += e;
        }
        float* out = ctx.data() + h * head_dim;
        for (int t = first; t < n_pos; ++t) {
            const float wgt = scores[static_cast<size_t>(t)] / sum;
            const float* vt = v_cache + static_cast<size_t>(t) * row + kvh * head_dim;
            for (uint32_t d = 0; d < head_dim; ++d) out[d] += wgt * vt[d];
        }
    }
    gturbo::matvec(qt_of(L->o), ctx.data(), attn_out);
    if (q_out) std::copy(q.begin(), q.end(), q_out);
    if (k_out) std::copy(k.begin(), k.end(), k_out);
    if (v_out) std::copy(v.begin(), v.end(), v_out);
    return 0;
}

/* ---- token sampling: the reference's src/sampling.cpp, linked into this library ---- */

/* Mirrors orc_sampling in oracle/sampling_oracle.h field for field. */
struct gtref_sampling {
    float temperature, top_p;
    int32_t top_k;
    float repetition_penalty;
    int32_t has_seed;
    uint32_t pad_;
    uint64_t seed;
};

static gturbo::SamplingParams params_of(const gtref_sampling* p) {
    gturbo::SamplingParams q;
    q.temperature = p->temperature;
    q.top_p = p->top_p;
    q.top_k = p->top_k;
    q.repetition_penalty = p->repetition_penalty;
    q.has_seed = p->has_seed != 0;
    q.seed = p->seed;
    return q;
}

/* 0 = accepted, 1 = GTurboFormatError. */
int gtref_validate_sampling(const gtref_sampling* p) {
    try {
        gturbo::validate_sampling(params_of(p));
        return 0;
    } catch (const gturbo::GTurboFormatError&) {
        return 1;
    }
}

uint64_t gtref_splitmix64(uint64_t x) { return gturbo::splitmix64(x); }

uint64_t gtref_seed_for(const gtref_sampling* p, int position) { return gturbo::seed_for(params_of(p), position); }

void gtref_apply_repetition_penalty(float* logits, uint32_t vocab, const uint32_t* history, size_t n_history,
                                    float penalty, float softcap) {
    const std::vector<uint32_t> h(history, history + n_history);
    gturbo::apply_repetition_penalty(logits, vocab, h, penalty, softcap);
}

/* 0 = a token in *token, 1 = GTurboFormatError (empty vocabulary, degenerate distribution). */
int gtref_sample_token(const float* logits, uint32_t vocab, const gtref_sampling* p, uint64_t seed, uint32_t* token) {
    try {
        *token = gturbo::sample_token(logits, vocab, params_of(p), seed);
        return 0;
    } catch (const gturbo::GTurboFormatError&) {
        return 1;
    }
}

/* ---- the whole model: CpuReference::load + generate on a bundle directory ---- */

static std::string read_all(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw gturbo::GTurboFormatError("cannot open " + path);
    std::ostringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

/* The reference's public generation path (cpu_reference.cpp:167-219 load, :544-595 generate)
 * with greedy decoding (temperature 0) or, given `sampling`, the reference's sampling (softcapped
 * logits, repetition penalty, sample_token with seed_for(position)): the prompt is prefilled
 * token by token, then up to
 * max_tokens tokens are produced, stopping before any stop token. With dump_dir set, the reference
 * also writes the first prompt token's stages there (embed, layerN_hidden, final_norm, logits as
 * raw .f32 files, cpu_reference.cpp:142-150). 0, or 1 with the exception's message in err. */
int gtref_generate(const char* dir, const uint32_t* prompt, uint32_t n_prompt, int max_tokens, const char* dump_dir,
                   const gtref_sampling* sampling, uint32_t* out, uint32_t* n_out, char* err, size_t err_len) {
    try {
        const std::string d(dir);
        auto manifest = gturbo::GTurboManifestV1::from_json_string(read_all(d + "/manifest.json"));
        auto layout = gturbo::PackedExpertsLayoutV1::from_json_string(read_all(d + "/packed_experts/layout.json"));
        gturbo::CpuReference ref(manifest, layout, d);
        ref.load();
        gturbo::CpuGenerationOptions opts;
        opts.max_tokens = max_tokens;
        opts.temperature = 0.0f;
        if (sampling) {   // CpuGenerationOptions carries the seed as "0 = none"
            opts.temperature = sampling->temperature;
            opts.top_p = sampling->top_p;
            opts.top_k = sampling->top_k;
            opts.repetition_penalty = sampling->repetition_penalty;
            opts.seed = sampling->has_seed ? sampling->seed : 0;
        }
        if (dump_dir) opts.dump_dir = dump_dir;   // per-stage tensors of the first prompt token
        const std::vector<uint32_t> tokens =
            ref.generate(std::vector<uint32_t>(prompt, prompt + n_prompt), opts);
        std::copy(tokens.begin(), tokens.end(), out);
        *n_out = static_cast<uint32_t>(tokens.size());
        return 0;
    } catch (const std::exception& e) {
        if (err && err_len) {
            std::strncpy(err, e.what(), err_len - 1);
            err[err_len - 1] = '\0';
        }
        return 1;
    }
}

}  // extern "C"

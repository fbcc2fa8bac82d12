// TEST INFRASTRUCTURE ONLY. Regenerates the known-answer fixtures of the reference's GPU
// kernel test (tests/test_gpu_kernels.cpp) for the MoE hot path: the same std::mt19937(12345)
// stream consumed in the same order with the same distributions (:226-227 and QuantMatrix::build
// :118-147), and the expected outputs computed with the test's own inline CPU formulas.
//
// Output: a flat record file, read by tests/golden/make_golden.py into tests/golden/kat.npz.
// Record: u32 name_len, name bytes, u32 dtype (0 f32, 1 u16, 2 u8, 3 u32), u64 count, payload.
//
// Cases, in the test's order (the ones not on the MoE path only advance the generator):
//   GemvInt4 96x2816 (:241-266)       EmbedLookup 64x2816, row 37 (:268-292)
//   RMSNormK (:294-336)               GemvInt8 128x2816 (:338-361)
//   GeGLU n=2112 (:363-387)           Softcap n=4096 (:389-411)
//   MulBF16 n=2816 (:413-441)         ScaleAccum 8x2816 (:443-482)
//   RouterTopK 128, K=8, tie 11/70 (:484-542)
//   PostAttn D=2816 (:544-601)        LayerTail D=2816 (:603-647)
//   QKVEpilogue 2x512, 64 pairs (:649-692)
//   Attention GQA 16/8, window 128, n_pos 300 (:694-741)
//   LMHeadGreedy 4096x2816 (:743-802, draws only)
//   Attention across the ring wrap, capacity 128 (:804-858)
// The attention cases' K/V caches (2.4 MB and 1 MB) are not stored: the record holds the
// generator state at the start of the case (624 words and the position, the engine's own
// textual state), from which the inputs are drawn again.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <sstream>
#include <string>
#include <vector>

namespace {
constexpr uint32_t kGroup = 64;

float f_of_bf16(uint16_t bits) {
    uint32_t w = static_cast<uint32_t>(bits) << 16;
    float f;
    std::memcpy(&f, &w, 4);
    return f;
}
uint16_t bf16_of_f(float f) {  // round to nearest even, as the test's bf16_bits()
    uint32_t w;
    std::memcpy(&w, &f, 4);
    return static_cast<uint16_t>((w + 0x7FFFu + ((w >> 16) & 1u)) >> 16);
}

FILE* g_out = nullptr;
template <class T>
void put(const std::string& name, const std::vector<T>& v, uint32_t dtype) {
    uint32_t n = static_cast<uint32_t>(name.size());
    uint64_t count = v.size();
    std::fwrite(&n, 4, 1, g_out);
    std::fwrite(name.data(), 1, n, g_out);
    std::fwrite(&dtype, 4, 1, g_out);
    std::fwrite(&count, 8, 1, g_out);
    std::fwrite(v.data(), sizeof(T), v.size(), g_out);
}
void put_f(const std::string& n, const std::vector<float>& v) { put(n, v, 0); }
void put_h(const std::string& n, const std::vector<uint16_t>& v) { put(n, v, 1); }
void put_b(const std::string& n, const std::vector<uint8_t>& v) { put(n, v, 2); }
void put_u(const std::string& n, const std::vector<uint32_t>& v) { put(n, v, 3); }

// Affine-quantised matrix drawn like the test's QuantMatrix::build: all (scale, bias) pairs
// first, interleaved, then every element row by row.
struct Quant {
    std::vector<uint8_t> packed;
    std::vector<uint16_t> scales, biases;
    uint32_t rows = 0, in_dim = 0;
    int bits = 4;
    void draw(uint32_t r, uint32_t n, int b, std::mt19937& rng) {
        rows = r; in_dim = n; bits = b;
        const uint32_t groups = n / kGroup;
        packed.assign(b == 4 ? size_t(r) * n / 2 : size_t(r) * n, 0);
        scales.resize(size_t(r) * groups);
        biases.resize(size_t(r) * groups);
        std::uniform_int_distribution<int> q(0, b == 4 ? 15 : 255);
        std::uniform_real_distribution<float> sf(0.001f, 0.05f);
        std::uniform_real_distribution<float> bf(-0.4f, 0.4f);
        for (size_t i = 0; i < scales.size(); ++i) {
            scales[i] = bf16_of_f(sf(rng));
            biases[i] = bf16_of_f(bf(rng));
        }
        for (uint32_t row = 0; row < r; ++row) {
            for (uint32_t c = 0; c < n; ++c) {
                const uint32_t v = static_cast<uint32_t>(q(rng));
                if (b == 4) {
                    const size_t idx = size_t(row) * (n / 2) + c / 2;
                    packed[idx] = (c & 1u) == 0u ? uint8_t((packed[idx] & 0xF0) | v)
                                                 : uint8_t((packed[idx] & 0x0F) | (v << 4));
                } else {
                    packed[size_t(row) * n + c] = uint8_t(v);
                }
            }
        }
    }
    uint32_t q_at(uint32_t row, uint32_t c) const {
        if (bits == 4) {
            const uint8_t byte = packed[size_t(row) * (in_dim / 2) + c / 2];
            return (c & 1u) == 0u ? (byte & 0x0Fu) : (byte >> 4);
        }
        return packed[size_t(row) * in_dim + c];
    }
    // The test's expected GEMV: element-wise dequantised weights, one running sum per row.
    std::vector<float> expect(const std::vector<float>& x) const {
        const uint32_t groups = in_dim / kGroup;
        std::vector<float> out(rows);
        for (uint32_t row = 0; row < rows; ++row) {
            float acc = 0.0f;
            for (uint32_t g = 0; g < groups; ++g) {
                const float s = f_of_bf16(scales[size_t(row) * groups + g]);
                const float b = f_of_bf16(biases[size_t(row) * groups + g]);
                for (uint32_t j = 0; j < kGroup; ++j) {
                    const uint32_t c = g * kGroup + j;
                    acc += (static_cast<float>(q_at(row, c)) * s + b) * x[c];
                }
            }
            out[row] = acc;
        }
        return out;
    }
    void save(const std::string& p) const {
        put_b(p + ".w", packed);
        put_h(p + ".s", scales);
        put_h(p + ".b", biases);
        put_u(p + ".shape", {rows, in_dim, uint32_t(bits)});
    }
};

float rms_inv(const std::vector<float>& v, float eps) {
    double a = 0.0;
    for (float x : v) a += double(x) * x;
    return 1.0f / std::sqrt(static_cast<float>(a / v.size()) + eps);
}
}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) { std::fprintf(stderr, "usage: kat_gen OUT\n"); return 2; }
    g_out = std::fopen(argv[1], "wb");
    if (!g_out) return 1;

    std::mt19937 rng(12345);
    std::uniform_real_distribution<float> xf(-1.5f, 1.5f);

    {   // GemvInt4, 96 rows x 2816
        Quant m; m.draw(96, 2816, 4, rng);
        std::vector<float> x(2816); for (auto& v : x) v = xf(rng);
        m.save("gemv_int4"); put_f("gemv_int4.x", x); put_f("gemv_int4.want", m.expect(x));
    }
    {   // EmbedLookup: row 37 dequantised, times sqrt(2816) as a float
        Quant m; m.draw(64, 2816, 4, rng);
        const uint32_t token = 37;
        const float scale = std::sqrt(static_cast<float>(2816));
        std::vector<float> want(2816);
        const uint32_t groups = 2816 / kGroup;
        for (uint32_t g = 0; g < groups; ++g) {
            const float sc = f_of_bf16(m.scales[size_t(token) * groups + g]);
            const float b = f_of_bf16(m.biases[size_t(token) * groups + g]);
            for (uint32_t j = 0; j < kGroup; ++j) {
                const uint32_t c = g * kGroup + j;
                want[c] = static_cast<float>(m.q_at(token, c)) * sc + b;
            }
        }
        for (auto& v : want) v *= scale;
        m.save("embed"); put_u("embed.token", {token}); put_f("embed.want", want);
    }
    {   // RMSNormK, unweighted and weighted
        const uint32_t n = 2816; const float eps = 1e-6f;
        std::vector<float> x(n); for (auto& v : x) v = xf(rng);
        std::vector<uint16_t> w(n); for (auto& v : w) v = bf16_of_f(xf(rng) * 0.3f);
        const float inv = rms_inv(x, eps);
        std::vector<float> a(n), b(n);
        for (uint32_t i = 0; i < n; ++i) { a[i] = x[i] * inv; b[i] = x[i] * inv * f_of_bf16(w[i]); }
        put_f("rmsnorm.x", x); put_h("rmsnorm.w", w); put_f("rmsnorm.want_nw", a); put_f("rmsnorm.want_w", b);
    }
    {   // GemvInt8, 128 router rows x 2816
        Quant m; m.draw(128, 2816, 8, rng);
        std::vector<float> x(2816); for (auto& v : x) v = xf(rng);
        m.save("gemv_int8"); put_f("gemv_int8.x", x); put_f("gemv_int8.want", m.expect(x));
    }
    {   // GeGLU, n = 2112
        const uint32_t n = 2112;
        std::vector<float> g(n), u(n); for (auto& v : g) v = xf(rng); for (auto& v : u) v = xf(rng);
        std::vector<float> want(n);
        for (uint32_t i = 0; i < n; ++i) {
            const float x0 = g[i];
            const float t = 0.7978845608028654f * (x0 + 0.044715f * x0 * x0 * x0);
            want[i] = 0.5f * x0 * (1.0f + std::tanh(t)) * u[i];
        }
        put_f("geglu.g", g); put_f("geglu.u", u); put_f("geglu.want", want);
    }
    {   // Softcap: 30 * tanh(z / 30) in float
        const float cap = 30.0f;
        std::uniform_real_distribution<float> big(-200.0f, 200.0f);
        std::vector<float> z(4096), want(4096);
        for (auto& v : z) v = big(rng);
        for (size_t i = 0; i < z.size(); ++i) want[i] = cap * std::tanh(z[i] / cap);
        put_f("softcap.z", z); put_f("softcap.want", want);
    }
    {   // MulBF16
        const uint32_t n = 2816; const float scale = 0.0188478f;
        std::vector<float> x(n); std::vector<uint16_t> w(n);
        for (auto& v : x) v = xf(rng) * 2.0f;
        for (auto& v : w) v = bf16_of_f(xf(rng) * 0.3f);
        std::vector<float> want(n); for (uint32_t i = 0; i < n; ++i) want[i] = x[i] * f_of_bf16(w[i]) * scale;
        put_f("mulbf16.x", x); put_h("mulbf16.w", w); put_f("mulbf16.scale", {scale}); put_f("mulbf16.want", want);
    }
    {   // ScaleAccum, 8 experts into a destination pre-dirtied to 12345.0
        const uint32_t n = 2816, K = 8;
        std::vector<float> outs(size_t(K) * n);
        for (auto& v : outs) v = xf(rng);
        std::vector<float> weights(K); for (auto& v : weights) v = 0.05f + std::fabs(xf(rng)) * 0.2f;
        std::vector<float> want(n, 0.0f);
        for (uint32_t k = 0; k < K; ++k) for (uint32_t i = 0; i < n; ++i) want[i] += weights[k] * outs[size_t(k) * n + i];
        put_f("scaleaccum.in", outs); put_f("scaleaccum.weights", weights); put_f("scaleaccum.want", want);
    }
    {   // RouterTopK with a forced tie at 11/70
        const uint32_t NE = 128, K = 8;
        std::vector<float> logits(NE); for (auto& v : logits) v = xf(rng) * 4.0f;
        logits[11] = logits[70] = 9.5f;
        std::vector<uint16_t> pes(NE); for (auto& v : pes) v = bf16_of_f(0.5f + std::fabs(xf(rng)));
        std::vector<int> order(NE); for (uint32_t i = 0; i < NE; ++i) order[i] = int(i);
        std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
            if (logits[a] != logits[b]) return logits[a] > logits[b];
            return a < b;
        });
        float best = logits[order[0]], sum = 0.0f;
        std::vector<float> w(K); std::vector<uint32_t> idx(K);
        for (uint32_t i = 0; i < K; ++i) { w[i] = std::exp(logits[order[i]] - best); sum += w[i]; idx[i] = uint32_t(order[i]); }
        for (uint32_t i = 0; i < K; ++i) w[i] = w[i] / sum * f_of_bf16(pes[order[i]]);
        put_f("topk.logits", logits); put_h("topk.pes", pes); put_u("topk.want_idx", idx); put_f("topk.want_w", w);
    }
    {   // PostAttn: residual, then the three pre-FFN views
        const uint32_t D = 2816; const float eps = 1e-6f;
        std::vector<float> attn(D), hidden(D); for (auto& v : attn) v = xf(rng); for (auto& v : hidden) v = xf(rng);
        std::vector<uint16_t> wp(D), w1(D), w2(D);
        for (auto& v : wp) v = bf16_of_f(xf(rng) * 0.3f);
        for (auto& v : w1) v = bf16_of_f(xf(rng) * 0.3f);
        for (auto& v : w2) v = bf16_of_f(xf(rng) * 0.3f);
        const float ai = rms_inv(attn, eps);
        std::vector<float> wh(D); for (uint32_t i = 0; i < D; ++i) wh[i] = hidden[i] + attn[i] * ai * f_of_bf16(wp[i]);
        const float hi = rms_inv(wh, eps);
        std::vector<float> wd(D), wr(D), wx(D);
        for (uint32_t i = 0; i < D; ++i) {
            const float h = wh[i] * hi;
            wd[i] = h * f_of_bf16(w1[i]); wr[i] = h * f_of_bf16(w2[i]); wx[i] = h;
        }
        put_f("postattn.attn", attn); put_f("postattn.hidden", hidden);
        put_h("postattn.w_post", wp); put_h("postattn.w_pre", w1); put_h("postattn.w_pre2", w2);
        put_f("postattn.want_hidden", wh); put_f("postattn.want_dense", wd);
        put_f("postattn.want_routed", wr); put_f("postattn.want_router", wx);
    }
    {   // LayerTail: sandwich norms times layer_scalar 1.37
        const uint32_t D = 2816; const float eps = 1e-6f, ls = 1.37f;
        std::vector<float> h2(D), h1(D), hidden(D);
        for (auto& v : h2) v = xf(rng); for (auto& v : h1) v = xf(rng); for (auto& v : hidden) v = xf(rng);
        std::vector<uint16_t> wpf2(D), wpf(D);
        for (auto& v : wpf2) v = bf16_of_f(xf(rng) * 0.3f);
        for (auto& v : wpf) v = bf16_of_f(xf(rng) * 0.3f);
        const float i2 = rms_inv(h2, eps);
        std::vector<float> h12(D); for (uint32_t i = 0; i < D; ++i) h12[i] = h1[i] + h2[i] * i2 * f_of_bf16(wpf2[i]);
        const float i12 = rms_inv(h12, eps);
        std::vector<float> want(D);
        for (uint32_t i = 0; i < D; ++i) want[i] = (hidden[i] + h12[i] * i12 * f_of_bf16(wpf[i])) * ls;
        put_f("layertail.h2", h2); put_f("layertail.h1", h1); put_f("layertail.hidden", hidden);
        put_h("layertail.w_pf2", wpf2); put_h("layertail.w_pf", wpf); put_f("layertail.scalar", {ls});
        put_f("layertail.want", want);
    }
    {   // QKVEpilogue: per-head weighted norm, then 64 of 256 pairs rotated at position 7
        const uint32_t head_dim = 512, heads = 2, rotated = 64, position = 7;
        const float eps = 1e-6f, theta = 1000000.0f;
        std::vector<float> vec(heads * head_dim); for (auto& v : vec) v = xf(rng);
        std::vector<uint16_t> w(head_dim); for (auto& v : w) v = bf16_of_f(0.5f + xf(rng) * 0.2f);
        std::vector<float> want(vec.size());
        for (uint32_t h = 0; h < heads; ++h) {
            const float* src = vec.data() + h * head_dim;
            float* dst = want.data() + h * head_dim;
            double a = 0.0;
            for (uint32_t i = 0; i < head_dim; ++i) a += static_cast<double>(src[i]) * src[i];
            const float inv = 1.0f / std::sqrt(static_cast<float>(a / head_dim) + eps);
            for (uint32_t i = 0; i < head_dim; ++i) dst[i] = src[i] * inv * f_of_bf16(w[i]);
            const uint32_t half = head_dim / 2;
            for (uint32_t i = 0; i < rotated; ++i) {
                const float freq = std::pow(theta, -static_cast<float>(2 * i) / static_cast<float>(head_dim));
                const float ang = static_cast<float>(position) * freq;
                const float c = std::cos(ang), sn = std::sin(ang);
                const float x0 = dst[i], x1 = dst[i + half];
                dst[i] = x0 * c - x1 * sn;
                dst[i + half] = x0 * sn + x1 * c;
            }
        }
        put_f("qkv.vec", vec); put_h("qkv.w", w); put_f("qkv.want", want);
        put_u("qkv.shape", {head_dim, heads, rotated, position});
    }
    // Attention: q, then the K and V caches, drawn in that order; the want of the test's formula
    auto attention = [&](const std::string& name, uint32_t n_pos, uint32_t window, uint32_t capacity) {
        const uint32_t q_heads = 16, kv_heads = 8, head_dim = 256;
        const uint32_t first = n_pos - window;
        {
            std::ostringstream os;
            os << rng;
            std::istringstream is(os.str());
            std::vector<uint32_t> state;
            unsigned long long w;
            while (is >> w) state.push_back(static_cast<uint32_t>(w));
            put_u(name + ".rng_state", state);
        }
        std::vector<float> q(q_heads * head_dim);
        std::vector<float> kc(static_cast<size_t>(capacity) * kv_heads * head_dim), vc(kc.size());
        for (auto& v : q) v = xf(rng) * 0.1f;
        for (auto& v : kc) v = xf(rng) * 0.1f;
        for (auto& v : vc) v = xf(rng);
        std::vector<float> want(q.size(), 0.0f);
        const uint32_t gqa = q_heads / kv_heads;
        for (uint32_t h = 0; h < q_heads; ++h) {
            const uint32_t kvh = h / gqa;
            std::vector<float> sc(n_pos, 0.0f);
            float best = -1e30f;
            for (uint32_t t = first; t < n_pos; ++t) {
                const float* kt = kc.data() + ((t % capacity) * size_t(kv_heads) + kvh) * head_dim;
                float dot = 0.0f;
                for (uint32_t d = 0; d < head_dim; ++d) dot += q[h * head_dim + d] * kt[d];
                sc[t] = dot;
                best = std::max(best, dot);
            }
            float sum = 0.0f;
            for (uint32_t t = first; t < n_pos; ++t) { sc[t] = std::exp(sc[t] - best); sum += sc[t]; }
            for (uint32_t t = first; t < n_pos; ++t) {
                const float wt = sc[t] / sum;
                const float* vt = vc.data() + ((t % capacity) * size_t(kv_heads) + kvh) * head_dim;
                for (uint32_t d = 0; d < head_dim; ++d) want[h * head_dim + d] += wt * vt[d];
            }
        }
        put_f(name + ".q", q); put_f(name + ".want", want);
        put_u(name + ".shape", {q_heads, kv_heads, head_dim, n_pos, window, capacity});
    };
    attention("attn", 300, 128, 300);   // capacity == n_pos: a linear cache
    {   // LMHeadGreedy: draws only
        Quant m; m.draw(4096, 2816, 4, rng);
        std::vector<float> x(2816); for (auto& v : x) v = xf(rng);
    }
    attention("attn_ring", 300, 128, 128);
    std::fclose(g_out);
    return 0;
}

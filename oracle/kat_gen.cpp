// TEST INFRASTRUCTURE ONLY. Regenerates the known-answer fixtures of the reference's GPU
// kernel test (tests/test_gpu_kernels.cpp) for the MoE hot path: the same std::mt19937(12345)
// stream consumed in the same order with the same distributions (:226-227 and QuantMatrix::build
// :118-147), and the expected outputs computed with the test's own inline CPU formulas.
//
// Output: a flat record file, read by tests/golden/make_golden.py into tests/golden/kat.npz.
// Record: u32 name_len, name bytes, u32 dtype (0 f32, 1 u16, 2 u8, 3 u32), u64 count, payload.
//
// Cases, in the test's order (the ones not on the MoE path only advance the generator):
//   GemvInt4 96x2816 (:241-266)       EmbedLookup 64x2816 (:268-292, draws only)
//   RMSNormK (:294-336)               GemvInt8 128x2816 (:338-361)
//   GeGLU n=2112 (:363-387)           Softcap n=4096 (:389-411, draws only)
//   MulBF16 n=2816 (:413-441)         ScaleAccum 8x2816 (:443-482)
//   RouterTopK 128, K=8, tie 11/70 (:484-542)
//   PostAttn D=2816 (:544-601)        LayerTail D=2816 (:603-647)
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
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
    {   // EmbedLookup: draws only
        Quant m; m.draw(64, 2816, 4, rng);
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
    {   // Softcap: draws only
        std::uniform_real_distribution<float> big(-200.0f, 200.0f);
        for (int i = 0; i < 4096; ++i) (void)big(rng);
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
    std::fclose(g_out);
    return 0;
}

/*
 * TEST INFRASTRUCTURE ONLY. CPU restatement of the reference's token sampling; see
 * sampling_oracle.h. Each function names the lines of src/sampling.cpp it follows.
 */
#include "sampling_oracle.h"

#include <math.h>
#include <stdlib.h>

static const uint64_t kGolden = 0x9E3779B97F4A7C15ULL;   /* sampling.cpp:57, 68, 71 */

/* sampling.cpp:32-54: the same checks in the same order; NaN fails isfinite first. */
int orc_validate_sampling(const orc_sampling* p) {
    if (!isfinite(p->temperature) || p->temperature < 0.0f) return ORC_SAMPLING_BAD_TEMPERATURE;
    if (!isfinite(p->top_p) || p->top_p <= 0.0f || p->top_p > 1.0f) return ORC_SAMPLING_BAD_TOP_P;
    if (p->top_k < 0 || p->top_k > ORC_SAMPLING_MAX_TOP_K) return ORC_SAMPLING_BAD_TOP_K;
    if (!isfinite(p->repetition_penalty) || p->repetition_penalty <= 0.0f) return ORC_SAMPLING_BAD_PENALTY;
    /* a nucleus cut is only defined inside a top-k bound (the shortlist below depends on it) */
    if (p->temperature > 0.0f && p->top_p < 1.0f && p->top_k == 0) return ORC_SAMPLING_NUCLEUS_NEEDS_TOP_K;
    return ORC_SAMPLING_OK;
}

/* cpu_reference.cpp:534-538, in float: z / cap, tanhf, cap * t. */
void orc_softcap(float* z, size_t n, float cap) {
    if (!(cap > 0.0f)) return;
    for (size_t i = 0; i < n; ++i) z[i] = cap * tanhf(z[i] / cap);
}

/* sampling.cpp:56-61: Vigna's splitmix64 finaliser. */
uint64_t orc_splitmix64(uint64_t x) {
    uint64_t z = x + kGolden;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* sampling.cpp:63-72: one generator state per position; never 0 (xorshift would stick at 0). */
uint64_t orc_seed_for(const orc_sampling* p, int position) {
    const uint64_t pos = (uint64_t)(int64_t)position;
    const uint64_t base = p->has_seed ? p->seed + pos : (kGolden ^ (pos * 0xD1B54A32D192ED03ULL));
    const uint64_t s = orc_splitmix64(base);
    return s != 0 ? s : kGolden;
}

/* sampling.cpp:74-90: for every history entry in order (duplicates apply again), a positive
 * logit is divided by the penalty and any other multiplied, then clamped inside the softcap. */
void orc_apply_repetition_penalty(float* logits, uint32_t vocab, const uint32_t* history, size_t n_history,
                                  float penalty, float softcap) {
    if (penalty == 1.0f || n_history == 0) return;
    const float limit = softcap > 0.0f ? softcap * 0.9999f : 0.0f;
    for (size_t h = 0; h < n_history; ++h) {
        const uint32_t id = history[h];
        if (id >= vocab) continue;
        float v = logits[id];
        v = v > 0.0f ? v / penalty : v * penalty;
        if (limit > 0.0f) v = v < -limit ? -limit : (limit < v ? limit : v);
        logits[id] = v;
    }
}

/* The candidate order of sampling.cpp:128-131: logit descending, then id ascending. */
static int before(const float* l, uint32_t a, uint32_t b) {
    if (l[a] != l[b]) return l[a] > l[b];
    return a < b;
}

/* sampling.cpp:106-151: max logit, the full-vocabulary double denominator, the shortlist (a
 * partial selection of the first `want` ids in candidate order, kept sorted by insertion), then
 * the nucleus cut measured against the full denominator and the top-k cut. */
static int shortlist(const float* logits, uint32_t vocab, const orc_sampling* p, uint32_t* ids, uint32_t* n_ids,
                     uint32_t* cut_out, float* max_out) {
    if (vocab == 0) return ORC_SAMPLE_EMPTY_VOCAB;
    float mx = logits[0];
    for (uint32_t i = 1; i < vocab; ++i) mx = mx < logits[i] ? logits[i] : mx;   /* std::max(mx, l) */
    double total = 0.0;
    for (uint32_t i = 0; i < vocab; ++i) total += exp((double)logits[i] - (double)mx);
    if (!(total > 0.0)) return ORC_SAMPLE_DEGENERATE;

    const uint32_t cap = p->top_k > 0 ? (uint32_t)p->top_k : ORC_SAMPLING_MAX_TOP_K;
    const uint32_t want = cap < vocab ? cap : vocab;
    uint32_t n = 0;
    for (uint32_t i = 0; i < vocab; ++i) {
        if (n == want && !before(logits, i, ids[n - 1])) continue;
        uint32_t j = n < want ? n++ : n - 1;   /* drop the last when full */
        while (j > 0 && before(logits, i, ids[j - 1])) {
            ids[j] = ids[j - 1];
            --j;
        }
        ids[j] = i;
    }

    uint32_t cut = n;
    if (p->top_p < 1.0f) {
        double run = 0.0;
        for (uint32_t i = 0; i < n; ++i) {
            run += exp((double)logits[ids[i]] - (double)mx) / total;
            if (run >= (double)p->top_p) {
                cut = i + 1;
                break;
            }
        }
    }
    if (p->top_k > 0 && cut > (uint32_t)p->top_k) cut = (uint32_t)p->top_k;
    if (cut < 1) cut = 1;
    *n_ids = n;
    *cut_out = cut;
    *max_out = mx;
    return ORC_SAMPLE_OK;
}

int orc_sample_shortlist(const float* logits, uint32_t vocab, const orc_sampling* p, uint32_t* ids,
                         uint32_t* n_ids, uint32_t* cut) {
    float mx;
    return shortlist(logits, vocab, p, ids, n_ids, cut, &mx);
}

/* sampling.cpp:17-28: xorshift64*, then 24 bits as a float in [0, 1). */
static float uniform24(uint64_t state) {
    state ^= state >> 12;
    state ^= state << 25;
    state ^= state >> 27;
    const uint64_t r = state * 0x2545F4914F6CDD1DULL;
    return (float)((r >> 40) & 0xFFFFFFu) / 16777216.0f;
}

/* sampling.cpp:92-169. */
int orc_sample_token(const float* logits, uint32_t vocab, const orc_sampling* p, uint64_t seed, uint32_t* token) {
    if (vocab == 0) return ORC_SAMPLE_EMPTY_VOCAB;
    if (p->temperature <= 0.0f) {   /* greedy: strict >, so ties stay on the lower id */
        uint32_t best = 0;
        float bv = logits[0];
        for (uint32_t i = 1; i < vocab; ++i)
            if (logits[i] > bv) {
                bv = logits[i];
                best = i;
            }
        *token = best;
        return ORC_SAMPLE_OK;
    }
    uint32_t ids[ORC_SAMPLING_MAX_TOP_K], n, cut;
    float mx;
    const int rc = shortlist(logits, vocab, p, ids, &n, &cut, &mx);
    if (rc != ORC_SAMPLE_OK) return rc;

    /* temperature acts on the final draw only, over the survivors, in double */
    double q[ORC_SAMPLING_MAX_TOP_K], denom = 0.0;
    for (uint32_t i = 0; i < cut; ++i) {
        q[i] = exp(((double)logits[ids[i]] - (double)mx) / (double)p->temperature);
        denom += q[i];
    }
    const double r = (double)uniform24(seed) * denom;
    double acc = 0.0;
    for (uint32_t i = 0; i < cut; ++i) {
        acc += q[i];
        if (acc >= r) {
            *token = ids[i];
            return ORC_SAMPLE_OK;
        }
    }
    *token = ids[cut - 1];   /* reachable only through rounding */
    return ORC_SAMPLE_OK;
}

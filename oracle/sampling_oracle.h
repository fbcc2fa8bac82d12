/*
 * TEST INFRASTRUCTURE ONLY. CPU restatement of the reference's token sampling
 * (src/sampling.cpp, include/gturbo/sampling.hpp): the checker for a device sampler and for the
 * host-side parameter rules. Nothing on the product path links or calls this code.
 *
 * Pinned against the reference's own compiled sampling.cpp (oracle/_ref/libgtref.so) and the
 * known answers of its tests/test_sampling.cpp (tests/golden/sampling.npz). Build with
 * -O2 -ffp-contract=off (no FMA contraction, no fast-math); `exp` is the C library's, the same
 * routine the reference's std::exp(double) calls on this host.
 */
#ifndef GTM_SAMPLING_ORACLE_H
#define GTM_SAMPLING_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* include/gturbo/sampling.hpp:21-30 SamplingParams; has_seed widened to an int. */
typedef struct orc_sampling {
    float temperature;          /* 0 = greedy */
    float top_p;                /* 1 = no nucleus cut */
    int32_t top_k;              /* 0 = no top-k cut (the shortlist is still the top 256) */
    float repetition_penalty;   /* 1 = off */
    int32_t has_seed;
    uint32_t pad_;
    uint64_t seed;
} orc_sampling;

/* The rule validate_sampling rejects (0 = accepted), in the order sampling.cpp:32-54 checks. */
enum {
    ORC_SAMPLING_OK = 0,
    ORC_SAMPLING_BAD_TEMPERATURE = 1,
    ORC_SAMPLING_BAD_TOP_P = 2,
    ORC_SAMPLING_BAD_TOP_K = 3,
    ORC_SAMPLING_BAD_PENALTY = 4,
    ORC_SAMPLING_NUCLEUS_NEEDS_TOP_K = 5,
};

/* sample_token's failures (sampling.cpp:94, 116-118). */
enum { ORC_SAMPLE_OK = 0, ORC_SAMPLE_EMPTY_VOCAB = 1, ORC_SAMPLE_DEGENERATE = 2 };

#define ORC_SAMPLING_MAX_TOP_K 256   /* sampling.cpp:15 */

int orc_validate_sampling(const orc_sampling* p);
/* Final logit softcapping (cpu_reference.cpp:534-538): z = cap * tanhf(z / cap) when cap > 0. */
void orc_softcap(float* z, size_t n, float cap);
uint64_t orc_splitmix64(uint64_t x);
uint64_t orc_seed_for(const orc_sampling* p, int position);
void orc_apply_repetition_penalty(float* logits, uint32_t vocab, const uint32_t* history, size_t n_history,
                                  float penalty, float softcap);
/* Writes the drawn token id to *token. Logits must not hold NaN: the reference's candidate
 * ordering is not a strict weak order with NaN, so its result is unspecified there. */
int orc_sample_token(const float* logits, uint32_t vocab, const orc_sampling* p, uint64_t seed, uint32_t* token);
/* The shortlist sample_token draws from: min(top_k or 256, vocab) ids in (logit desc, id asc)
 * order, and how many of them survive the nucleus and top-k cuts. Returns the same codes. */
int orc_sample_shortlist(const float* logits, uint32_t vocab, const orc_sampling* p, uint32_t* ids,
                         uint32_t* n_ids, uint32_t* cut);

#ifdef __cplusplus
}
#endif
#endif

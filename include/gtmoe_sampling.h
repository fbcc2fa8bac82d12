/*
 * gtmoe_sampling.h -- token sampling after the LM head (C ABI).
 *
 * Replaces the host-side sampling the reference runs on logits read back from the GPU
 * (src/sampling.cpp, include/gturbo/sampling.hpp; called from the sampled branch of
 * ForwardRunner::produce_token, src/runner.cpp:771-806, and from src/cpu_reference.cpp): the
 * repetition penalty is applied to the softcapped logits in device memory, and the token is
 * drawn on the device, so a sampled token needs no 1 MB read-back.
 *
 * Same rules as the reference: Top-P over the FULL distribution, then Top-K over the
 * survivors, then temperature on the final draw; greedy (temperature <= 0) is the argmax with
 * ties to the lower id; one xorshift64* uniform per token from a per-position seed.
 * Logits must not contain NaN (the reference's candidate order is undefined there).
 *
 * The device entries are built to match the reference bit for bit except where a decision
 * compares two doubles that agree to ~1e-10 relative: the reference sums exp() of the whole
 * vocabulary in order on the host, the device in parallel, and CUDA's double exp() may differ
 * from the C library's in the last bit. The status word reports every decision whose margin lies
 * inside that bound. The device entries are checked on a B200 against the reference's compiled
 * sampling.cpp outputs (tokens and penalised logits bit-identical, no draw flagged); the
 * host-side rules (validate, splitmix64, seed_for) against the same code on the CPU.
 */
#ifndef GTMOE_SAMPLING_H
#define GTMOE_SAMPLING_H

#include "gtmoe.h"

#ifdef __cplusplus
extern "C" {
#endif

/* SamplingParams (include/gturbo/sampling.hpp:21-30); has_seed as an int. */
typedef struct GtmSampling {
    float temperature;          /* 0 = greedy */
    float top_p;                /* 1 = no nucleus cut */
    int32_t top_k;              /* 0 = no top-k cut; the shortlist is then the top 256 */
    float repetition_penalty;   /* 1 = off */
    int32_t has_seed;
    uint32_t reserved;          /* 0 */
    uint64_t seed;
} GtmSampling;

#define GTM_SAMPLE_MAX_TOP_K 256          /* sampling.cpp:15 */
#define GTM_SAMPLE_MAX_VOCAB (1u << 22)

/* Bits of the device status word written by gtm_sample_token. */
#define GTM_SAMPLE_DEGENERATE 1u   /* max logit is +-inf: the reference throws "degenerate"; token = 0xFFFFFFFF */
#define GTM_SAMPLE_NEAR_CUT 2u     /* the nucleus cut compared values inside the error bound */
#define GTM_SAMPLE_NEAR_DRAW 4u    /* the draw compared values inside the error bound */

/* validate_sampling (sampling.cpp:32-54): GTM_OK, or GTM_ERR_INVALID with the reference's
 * message in gtm_last_error(). Host only. */
GTM_API int gtm_sampling_validate(const GtmSampling* p);
/* splitmix64 (sampling.cpp:56-61). Host only. */
GTM_API uint64_t gtm_sampling_splitmix64(uint64_t x);
/* seed_for (sampling.cpp:63-72): the generator state for `position`; never 0. Host only. */
GTM_API uint64_t gtm_sampling_seed_for(const GtmSampling* p, int position);

/* Softcap (shaders/Softcap.hlsl; cpu_reference.cpp:534-538): out = cap * tanh(in / cap) for n
 * fp32 values, in place when in_dev == out_dev. Device tanhf rounds differently from the C
 * library's in the last bits. */
GTM_API int gtm_softcap(uint32_t n, const float* in_dev, float cap, float* out_dev, void* stream);

/* Device workspace for a vocabulary of `vocab` ids (256-byte aligned; no initialisation). */
GTM_API size_t gtm_sample_workspace_bytes(uint32_t vocab);

/* apply_repetition_penalty (sampling.cpp:74-90) on device logits, in place: for every history
 * entry in order (repeats apply again; ids >= vocab are ignored) a positive logit is divided by
 * `penalty`, any other multiplied, then clamped to +-0.9999 * softcap when softcap > 0.
 * history_dev: uint32 ids on the device. Asynchronous on `stream`. */
GTM_API int gtm_repetition_penalty(float* logits_dev, uint32_t vocab, const uint32_t* history_dev, uint32_t n_history,
                                   float penalty, float softcap, void* workspace_dev, size_t workspace_bytes,
                                   void* stream);

/* sample_token (sampling.cpp:92-169) on device logits: writes the token id to token_dev and the
 * GTM_SAMPLE_* bits to status_dev (both uint32 on the device; 0 = a token, no near decision).
 * `p` must pass gtm_sampling_validate; `seed` is the state from gtm_sampling_seed_for.
 * Asynchronous on `stream`. */
GTM_API int gtm_sample_token(const float* logits_dev, uint32_t vocab, const GtmSampling* p, uint64_t seed,
                             uint32_t* token_dev, uint32_t* status_dev, void* workspace_dev, size_t workspace_bytes,
                             void* stream);

#ifdef __cplusplus
}
#endif
#endif

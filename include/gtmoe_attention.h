/*
 * gtmoe_attention.h -- the decoder remainder around the MoE block for batch-1 decode (C ABI):
 * embedding lookup, the per-head q/k/v epilogue and attention over the FP32 ring KV cache.
 *
 * Replaces, for one token of ForwardRunner::produce_token (src/runner.cpp:487-533), the
 * EmbedLookup, QKVEpilogue and Attention dispatches (shaders/EmbedLookup.hlsl,
 * shaders/QKVEpilogue.hlsl, shaders/Attention.hlsl); the q/k/v/o projections stay on
 * gtm_gemv_q4 (GemvInt4). Arithmetic contract: src/cpu_reference.cpp:108-140, 322-417.
 * KV rows live where KVCacheManager puts them (src/kv_cache.cpp:36-50): position p of a layer
 * in row p % capacity, each row kv_heads * head_dim floats.
 *
 * Checked on a B200 against the reference's kernel-test known answers (EmbedLookup bit-identical,
 * QKVEpilogue and Attention with window and ring wrap within its allclose rule) and, chained with
 * the MoE block and the greedy LM head, against the reference's own generate tokens.
 */
#ifndef GTMOE_ATTENTION_H
#define GTMOE_ATTENTION_H

#include "gtmoe.h"

#ifdef __cplusplus
extern "C" {
#endif

/* EmbedLookup (cpu_reference.cpp:322-330): out[c] = (q[token][c] * s + b) * scale, int4 MLX
 * affine rows of in_dim elements (group 64). Bit-identical to the CPU reference with
 * scale = sqrtf(in_dim). */
GTM_API int gtm_embed_lookup(uint32_t rows, uint32_t in_dim, const void* w_dev, const uint16_t* s_dev,
                             const uint16_t* b_dev, uint32_t token, float scale, float* out_dev, void* stream);

/* QKVEpilogue (cpu_reference.cpp:360-376): for each of `heads` vectors of head_dim floats, an
 * RMS norm with bf16 weight w_dev (NULL = no scale), then NeoX RoPE of the first rotated_pairs
 * pairs at `position` with base theta (rotated_pairs = 0: no rotation). in_dev and out_dev may
 * be the same buffer; out_dev may point into a KV cache row. head_dim in {128, 256, 512}. */
GTM_API int gtm_qkv_epilogue(uint32_t heads, uint32_t head_dim, const float* in_dev, const uint16_t* w_dev, float eps,
                             uint32_t rotated_pairs, uint32_t position, float theta, float* out_dev, void* stream);

/* Workspace for gtm_attention_decode with at most `max_window` attended positions. */
GTM_API size_t gtm_attention_workspace_bytes(uint32_t q_heads, uint32_t head_dim, uint32_t max_window);

/* Attention (cpu_reference.cpp:382-414): for each query head h (kv head h / (q_heads /
 * kv_heads)), scores q.k with scale 1.0 over positions [first, n_pos), softmax, and the
 * weighted sum of V into ctx_dev [q_heads * head_dim]. Position t is cache row t % capacity.
 * q_heads a multiple of kv_heads with q_heads / kv_heads <= 8; head_dim in {128, 256, 512};
 * first < n_pos; n_pos - first <= capacity. */
GTM_API int gtm_attention_decode(uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim, uint32_t n_pos,
                                 uint32_t first, uint32_t capacity, const float* q_dev, const float* k_cache_dev,
                                 const float* v_cache_dev, float* ctx_dev, void* workspace_dev, size_t workspace_bytes,
                                 void* stream);

/* ---------------------------------------------------------------------------------------
 * The same steps for n sequences at once (a batched decode step; the reference decodes one
 * sequence per produce_token call, runner.cpp:487-533). Row i of every [n][...] array belongs to
 * the i-th sequence of the step; per-row token ids, positions and sequence indices are HOST
 * arrays of n values (n <= 512), checked on the host and passed to the kernels by value. Every
 * row's result is bit-identical to the single-sequence entry on that row.
 * ------------------------------------------------------------------------------------- */
/* EmbedLookup of tokens[i] into out_dev row i ([n][in_dim]). */
GTM_API int gtm_embed_lookup_rows(uint32_t rows, uint32_t in_dim, const void* w_dev, const uint16_t* s_dev,
                                  const uint16_t* b_dev, const uint32_t* tokens, uint32_t n, float scale, float* out_dev,
                                  void* stream);
/* QKVEpilogue of in_dev row i ([n][heads * head_dim]) at positions[i]. capacity = 0: into out_dev
 * row i (out may be in). capacity > 0: into ring row positions[i] % capacity of the cache of
 * sequence seqs[i] < num_seqs, the caches laid out [num_seqs][capacity][heads * head_dim]. */
GTM_API int gtm_qkv_epilogue_rows(uint32_t heads, uint32_t head_dim, uint32_t n, const float* in_dev,
                                  const uint16_t* w_dev, float eps, uint32_t rotated_pairs, const uint32_t* positions,
                                  float theta, float* out_dev, const uint32_t* seqs, uint32_t num_seqs,
                                  uint32_t capacity, void* stream);
/* Workspace of gtm_attention_decode_rows for n rows attending at most max_window positions. */
GTM_API size_t gtm_attention_rows_workspace_bytes(uint32_t q_heads, uint32_t head_dim, uint32_t max_window,
                                                  uint32_t n);
/* Attention of q_dev row i ([n][q_heads * head_dim]) over the caches of sequence seqs[i]
 * ([num_seqs][capacity][kv_heads * head_dim]) at position positions[i]: positions
 * [first, positions[i]] with first = max(0, positions[i] + 1 - window) (window 0 = all), into
 * ctx_dev row i. The attended span must fit the ring (<= capacity). */
GTM_API int gtm_attention_decode_rows(uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim, uint32_t n,
                                      uint32_t window, uint32_t capacity, const float* q_dev, const float* k_cache_dev,
                                      const float* v_cache_dev, const uint32_t* seqs, uint32_t num_seqs,
                                      const uint32_t* positions, float* ctx_dev, void* workspace_dev,
                                      size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif

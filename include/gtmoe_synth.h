/*
 * gtmoe_synth.h -- synthetic MoE weights and activations generated on the device.
 *
 * Benchmark and test support with no counterpart in the reference: the reference loads a
 * converted checkpoint; the benchmark configurations use random-init weights of the same
 * shapes, generated here straight into HBM in the .gturbo byte layouts (an expert image laid
 * out like packed_experts/layer_NN.bin, and one layer's resident tensors on 16 KB boundaries
 * like resident.bin). The values are a pure function of (seed, layer, tensor, index) and are
 * bit-identical with the CPU generator used by the test oracle.
 */
#ifndef GTMOE_SYNTH_H
#define GTMOE_SYNTH_H

#include <stddef.h>
#include <stdint.h>

#include "gtmoe.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Byte layout of one routed-expert block: offsets[9] (gate w/s/b, up w/s/b, down w/s/b, the
 * converter's order) and the 16 KB-padded stride. */
GTM_API int gtm_synth_expert_layout(uint32_t hidden, uint32_t inter, uint64_t offsets[9], uint64_t* stride);
/* Byte layout of one layer's resident tensors: offsets[20] in the order router w/s/b,
 * router.scale, per_expert_scale, shared gate w/s/b, up w/s/b, down w/s/b, pre_ffn_norm,
 * pre_ffn_norm_2, post_ffn_norm_1, post_ffn_norm_2, post_ffn_norm, layer_scalar. */
GTM_API int gtm_synth_resident_layout(uint32_t hidden, uint32_t ffn, uint32_t experts, uint64_t offsets[20],
                                      uint64_t* total);
/* Fills experts [first, first + count) of `layer` into dst_dev (expert e at
 * (e - first) * stride). */
GTM_API int gtm_synth_experts(uint64_t seed, uint32_t layer, uint32_t hidden, uint32_t inter, uint32_t first,
                              uint32_t count, void* dst_dev, void* stream);
/* Fills one layer's resident image (size from gtm_synth_resident_layout). */
GTM_API int gtm_synth_resident(uint64_t seed, uint32_t layer, uint32_t hidden, uint32_t ffn, uint32_t experts,
                               void* dst_dev, void* stream);
/* Block inputs x ~ N(0,1) for tokens [token0, token0 + count): fp32 [count][hidden]. */
GTM_API int gtm_synth_x(uint64_t seed, uint32_t token0, uint32_t count, uint32_t hidden, float* dst_dev, void* stream);
/* A synthetic int4 matrix outside the MoE block (attention projections, tied embedding of the
 * decoder benchmark): packed words [rows][in_dim/8], bf16 scales and biases [rows][in_dim/64]
 * drawn like the expert matrices (q ~ U{0..15}, scale |N(0, 0.02)|, bias -8 scale) from the
 * streams (seed, layer, kind_w) and (seed, layer, kind_s); callers use kinds >= 32. */
GTM_API int gtm_synth_quant(uint64_t seed, uint32_t layer, uint32_t kind_w, uint32_t kind_s, uint32_t rows,
                            uint32_t in_dim, void* w_dev, uint16_t* s_dev, uint16_t* b_dev, void* stream);
/* A synthetic bf16 norm vector of n elements (1 + N(0, 0.1), like the MoE norm weights). */
GTM_API int gtm_synth_norm(uint64_t seed, uint32_t layer, uint32_t kind, uint32_t n, uint16_t* dst_dev, void* stream);
/* Fills a GtmLayer for a synthetic layer whose resident image and expert image live at the
 * given device addresses. */
GTM_API int gtm_synth_layer_desc(uint32_t hidden, uint32_t moe_inter, uint32_t ffn, uint32_t experts,
                                 const void* resident_dev, const void* experts_dev, GtmLayer* out);

#ifdef __cplusplus
}
#endif
#endif

/*
 * gtmoe_bundle.h -- `.gturbo` bundle loader straight into device memory (C ABI).
 *
 * A bundle directory holds (the reference's v1 format):
 *   manifest.json               magic "GTURBO", version 1.x, flags, arch, numLayers,
 *                               expertsPerLayer, expertStride        (src/manifest.cpp:24-49, 157-240)
 *   packed_experts/layout.json  expertStride, numLayers, expertsPerLayer, the nine expertBlock
 *                               sub-tensors, layers[] -> layer file  (src/packed_experts.cpp:15-166)
 *   packed_experts/layer_NN.bin expert e of the layer at e * expertStride
 *   resident.bin                a little-endian index (24-byte header, 72-byte entries, string
 *                               table; 16 KB-aligned, at most 16 MB) followed by the tensors at
 *                               their file offsets             (src/resident_index.cpp:40-97)
 *
 * Replaces, for the MoE path, the engine's bundle loading (ForwardRunner resident.bin upload,
 * src/runner.cpp:248-292, resident_ref / layer_ref :319-353) and the NVMe expert streamer
 * (src/streamer.cpp): every expert is loaded once into HBM, so the decode path needs no slot
 * cache. The bytes are copied unchanged; GtmLayer then addresses them by the index's offsets.
 *
 * Loads are blocking: they return once the bytes are in device memory. Reader threads read the
 * files into pinned staging buffers (allocated on the first load, kept until gtm_bundle_close)
 * and copy each chunk to the device with cudaMemcpyAsync. One thread at a time per bundle.
 */
#ifndef GTMOE_BUNDLE_H
#define GTMOE_BUNDLE_H

#include "gtmoe.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct GtmBundle GtmBundle;

typedef struct GtmBundleInfo {
    uint32_t num_layers, experts_per_layer;
    uint32_t hidden, moe_inter, ffn_inter, top_k;
    float rms_norm_eps;
    uint32_t resident_entries;
    uint64_t expert_stride;
    uint64_t resident_bytes;        /* size of resident.bin: what gtm_bundle_load_resident copies */
    uint64_t resident_index_bytes;  /* the index region at its start                               */
    uint64_t layer_file_bytes;      /* experts_per_layer * expert_stride                           */
} GtmBundleInfo;

/* Parses and validates manifest.json, packed_experts/layout.json (each against the other) and
 * the resident.bin index, and checks that every layer file holds experts_per_layer strides.
 * GTM_ERR_INVALID with a message naming the field for a malformed bundle. */
GTM_API int gtm_bundle_open(const char* dir, GtmBundle** bundle_out);
GTM_API int gtm_bundle_close(GtmBundle* bundle);
GTM_API int gtm_bundle_info(const GtmBundle* bundle, GtmBundleInfo* info_out);
/* resident.bin, whole, into dst_dev (dst_bytes >= info.resident_bytes). Blocking. */
GTM_API int gtm_bundle_load_resident(GtmBundle* bundle, void* dst_dev, uint64_t dst_bytes);
/* Experts [first, first + count) of `layer` into dst_dev, expert e at (e - first) * stride
 * (dst_bytes >= count * stride). An expert-parallel rank loads only its own experts. Blocking. */
GTM_API int gtm_bundle_load_experts(GtmBundle* bundle, uint32_t layer, uint32_t first, uint32_t count,
                                    void* dst_dev, uint64_t dst_bytes);
/* The MoE tensors of `layer` (model.layers.<layer>.router.proj.weight, router.scale,
 * router.per_expert_scale, mlp.{gate,up,down}_proj.weight, the pre/post feed-forward norms,
 * layer_scalar) looked up by name in the resident index, and the expertBlock offsets, as a
 * GtmLayer over resident_dev (resident.bin as loaded) and experts_dev (the layer's experts as
 * loaded, the first one at experts_dev). GTM_ERR_INVALID when a tensor is missing or its
 * size, dtype or shape does not fit the MoE block's dimensions. */
GTM_API int gtm_bundle_layer_desc(const GtmBundle* bundle, uint32_t layer, const void* resident_dev,
                                  const void* experts_dev, GtmLayer* layer_out);

#ifdef __cplusplus
}
#endif
#endif /* GTMOE_BUNDLE_H */

"""Test helper: writes a `.gturbo` v1 bundle of the synthetic model, so the loader
(include/gtmoe_bundle.h) can be checked against bytes whose origin is known.

The on-disk scheme restates the reference converter (tools/convert_hf_to_gturbo.py):
- resident.bin: one entry per tensor, named as the Hugging Face tensor minus "language_model."
  (:293-329); the index is a 24-byte header (index_size, resident_size, entry_count), 72-byte
  entries (name offset u32, name length u16, dtype u8, reserved 0, offset, size, shape[4],
  scale offset/size, bias offset/size) and the names, padded to 16 KB (:352-376); each payload,
  scale table and bias table starts on a 16 KB boundary after the index (:332-349);
- packed_experts/layer_NN.bin: expert e at e * expertStride; layout.json lists the nine
  expertBlock sub-tensors and the layer files (src/packed_experts.cpp:86-113);
- manifest.json: magic, version, flags, arch, numLayers, expertsPerLayer, expertStride
  (src/manifest.cpp:54-135).

Contents come from the oracle's generator (byte-identical to the device's gtm_synth_*), layer by
layer: the 20 resident regions of the synthetic per-layer image become the layer's MoE tensors.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import struct

import numpy as np

import oracle

ALIGN = 16384
HIDDEN, MOE_INTER, FFN, EXPERTS = 2816, 704, 2112, 128
U32, BF16 = 0, 1


def align_up(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def synth_resident_layout():
    """Offsets and sizes of the 20 regions of one synthetic layer image (csrc/gtm_synth.h)."""
    H, F, E = HIDDEN, FFN, EXPERTS
    sizes = [E * H, E * (H // 64) * 2, E * (H // 64) * 2, H * 2, E * 2,
             F * H // 2, F * (H // 64) * 2, F * (H // 64) * 2,
             F * H // 2, F * (H // 64) * 2, F * (H // 64) * 2,
             H * F // 2, H * (F // 64) * 2, H * (F // 64) * 2,
             H * 2, H * 2, H * 2, H * 2, H * 2, 2]
    offs, cur = [], 0
    for sz in sizes:
        offs.append(cur)
        cur = align_up(cur + sz)
    return offs, sizes, cur


def synth_resident_bytes(seed: int, layer: int) -> np.ndarray:
    offs, sizes, total = synth_resident_layout()
    buf = np.zeros(total, np.uint8)
    oracle.lib().orc_synth_resident(C.c_uint64(seed), layer, HIDDEN, FFN, EXPERTS,
                                    buf.ctypes.data_as(C.c_void_p))
    return buf


def layer_entries(layer: int, img: np.ndarray):
    """(name, dtype, shape, payload, scales, biases) of one layer's MoE tensors."""
    offs, sizes, _ = synth_resident_layout()
    reg = [img[o:o + s] for o, s in zip(offs, sizes)]
    P = f"model.layers.{layer}."
    H, F, E = HIDDEN, FFN, EXPERTS
    return [
        (P + "router.proj.weight", U32, [E, H // 4], reg[0], reg[1], reg[2]),
        (P + "router.scale", BF16, [H], reg[3], None, None),
        (P + "router.per_expert_scale", BF16, [E], reg[4], None, None),
        (P + "mlp.gate_proj.weight", U32, [F, H // 8], reg[5], reg[6], reg[7]),
        (P + "mlp.up_proj.weight", U32, [F, H // 8], reg[8], reg[9], reg[10]),
        (P + "mlp.down_proj.weight", U32, [H, F // 8], reg[11], reg[12], reg[13]),
        (P + "pre_feedforward_layernorm.weight", BF16, [H], reg[14], None, None),
        (P + "pre_feedforward_layernorm_2.weight", BF16, [H], reg[15], None, None),
        (P + "post_feedforward_layernorm_1.weight", BF16, [H], reg[16], None, None),
        (P + "post_feedforward_layernorm_2.weight", BF16, [H], reg[17], None, None),
        (P + "post_feedforward_layernorm.weight", BF16, [H], reg[18], None, None),
        (P + "layer_scalar", BF16, [1], reg[19], None, None),
    ]


def expert_block():
    """The nine sub-tensors of one expert block in converter order (offsets packed tight)."""
    H, M = HIDDEN, MOE_INTER
    w, gs, ds = M * H // 2, M * (H // 64) * 2, H * (M // 64) * 2
    parts = [("gate_proj.weight", w, U32, [M, H // 8]), ("gate_proj.scales", gs, BF16, [M, H // 64]),
             ("gate_proj.biases", gs, BF16, [M, H // 64]), ("up_proj.weight", w, U32, [M, H // 8]),
             ("up_proj.scales", gs, BF16, [M, H // 64]), ("up_proj.biases", gs, BF16, [M, H // 64]),
             ("down_proj.weight", w, U32, [H, M // 8]), ("down_proj.scales", ds, BF16, [H, M // 64]),
             ("down_proj.biases", ds, BF16, [H, M // 64])]
    block, cur = {}, 0
    for name, size, dt, shape in parts:
        block[name] = {"offset": cur, "size": size, "dtype": dt, "shape": shape}
        cur += size
    return block, align_up(cur)


def write_resident(path: str, entries, extra_names=()):
    """resident.bin with the converter's index and 16 KB-aligned payloads. Returns
    {name: (offset, size, scale_offset, scale_size, bias_offset, bias_size)}."""
    entries = list(entries) + [(n, BF16, [8], np.zeros(16, np.uint8), None, None) for n in extra_names]
    names = [e[0].encode() for e in entries]
    raw_index = 24 + 72 * len(entries) + sum(len(n) for n in names)
    index_size = align_up(raw_index)
    cursor = index_size
    plan = {}
    for name, dt, shape, pay, sc, bi in entries:
        off = cursor
        cursor = align_up(cursor + pay.size)
        so = ss = bo = bs = 0
        if sc is not None:
            so, ss = cursor, sc.size
            cursor = align_up(cursor + sc.size)
        if bi is not None:
            bo, bs = cursor, bi.size
            cursor = align_up(cursor + bi.size)
        plan[name] = (off, pay.size, so, ss, bo, bs)
    resident_size = cursor
    table_end = 24 + 72 * len(entries)
    table, strings = bytearray(), bytearray()
    for (name, dt, shape, pay, sc, bi), raw in zip(entries, names):
        off, sz, so, ss, bo, bs = plan[name]
        table += struct.pack("<IHBB", table_end + len(strings), len(raw), dt, 0)
        table += struct.pack("<QQ", off, sz)
        table += struct.pack("<4I", *((list(shape) + [0, 0, 0, 0])[:4]))
        table += struct.pack("<QQQQ", so, ss, bo, bs)
        strings += raw
    region = struct.pack("<QQQ", index_size, resident_size, len(entries)) + bytes(table) + bytes(strings)
    out = np.zeros(resident_size, np.uint8)
    out[:len(region)] = np.frombuffer(region, np.uint8)
    for name, dt, shape, pay, sc, bi in entries:
        off, sz, so, ss, bo, bs = plan[name]
        out[off:off + sz] = pay
        if sc is not None:
            out[so:so + ss] = sc
        if bi is not None:
            out[bo:bo + bs] = bi
    out.tofile(path)
    return plan


def write_bundle(root: str, num_layers: int = 2, seed: int = 0, expert_images=None, manifest_edit=None,
                 layout_edit=None, extra_names=("model.norm.weight",)):
    """Writes a bundle under `root`. expert_images(layer) -> uint8 array of the layer file, or
    None for a sparse file of the right size (enough for parsing). Returns the resident plan."""
    os.makedirs(os.path.join(root, "packed_experts"), exist_ok=True)
    entries = []
    for layer in range(num_layers):
        entries += layer_entries(layer, synth_resident_bytes(seed, layer))
    plan = write_resident(os.path.join(root, "resident.bin"), entries, extra_names)
    block, stride = expert_block()
    layers = []
    for layer in range(num_layers):
        fname = f"layer_{layer:02d}.bin"
        path = os.path.join(root, "packed_experts", fname)
        img = expert_images(layer) if expert_images else None
        if img is None:
            with open(path, "wb") as f:
                f.truncate(EXPERTS * stride)
        else:
            img.tofile(path)
        layers.append({"layer": layer, "file": fname})
    layout = {"expertStride": stride, "numLayers": num_layers, "expertsPerLayer": EXPERTS,
              "expertBlock": block, "layers": layers}
    manifest = {"magic": "GTURBO", "versionMajor": 1, "versionMinor": 0, "flags": {"streamingPresent": True},
                "modelId": "synthetic-gemma-4-26b-a4b-moe", "numLayers": num_layers, "expertsPerLayer": EXPERTS,
                "expertStride": stride,
                "arch": {"hiddenSize": HIDDEN, "ffnIntermediate": FFN, "moeIntermediateSize": MOE_INTER,
                         "numLayers": num_layers, "numExperts": EXPERTS, "topKExperts": 8, "rmsNormEps": 1e-6,
                         "fullAttentionLayerMask": [1 if i % 6 == 5 else 0 for i in range(num_layers)]},
                "files": {}}
    if layout_edit:
        layout_edit(layout)
    if manifest_edit:
        manifest_edit(manifest)
    with open(os.path.join(root, "packed_experts", "layout.json"), "w") as f:
        json.dump(layout, f, indent=2)
    with open(os.path.join(root, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=2)
    return plan


def quant_entry(name: str, m: dict):
    """An int4 MLX-affine tensor as the converter stores it: u32 words, shape [rows, in_dim / 8]."""
    return (name, U32, [m["rows"], m["in_dim"] // 8], np.ascontiguousarray(m["w"]).reshape(-1),
            np.ascontiguousarray(m["s"]).reshape(-1).view(np.uint8),
            np.ascontiguousarray(m["b"]).reshape(-1).view(np.uint8))


def bf16_entry(name: str, v: np.ndarray):
    return (name, BF16, [v.size], np.ascontiguousarray(v).reshape(-1).view(np.uint8), None, None)


def write_model_bundle(root: str, dec) -> None:
    """Writes the whole synthetic decoder `dec` (oracle.SynthDecoder) as a bundle the reference's
    CpuReference loads (src/cpu_reference.cpp:167-219): the MoE tensors of write_bundle, the
    attention tensors (full-attention layers without v_proj), the tied embedding and the final
    norm in resident.bin; each layer file sparse except for the experts the decoder has routed
    to (dec.used), which are the only blocks the reference reads when it routes the same way;
    the manifest's arch; and a minimal tokenizer whose stop pieces lie outside the vocabulary,
    so generation never stops early."""
    os.makedirs(os.path.join(root, "packed_experts"), exist_ok=True)
    os.makedirs(os.path.join(root, "tokenizer"), exist_ok=True)
    entries = [quant_entry("model.embed_tokens.weight", dec.embed_w), bf16_entry("model.norm.weight", dec.final_norm)]
    for l in range(dec.num_layers):
        P = f"model.layers.{l}."
        entries += layer_entries(l, synth_resident_bytes(dec.seed, l))
        a = dec.attn[l]
        entries += [quant_entry(P + "self_attn.q_proj.weight", a.q), quant_entry(P + "self_attn.k_proj.weight", a.k),
                    quant_entry(P + "self_attn.o_proj.weight", a.o),
                    bf16_entry(P + "self_attn.q_norm.weight", a.q_norm),
                    bf16_entry(P + "self_attn.k_norm.weight", a.k_norm),
                    bf16_entry(P + "input_layernorm.weight", a.input_norm),
                    bf16_entry(P + "post_attention_layernorm.weight", dec.post_attn[l])]
        if not dec.full_mask[l]:
            entries.append(quant_entry(P + "self_attn.v_proj.weight", a.v))
    write_resident(os.path.join(root, "resident.bin"), entries, extra_names=())
    block, stride = expert_block()
    layers = []
    buf = np.zeros(stride, np.uint8)
    for l in range(dec.num_layers):
        fname = f"layer_{l:02d}.bin"
        with open(os.path.join(root, "packed_experts", fname), "wb") as f:
            f.truncate(EXPERTS * stride)
            for e in sorted(dec.used[l]):
                buf[:] = 0
                oracle.lib().orc_synth_expert(C.c_uint64(dec.seed), l, e, HIDDEN, MOE_INTER,
                                              buf.ctypes.data_as(C.c_void_p))
                f.seek(e * stride)
                f.write(buf.tobytes())
        layers.append({"layer": l, "file": fname})
    layout = {"expertStride": stride, "numLayers": dec.num_layers, "expertsPerLayer": EXPERTS, "expertBlock": block,
              "layers": layers}
    arch = {"hiddenSize": HIDDEN, "ffnIntermediate": FFN, "moeIntermediateSize": MOE_INTER, "numHeads": 16,
            "numKVHeads": 8, "numFullKVHeads": 2, "headDim": 256, "fullHeadDim": 512, "vocabSize": dec.vocab,
            "slidingWindow": dec.window, "finalLogitSoftcap": dec.SOFTCAP, "ropeTheta": 10000.0,
            "fullRopeTheta": 1000000.0, "partialRotaryFactor": 0.25, "rmsNormEps": 1e-6,
            "numLayers": dec.num_layers, "numExperts": EXPERTS, "topKExperts": 8, "tieWordEmbeddings": True,
            "attentionKEqV": True, "hiddenActivation": "gelu_pytorch_tanh",
            "fullAttentionLayerMask": list(dec.full_mask)}
    manifest = {"magic": "GTURBO", "versionMajor": 1, "versionMinor": 0, "flags": {"streamingPresent": True},
                "modelId": "synthetic-gemma-4-26b-a4b", "numLayers": dec.num_layers, "expertsPerLayer": EXPERTS,
                "expertStride": stride, "arch": arch, "files": {}}
    with open(os.path.join(root, "packed_experts", "layout.json"), "w") as f:
        json.dump(layout, f, indent=2)
    with open(os.path.join(root, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=2)
    vocab = {"<eos>": dec.vocab + 1, "<turn|>": dec.vocab + 2, "<|tool_response>": dec.vocab + 3, "a": 3}
    with open(os.path.join(root, "tokenizer", "tokenizer.json"), "w") as f:
        json.dump({"model": {"type": "BPE", "vocab": vocab, "merges": []}}, f)

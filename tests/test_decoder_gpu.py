"""The whole decoder on the device (gtmoe.decoder.DeviceDecoder: embedding lookup, attention,
MoE block per layer, final norm, greedy LM head through the C ABI) against the reference's own
CpuReference::generate tokens on the same synthetic two- and three-layer models (tests/golden/decoder.npz,
pinned bit-exact to the composed CPU oracle by tests/test_decoder_oracle.py).

Bar: identical greedy tokens (north_star's bar for config 4); for sampled decoding identical
tokens with no draw flagged inside the double-exp bound.

"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "turbo-winfare_b200"), os.path.join(ROOT, "tests", "golden")]

import oracle  # noqa: E402
from make_golden import (BATCH_CASE, BATCH_NEW_TOKENS, DECODER_CASES, DECODER_NEW_TOKENS,  # noqa: E402
                         DECODER_SAMPLING, DECODER_STOPS)

pytestmark = pytest.mark.gpu


def device_decoder(args, prompts, batch: bool = False, new_tokens: int = DECODER_NEW_TOKENS):
    import torch
    import gtmoe
    from gtmoe.decoder import AttnLayerWeights, DeviceDecoder

    def quant(m):
        return {"w": torch.from_numpy(np.ascontiguousarray(m["w"])).cuda(),
                "s": torch.from_numpy(np.ascontiguousarray(m["s"]).view(np.int16)).cuda(),
                "b": torch.from_numpy(np.ascontiguousarray(m["b"]).view(np.int16)).cuda(),
                "rows": m["rows"], "in_dim": m["in_dim"]}

    def bf16(v):
        return torch.from_numpy(np.ascontiguousarray(v).view(np.int16)).cuda()

    dec = oracle.SynthDecoder(**args)
    layers = []
    for l in range(dec.num_layers):
        a, s = dec.attn[l], dec.attn[l].shape
        full = bool(dec.full_mask[l])
        layers.append(AttnLayerWeights(quant(a.q), quant(a.k), None if full else quant(a.v), quant(a.o),
                                       bf16(a.input_norm), bf16(a.q_norm), bf16(a.k_norm), bf16(dec.post_attn[l]),
                                       s.num_heads, s.kv_heads, s.head_dim, s.rotated_pairs, s.theta,
                                       0 if full else s.sliding_window))
    moe = gtmoe.SynthModel(dec.num_layers, seed=args["seed"])
    max_pos = max(len(p) for p in prompts) + new_tokens + 1
    if batch:
        from gtmoe.batch import BatchDecoder, LocalMoe
        return BatchDecoder(layers, LocalMoe(moe.layers, len(prompts)), quant(dec.embed_w), bf16(dec.final_norm),
                            max_pos, len(prompts)), moe
    return DeviceDecoder(layers, moe.layers, quant(dec.embed_w), bf16(dec.final_norm), max_pos), moe


@pytest.mark.parametrize("case", sorted(DECODER_CASES))
def test_greedy_tokens_match_reference(case):
    g = np.load(os.path.join(ROOT, "tests", "golden", "decoder.npz"))
    args, prompts = DECODER_CASES[case]
    dd, _moe = device_decoder(args, prompts)
    for i, p in enumerate(prompts):
        assert dd.greedy(p, DECODER_NEW_TOKENS, DECODER_STOPS) == g[f"{case}.prompt{i}.tokens"].tolist(), (case, i)


def test_sampled_tokens_match_reference():
    from gtmoe.sampling import SamplingParams
    g = np.load(os.path.join(ROOT, "tests", "golden", "decoder.npz"))
    args, prompts = DECODER_CASES["d3"]
    dd, _moe = device_decoder(args, prompts)
    for j, (t, tp, tk, pen, seed) in enumerate(DECODER_SAMPLING):
        sp = SamplingParams(t, tp, tk, pen, seed is not None, 0 if seed is None else seed)
        for i, p in enumerate(prompts):
            assert dd.sample(p, DECODER_NEW_TOKENS, sp, DECODER_STOPS) == g[f"d3.sampled{j}.prompt{i}.tokens"].tolist(), \
                (j, i)


def test_batched_greedy_64_tokens_match_reference():
    """BASELINE config 4's bar in miniature: four sequences of different prompt lengths decoded
    together (gtmoe.batch.BatchDecoder: attention per sequence, one gtm_moe_tokens call per layer
    for all the step's tokens, the greedy LM head per sequence); every sequence's 64 greedy ids
    equal the reference's own CpuReference::generate ids (tests/golden/batch_decode.npz)."""
    g = np.load(os.path.join(ROOT, "tests", "golden", "batch_decode.npz"))
    args, prompts = BATCH_CASE
    bd, _moe = device_decoder(args, prompts, batch=True, new_tokens=BATCH_NEW_TOKENS)
    got = bd.greedy(prompts, BATCH_NEW_TOKENS, DECODER_STOPS)
    for i in range(len(prompts)):
        assert got[i] == g[f"b4.prompt{i}.tokens"].tolist(), i


def test_single_sequence_64_tokens_match_reference():
    """The same bar through the single-sequence DeviceDecoder (the fused batch-1 decode per layer):
    sequence 0 of the batch case, 64 greedy ids."""
    g = np.load(os.path.join(ROOT, "tests", "golden", "batch_decode.npz"))
    args, prompts = BATCH_CASE
    dd, _moe = device_decoder(args, prompts, new_tokens=BATCH_NEW_TOKENS)
    assert dd.greedy(prompts[0], BATCH_NEW_TOKENS, DECODER_STOPS) == g["b4.prompt0.tokens"].tolist()

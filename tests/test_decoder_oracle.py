"""The whole decoder composed from the oracle's pieces (oracle.SynthDecoder: embedding, per layer
attention + MoE block, final norm, tied LM head, softcap, greedy) pinned to the reference's own
end-to-end generation path, CpuReference::load + generate (src/cpu_reference.cpp:167-219,
313-595), on synthetic bundles: two layers (sliding window 3, then full attention) and three
layers (full, sliding window 2, full).

Anchors:
* tests/golden/decoder.npz: the reference's greedy tokens for each prompt and SHA-256 digests
  of every stage it dumps for the first prompt token (embed, each layerN_hidden, final_norm,
  logits), replayed here without the reference tree;
* live: the bundle is written (tests/bundle_writer.py) and the compiled reference generates on
  it, when oracle/_ref is built.

This is the oracle for end-to-end greedy decode (config 4); the stage digests are bit-exact, the
tokens after the first prompt token are compared as tokens. Sampled generation (the reference's
softcap, repetition penalty, Top-P then Top-K then temperature, per-position seeds) is pinned the
same way on the three-layer case.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "tests"), os.path.join(ROOT, "tests", "golden")]

import oracle  # noqa: E402
from make_golden import DECODER_CASES, DECODER_NEW_TOKENS, DECODER_SAMPLING, DECODER_STOPS, digest  # noqa: E402

needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built (reference tree absent)")


def stages(n_layers: int) -> list[str]:
    return ["embed"] + [f"layer{l}_hidden" for l in range(n_layers)] + ["final_norm", "logits"]


@pytest.fixture(scope="module", params=sorted(DECODER_CASES))
def runs(request):
    """The oracle's greedy run and first-token stages for each prompt of one decoder case."""
    args, prompts = DECODER_CASES[request.param]
    dec = oracle.SynthDecoder(**args)
    out = []
    for p in prompts:
        trace = {}
        toks = dec.greedy(p, DECODER_NEW_TOKENS, DECODER_STOPS, trace=trace)
        out.append((toks, trace))
    return request.param, dec, prompts, out


def test_matches_reference_golden(runs):
    g = np.load(os.path.join(ROOT, "tests", "golden", "decoder.npz"))
    case, dec, _, out = runs
    for i, (toks, trace) in enumerate(out):
        assert toks == g[f"{case}.prompt{i}.tokens"].tolist(), (case, i)
        for name in stages(dec.num_layers):
            assert np.array_equal(digest(trace[name]), g[f"{case}.prompt{i}.{name}.sha256"]), (case, i, name)


def test_stages_are_not_degenerate(runs):
    _, dec, _, out = runs
    for toks, trace in out:
        assert len(toks) == DECODER_NEW_TOKENS
        assert np.all(np.isfinite(trace["logits"])) and np.abs(trace["logits"]).max() <= 30.0
        assert trace["logits"].std() > 0.05           # the LM head separates tokens
        assert not np.array_equal(trace["embed"], trace[f"layer{dec.num_layers - 1}_hidden"])


@needs_ref
def test_live_against_reference_generate(runs, tmp_path):
    import bundle_writer as bw
    _, dec, prompts, out = runs
    bw.write_model_bundle(str(tmp_path), dec)
    for i, (p, (toks, trace)) in enumerate(zip(prompts, out)):
        dd = tmp_path / f"dump{i}"
        assert oracle.ref_generate(str(tmp_path), p, DECODER_NEW_TOKENS, str(dd)) == toks, i
        for name in stages(dec.num_layers):
            ref = np.fromfile(dd / (name + ".f32"), np.float32)
            assert np.array_equal(ref.view(np.uint32), trace[name].view(np.uint32)), (i, name)


@pytest.fixture(scope="module")
def sampled():
    args, prompts = DECODER_CASES["d3"]
    dec = oracle.SynthDecoder(**args)
    runs = [[dec.sample(p, DECODER_NEW_TOKENS, oracle.sampling_params(t, tp, tk, pen, seed=seed), DECODER_STOPS)
             for p in prompts] for t, tp, tk, pen, seed in DECODER_SAMPLING]
    return dec, prompts, runs


def test_sampled_matches_reference_golden(sampled):
    g = np.load(os.path.join(ROOT, "tests", "golden", "decoder.npz"))
    _, _, runs = sampled
    for j, per_prompt in enumerate(runs):
        for i, toks in enumerate(per_prompt):
            assert toks == g[f"d3.sampled{j}.prompt{i}.tokens"].tolist(), (j, i)
    assert len({t for per_prompt in runs for toks in per_prompt for t in toks}) > 10   # not a fixed point


@needs_ref
def test_sampled_live_against_reference_generate(sampled, tmp_path):
    import bundle_writer as bw
    dec, prompts, runs = sampled
    bw.write_model_bundle(str(tmp_path), dec)
    for (t, tp, tk, pen, seed), per_prompt in zip(DECODER_SAMPLING, runs):
        sp = oracle.sampling_params(t, tp, tk, pen, seed=seed)
        for p, toks in zip(prompts, per_prompt):
            assert oracle.ref_generate(str(tmp_path), p, DECODER_NEW_TOKENS, None, sp) == toks

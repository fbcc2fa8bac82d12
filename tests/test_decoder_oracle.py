"""The whole decoder composed from the oracle's pieces (oracle.SynthDecoder: embedding, per layer
attention + MoE block, final norm, tied LM head, softcap, greedy) pinned to the reference's own
end-to-end generation path, CpuReference::load + generate (src/cpu_reference.cpp:167-219,
313-595), on a synthetic two-layer bundle (a sliding-window layer with window 3 and a
full-attention layer).

Anchors:
* tests/golden/decoder.npz: the reference's greedy tokens for three prompts and SHA-256 digests
  of every stage it dumps for the first prompt token (embed, layer0_hidden, layer1_hidden,
  final_norm, logits), replayed here without the reference tree;
* live: the bundle is written (tests/bundle_writer.py) and the compiled reference generates on
  it, when oracle/_ref is built.

This is the oracle for end-to-end greedy decode (config 4); the stage digests are bit-exact, the
tokens after the first prompt token are compared as tokens.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "tests"), os.path.join(ROOT, "tests", "golden")]

import oracle  # noqa: E402
from make_golden import DECODER, DECODER_NEW_TOKENS, DECODER_PROMPTS, DECODER_STOPS, digest  # noqa: E402

STAGES = ("embed", "layer0_hidden", "layer1_hidden", "final_norm", "logits")
needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built (reference tree absent)")


@pytest.fixture(scope="module")
def runs():
    """The oracle's greedy run and first-token stages for each prompt."""
    dec = oracle.SynthDecoder(**DECODER)
    out = []
    for p in DECODER_PROMPTS:
        trace = {}
        toks = dec.greedy(p, DECODER_NEW_TOKENS, DECODER_STOPS, trace=trace)
        out.append((toks, trace))
    return dec, out


def test_matches_reference_golden(runs):
    g = np.load(os.path.join(ROOT, "tests", "golden", "decoder.npz"))
    _, out = runs
    for i, (toks, trace) in enumerate(out):
        assert toks == g[f"prompt{i}.tokens"].tolist(), i
        for name in STAGES:
            assert np.array_equal(digest(trace[name]), g[f"prompt{i}.{name}.sha256"]), (i, name)


def test_stages_are_not_degenerate(runs):
    _, out = runs
    for toks, trace in out:
        assert len(toks) == DECODER_NEW_TOKENS
        assert np.all(np.isfinite(trace["logits"])) and np.abs(trace["logits"]).max() <= 30.0
        assert trace["logits"].std() > 0.05           # the LM head separates tokens
        assert not np.array_equal(trace["embed"], trace["layer1_hidden"])


@needs_ref
def test_live_against_reference_generate(runs, tmp_path):
    import bundle_writer as bw
    dec, out = runs
    bw.write_model_bundle(str(tmp_path), dec)
    for i, (p, (toks, trace)) in enumerate(zip(DECODER_PROMPTS, out)):
        dd = tmp_path / f"dump{i}"
        assert oracle.ref_generate(str(tmp_path), p, DECODER_NEW_TOKENS, str(dd)) == toks, i
        for name in STAGES:
            ref = np.fromfile(dd / (name + ".f32"), np.float32)
            assert np.array_equal(ref.view(np.uint32), trace[name].view(np.uint32)), (i, name)

"""Device sampling (gtm_sample_token, gtm_repetition_penalty) against the reference's compiled
sampling.cpp outputs (tests/golden/sampling.npz) and the pinned sampling oracle.

Bar: identical tokens and bit-identical penalised logits; a draw whose status reports a decision
inside the double-exp error bound (NEAR_CUT / NEAR_DRAW) is counted, and none is expected on
these inputs.

"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "turbo-winfare_b200")]

import oracle  # noqa: E402

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(ROOT, "tests", "golden", "sampling.npz")


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN)


def logits_of(g, prefix: str) -> np.ndarray:
    if prefix + ".synth" in g:
        seed, vocab, scale, step = g[prefix + ".synth"]
        return oracle.synth_logits(int(seed), int(vocab), float(scale), float(step))
    return g[prefix + ".logits"]


def sp(t, tp, tk, pen=1.0):
    from gtmoe import sampling
    return sampling.SamplingParams(float(t), float(tp), int(tk), float(pen))


def device_draw(smp, dev_logits, p, seed):
    out = smp.sample_token(dev_logits, p, seed).cpu().numpy().view(np.uint32)
    return int(out[0]), int(out[1])


def test_draws_match_reference(g):
    import torch
    from gtmoe import sampling
    for c in range(int(g["draw.n"][0])):
        logits = logits_of(g, f"draw{c}")
        t, tp, tk = g[f"draw{c}.params"]
        p = sp(t, tp, tk)
        smp = sampling.Sampler(logits.size)
        dev = torch.from_numpy(logits).cuda()
        for s, rc, tok in zip(g[f"draw{c}.seeds"], g[f"draw{c}.rc"], g[f"draw{c}.token"]):
            got, st = device_draw(smp, dev, p, int(s))
            if rc != 0:
                assert st & sampling.DEGENERATE, (c, st)
                continue
            assert st == 0, (c, int(s), st)
            assert got == int(tok), (c, int(s), got, int(tok))


def test_penalty_matches_reference(g):
    import torch
    from gtmoe import sampling
    for c in range(int(g["penalty.n"][0])):
        logits = logits_of(g, f"penalty{c}")
        pen, cap = (float(v) for v in g[f"penalty{c}.args"])
        hist = g[f"penalty{c}.history"].astype(np.int32)
        smp = sampling.Sampler(logits.size)
        dev = torch.from_numpy(logits.copy()).cuda()
        smp.apply_repetition_penalty(dev, torch.from_numpy(hist).cuda() if hist.size else None, pen, cap)
        got = dev.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), g[f"penalty{c}.out"].view(np.uint32)), c


@pytest.mark.parametrize("in_place", [False, True])
def test_softcap_known_answer(in_place):
    """Within the rule the reference holds its own GPU Softcap to (allclose 1e-5 + 1e-4 |want|):
    device tanhf rounds differently from the C library's."""
    import torch
    from gtmoe import sampling
    k = np.load(os.path.join(ROOT, "tests", "golden", "kat.npz"))
    z = torch.from_numpy(k["softcap.z"].copy()).cuda()
    out = z if in_place else torch.empty_like(z)
    sampling.softcap(z, 30.0, out=out)
    got, want = out.cpu().numpy(), k["softcap.want"]
    assert np.all(np.abs(got - want) <= 1e-5 + 1e-4 * np.abs(want))


@pytest.mark.parametrize("vocab", [1, 2, 255, 256, 257, 5000, 262144, 1 << 20])
def test_random_against_oracle(vocab):
    import torch
    from gtmoe import sampling
    rng = np.random.default_rng(vocab)
    smp = sampling.Sampler(vocab)
    near = 0
    for trial in range(6):
        logits = oracle.synth_logits(300 + trial, vocab, float(rng.uniform(0.5, 10.0)), float(rng.choice([0.0, 0.5])))
        dev = torch.from_numpy(logits).cuda()
        for t, tp, tk in ((0.0, 1.0, 0), (0.7, 1.0, 0), (1.0, 0.9, 40), (0.3, 0.99, 256), (2.0, 1.0, 1)):
            p = sp(t, tp, tk)
            po = oracle.sampling_params(t, tp, tk)
            for i in range(4):
                seed = oracle.seed_for(oracle.sampling_params(t, tp, tk, seed=trial), i)
                got, st = device_draw(smp, dev, p, seed)
                rc, want = oracle.sample_token(logits, po, seed)
                assert rc == 0 and not (st & sampling.DEGENERATE)
                if st:
                    near += 1
                    continue
                assert got == want, (vocab, trial, t, tp, tk, i, got, want)
    assert near == 0


def test_penalty_repeats_against_oracle():
    import torch
    from gtmoe import sampling
    rng = np.random.default_rng(11)
    vocab = 262144
    smp = sampling.Sampler(vocab)
    for trial in range(4):
        logits = oracle.synth_logits(400 + trial, vocab, 25.0)
        hist = rng.integers(0, vocab + 1000, size=4096).astype(np.int64)
        hist[::7] = hist[0]   # one id repeated hundreds of times
        pen, cap = float(rng.choice([0.5, 1.1, 1.3])), float(rng.choice([0.0, 30.0]))
        want = oracle.apply_repetition_penalty(logits, hist, pen, cap)
        dev = torch.from_numpy(logits.copy()).cuda()
        smp.apply_repetition_penalty(dev, torch.from_numpy(hist.astype(np.int32)).cuda(), pen, cap)
        assert np.array_equal(dev.cpu().numpy().view(np.uint32), want.view(np.uint32)), trial


def test_timing_full_vocabulary():
    import torch
    from gtmoe import sampling
    vocab = 262144
    smp = sampling.Sampler(vocab)
    dev = torch.from_numpy(oracle.synth_logits(1, vocab, 6.0)).cuda()
    p = sp(0.8, 0.95, 64)
    for i in range(5):
        smp.sample_token(dev, p, i + 1)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(100):
        smp.sample_token(dev, p, i + 1)
    e1.record()
    torch.cuda.synchronize()
    print(f"\nsample_token V={vocab}: {e0.elapsed_time(e1) * 10:.1f} us per token (two launches)")

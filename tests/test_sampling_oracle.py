"""Token sampling oracle (oracle/sampling_oracle.c) pinned to the reference's src/sampling.cpp.

Three anchors:
* tests/golden/sampling.npz -- outputs of the reference's own compiled sampling.cpp
  (tests/golden/make_golden.py), replayed here without the reference tree;
* the assertions of the reference's tests/test_sampling.cpp, restated: splitmix64 vectors,
  validation outcomes, greedy ties, truncation order (Top-P over the full distribution, then
  Top-K), determinism, and the repetition-penalty numbers;
* live comparisons with oracle/_ref/libgtref.so when it is built.

The oracle is the checker for a device sampler; nothing here runs on a GPU.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

GOLDEN = os.path.join(ROOT, "tests", "golden", "sampling.npz")
needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built (reference tree absent)")


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN)


def logits_of(g, prefix: str) -> np.ndarray:
    if prefix + ".synth" in g:
        seed, vocab, scale, step = g[prefix + ".synth"]
        return oracle.synth_logits(int(seed), int(vocab), float(scale), float(step))
    return g[prefix + ".logits"]


def params(t, tp, tk, pen=1.0, seed=None):
    return oracle.sampling_params(float(t), float(tp), int(tk), float(pen), seed=seed)


# ---- against the reference's compiled outputs ----------------------------------------------

def test_splitmix64_golden(g):
    for x, want in zip(g["splitmix.in"], g["splitmix.out"]):
        assert oracle.splitmix64(int(x)) == int(want)


def test_seed_for_golden(g):
    for has, seed, pos, want in zip(g["seed.has"], g["seed.seed"], g["seed.pos"], g["seed.out"]):
        p = params(0.7, 1.0, 0, seed=int(seed) if has else None)
        got = oracle.seed_for(p, int(pos))
        assert got == int(want) and got != 0


def test_validation_golden(g):
    for (t, tp, tk, pen), rej in zip(g["validate.params"], g["validate.rejects"]):
        rc = oracle.validate_sampling(params(t, tp, tk, pen))
        assert (rc != 0) == bool(rej), (t, tp, tk, pen, rc)


def test_repetition_penalty_golden(g):
    for c in range(int(g["penalty.n"][0])):
        pen, cap = g[f"penalty{c}.args"]
        got = oracle.apply_repetition_penalty(logits_of(g, f"penalty{c}"), g[f"penalty{c}.history"], float(pen),
                                              float(cap))
        want = g[f"penalty{c}.out"]
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), c   # bit-exact, NaN and -0 included


def test_draws_golden(g):
    for c in range(int(g["draw.n"][0])):
        logits = logits_of(g, f"draw{c}")
        t, tp, tk = g[f"draw{c}.params"]
        p = params(t, tp, tk)
        for s, rc, tok in zip(g[f"draw{c}.seeds"], g[f"draw{c}.rc"], g[f"draw{c}.token"]):
            got_rc, got = oracle.sample_token(logits, p, int(s))
            assert (got_rc != 0) == (rc != 0), (c, got_rc, rc)
            assert got == int(tok), (c, int(s), got, int(tok))


# ---- the reference's own test assertions (tests/test_sampling.cpp), restated ------------------

def test_splitmix64_known_answers():
    # tests/test_sampling.cpp:118-121
    assert oracle.splitmix64(0) == 0xE220A8397B1DCDAF
    assert oracle.splitmix64(1) == 0x910A2DEC89025CC1
    assert oracle.splitmix64(2) == 0x975835DE1C9756CE
    assert oracle.splitmix64(3) == 0x1D0B14E4DB018FED


def test_validation_rules():
    # tests/test_sampling.cpp:94-110
    ok = [(0.2, 0.95, 64, 1.0), (0.0, 1.0, 0, 1.0), (0.7, 1.0, 0, 1.0), (0.0, 0.9, 0, 1.0)]
    bad = {(-0.1, 1.0, 0, 1.0): 1, (0.2, 0.0, 64, 1.0): 2, (0.2, 1.5, 64, 1.0): 2, (0.2, 0.95, 257, 1.0): 3,
           (0.2, 0.95, -1, 1.0): 3, (0.2, 0.95, 64, 0.0): 4, (0.7, 0.9, 0, 1.0): 5}
    for c in ok:
        assert oracle.validate_sampling(params(*c)) == 0, c
    for c, rule in bad.items():
        assert oracle.validate_sampling(params(*c)) == rule, c


def test_seed_for_stable_nonzero_and_decorrelated():
    # tests/test_sampling.cpp:123-135
    p = params(0.7, 1.0, 0, seed=12345)
    vals = [oracle.seed_for(p, pos) for pos in range(10000)]
    assert all(v != 0 for v in vals)
    assert vals[5] == oracle.seed_for(p, 5)
    assert vals[0] != vals[1]
    assert oracle.seed_for(p, 5) != oracle.seed_for(params(0.7, 1.0, 0, seed=99), 5)


def test_greedy_ties_to_lower_index():
    # tests/test_sampling.cpp:141-147
    greedy = params(0.0, 1.0, 0)
    assert oracle.sample_token(np.array([1, 5, 3, 5, 2], np.float32), greedy, 1) == (0, 1)
    assert oracle.sample_token(np.array([7], np.float32), greedy, 1) == (0, 0)


def test_truncation_order_nucleus_then_top_k():
    # tests/test_sampling.cpp:160-171: with top_p 0.9 then top_k 2, ids 0 and 1 are both reachable
    logits = np.array([3.0, 2.5, 2.0, 1.5, -1.0, -2.0, -3.0, -4.0], np.float32)
    p = params(1.0, 0.9, 2, seed=7)
    seen = {oracle.sample_token(logits, p, oracle.seed_for(p, i))[1] for i in range(4000)}
    assert seen == {0, 1}
    rc, ids, cut = oracle.sample_shortlist(logits, p)
    # the shortlist holds top_k ids when top_k > 0; their true mass (~0.72) never reaches 0.9
    assert rc == 0 and list(ids) == [0, 1] and cut == 2


def test_same_seed_reproduces_other_seed_diverges():
    # tests/test_sampling.cpp:176-193 (logits from this repository's generator)
    logits = oracle.synth_logits(4242, 4096, 4.0)
    p, q = params(0.8, 0.95, 64, seed=20260721), params(0.8, 0.95, 64, seed=20260722)
    first = [oracle.sample_token(logits, p, oracle.seed_for(p, i))[1] for i in range(64)]
    second = [oracle.sample_token(logits, p, oracle.seed_for(p, i))[1] for i in range(64)]
    third = [oracle.sample_token(logits, q, oracle.seed_for(q, i))[1] for i in range(64)]
    assert first == second and first != third


def test_repetition_penalty_rules():
    # tests/test_sampling.cpp:198-229
    logits = np.array([10.0, -10.0, 0.0, 29.999], np.float32)
    hist = [0, 1, 3, 99999]
    v = oracle.apply_repetition_penalty(logits, hist, 2.0, 30.0)
    assert abs(v[0] - 5.0) < 1e-5 and abs(v[1] + 20.0) < 1e-5 and v[2] == 0.0 and 14.9 < v[3] < 15.1
    assert np.all(np.abs(v) <= 30.0)
    assert np.array_equal(oracle.apply_repetition_penalty(logits, hist, 1.0, 30.0), logits)
    assert np.array_equal(oracle.apply_repetition_penalty(logits, [], 2.0, 30.0), logits)
    gl = np.array([9.0, 8.0], np.float32)
    greedy = params(0.0, 1.0, 0)
    assert oracle.sample_token(gl, greedy, 1)[1] == 0
    assert oracle.sample_token(oracle.apply_repetition_penalty(gl, [0], 2.0, 30.0), greedy, 1)[1] == 1


def test_shortlist_matches_full_sort():
    # tests/test_sampling.cpp:236-266 guards the partial selection with a full sort; here the
    # oracle's shortlist is checked against numpy's lexsort on (logit desc, id asc), ties included
    for seed, step in ((7, 0.0), (8, 0.25), (13, 1.0)):
        logits = oracle.synth_logits(seed, 262144, 6.0, step)
        order = np.lexsort((np.arange(logits.size), -logits.astype(np.float64)))
        for tk in (0, 1, 8, 64, 256):
            rc, ids, cut = oracle.sample_shortlist(logits, params(1.0, 1.0, tk))
            n = tk if tk > 0 else 256
            assert rc == 0 and np.array_equal(ids, order[:n].astype(np.uint32)), (seed, step, tk)
            assert cut == n


def test_softcap_known_answer():
    # the reference's Softcap case (tests/test_gpu_kernels.cpp:389-411), regenerated into kat.npz
    k = np.load(os.path.join(ROOT, "tests", "golden", "kat.npz"))
    got = oracle.softcap(k["softcap.z"], 30.0)
    assert np.array_equal(got.view(np.uint32), k["softcap.want"].view(np.uint32))
    assert np.all(np.abs(got) <= 30.0)


def test_failures():
    p = params(1.0, 1.0, 0)
    assert oracle.sample_token(np.zeros(0, np.float32), p, 1)[0] == 1            # empty vocabulary
    assert oracle.sample_token(np.zeros(0, np.float32), params(0.0, 1.0, 0), 1)[0] == 1
    assert oracle.sample_token(np.full(5, -np.inf, np.float32), p, 1)[0] == 2   # degenerate
    assert oracle.sample_token(np.array([0, np.inf], np.float32), p, 1)[0] == 2


# ---- live against the compiled reference ---------------------------------------------------

@needs_ref
def test_live_draws_against_reference():
    rng = np.random.default_rng(5)
    for trial in range(24):
        vocab = int(rng.choice([2, 17, 255, 256, 257, 3000, 65536]))
        step = float(rng.choice([0.0, 0.0, 0.5]))
        logits = oracle.synth_logits(100 + trial, vocab, float(rng.uniform(0.5, 10.0)), step)
        t = float(rng.choice([0.0, 0.05, 0.7, 1.0, 3.0]))
        tk = int(rng.choice([0, 1, 3, 40, 256]))
        tp = float(rng.choice([1.0, 0.5, 0.9, 0.999])) if tk > 0 else 1.0
        p = params(t, tp, tk, seed=trial)
        assert oracle.validate_sampling(p) == 0
        for i in range(20):
            s = oracle.seed_for(p, i)
            assert s == oracle.seed_for(p, i, impl="ref")
            assert oracle.sample_token(logits, p, s) == oracle.sample_token(logits, p, s, impl="ref"), (trial, i)


@needs_ref
def test_live_penalty_against_reference():
    rng = np.random.default_rng(6)
    for trial in range(20):
        vocab = int(rng.integers(1, 500))
        logits = oracle.synth_logits(200 + trial, vocab, 25.0)
        hist = rng.integers(0, vocab + 5, size=int(rng.integers(0, 300)))
        pen = float(rng.choice([0.5, 1.0, 1.1, 1.3, 2.0]))
        cap = float(rng.choice([0.0, 30.0]))
        a = oracle.apply_repetition_penalty(logits, hist, pen, cap)
        b = oracle.apply_repetition_penalty(logits, hist, pen, cap, impl="ref")
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), trial

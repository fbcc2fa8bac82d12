"""A numpy model of the device sampler's arithmetic (csrc/gtm_sampling.cu) against the reference's
draws (tests/golden/sampling.npz).

The model follows the kernels' plan, not the reference's order: the vocabulary is cut into the
same slices (one per SM, at most 4096 ids), each slice's exp sum is taken relative to its own max
and rescaled to the global max, sums are pairwise, and exp is numpy's rather than the C
library's. The shortlist, the nucleus cut against that denominator, the top-k cut, the
temperature weights, the xorshift64* draw and the near-decision tolerances are as in smp_finish.
Every golden draw must come out identical with no decision inside the tolerance: evidence that
the device's different summation order does not move a token on these inputs.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "tests")]

from test_sampling_oracle import GOLDEN, logits_of  # noqa: E402


MASK64 = (1 << 64) - 1


def model(logits: np.ndarray, t: float, tp: float, tk: int, seed: int, sms: int = 148) -> tuple[int, int]:
    """(token, status bits) as the device computes them, for temperature t, top_p tp, top_k tk."""
    V = logits.size
    if t <= 0:   # greedy: the best (logit desc, id asc) key
        return int(np.lexsort((np.arange(V), -logits.astype(np.float64)))[0]), 0
    mx = float(logits.max())
    if not np.isfinite(mx):
        return -1, 1
    # smp_scan's slices and their rescaled exp sums
    g0 = max(1, min(sms, -(-V // 256)))
    chunk = min(-(-V // g0), 4096)
    total = 0.0
    for c in range(-(-V // chunk)):
        sl = logits[c * chunk:(c + 1) * chunk].astype(np.float64)
        mc = sl.max()
        if mc == -np.inf:
            continue
        total += float(np.exp(sl - mc).sum()) * float(np.exp(mc - mx))
    # smp_finish: shortlist, nucleus cut, top-k cut, temperature weights, one draw
    want = min(tk if tk > 0 else 256, V)
    order = np.lexsort((np.arange(V), -logits.astype(np.float64)))[:want]
    lv = logits[order].astype(np.float64)
    ev = np.exp(lv - mx)
    qv = np.exp((lv - mx) / np.float64(np.float32(t)))
    st, cut = 0, want
    if tp < 1:
        tpd = float(np.float32(tp))
        tol = (V + 4 * want) * 2.0 ** -52 * tpd
        run = 0.0
        for i in range(want):
            run += ev[i] / total
            if abs(run - tpd) <= tol:
                st |= 2
            if run >= tpd:
                cut = i + 1
                break
    if tk > 0:
        cut = min(cut, tk)
    cut = max(cut, 1)
    denom = 0.0
    for i in range(cut):
        denom += qv[i]
    s = seed
    s ^= s >> 12
    s = (s ^ (s << 25)) & MASK64
    s ^= s >> 27
    r64 = (s * 0x2545F4914F6CDD1D) & MASK64
    u = np.float32((r64 >> 40) & 0xFFFFFF) * np.float32(2.0 ** -24)
    r = float(u) * denom
    tol2 = 4 * (cut + 2) * 2.0 ** -52 * denom
    acc, tok = 0.0, int(order[cut - 1])
    for i in range(cut):
        acc += qv[i]
        if abs(acc - r) <= tol2:
            st |= 4
        if acc >= r:
            tok = int(order[i])
            break
    return tok, st


def test_model_reproduces_reference_draws():
    g = np.load(GOLDEN)
    mismatches = flagged = 0
    for c in range(int(g["draw.n"][0])):
        logits = logits_of(g, f"draw{c}")
        t, tp, tk = (float(v) for v in g[f"draw{c}.params"])
        for s, rc, tok in zip(g[f"draw{c}.seeds"], g[f"draw{c}.rc"], g[f"draw{c}.token"]):
            got, st = model(logits, t, tp, int(tk), int(s))
            if rc != 0:
                assert st & 1, c
                continue
            flagged += st != 0
            mismatches += got != int(tok)
    assert mismatches == 0 and flagged == 0

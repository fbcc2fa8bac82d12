"""Pins the float64 whole-batch block (tests/block_f64.py) to the exact CPU oracle on the host, so
the GPU tests that check every token of a 4096-token batch against it rest on a checked
restatement. Runs on the CPU: the synthetic layer's byte images come from the oracle's own
generator and the offsets from the library's layout descriptor (pointer arithmetic only)."""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "turbo-winfare_b200"), os.path.join(ROOT, "tests")]

torch = pytest.importorskip("torch")

import gtmoe  # noqa: E402
import oracle  # noqa: E402
from block_f64 import block_f64, max_rel  # noqa: E402
from gtmoe import workloads  # noqa: E402


def host_layer(seed: int, layer: int, experts: list[int]):
    """(gtmoe.Layer, resident uint8 tensor, expert image uint8 tensor) on the host."""
    roff, rtotal = gtmoe.resident_layout()
    _, stride = gtmoe.expert_layout()
    res = np.zeros(rtotal, np.uint8)
    oracle.lib().orc_synth_resident(seed, layer, gtmoe.HIDDEN, gtmoe.FFN, gtmoe.EXPERTS, res.ctypes.data)
    img = np.zeros(gtmoe.EXPERTS * stride, np.uint8)
    for e in experts:
        oracle.lib().orc_synth_expert(seed, layer, e, gtmoe.HIDDEN, gtmoe.MOE_INTER,
                                      img[e * stride:].ctypes.data)
    L = gtmoe.Layer()
    gtmoe.check(gtmoe.lib().gtm_synth_layer_desc(gtmoe.HIDDEN, gtmoe.MOE_INTER, gtmoe.FFN, gtmoe.EXPERTS,
                                                 C.c_void_p(res.ctypes.data), C.c_void_p(img.ctypes.data),
                                                 C.byref(L)))
    return L, torch.from_numpy(res), torch.from_numpy(img)


def test_block_f64_matches_oracle_on_synthetic_tokens():
    T = 6
    ref_layer = oracle.SynthLayer(0, 0)
    rl = workloads.uniform_route_logits(T, seed=5)
    xs = np.stack([oracle.synth_x(0, 300 + t) for t in range(T)])
    refs = [ref_layer.block(xs[t], route_logits=rl[t]) for t in range(T)]
    idx = np.stack([r["idx"] for r in refs]).astype(np.int64)
    w = np.stack([r["w"] for r in refs])
    L, res, img = host_layer(0, 0, sorted(set(idx.reshape(-1).tolist())))
    got = block_f64(L, res, img, torch.from_numpy(xs), torch.from_numpy(idx), torch.from_numpy(w))
    for k in ("h1", "h2", "hidden"):
        want = torch.from_numpy(np.stack([r[k] for r in refs]))
        err = max_rel(want, got[k])
        # the oracle is float32 with the reference's rounding; float64 differs by rounding only
        assert err < 2e-5, (k, err)

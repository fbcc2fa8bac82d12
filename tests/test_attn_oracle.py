"""Decoder-remainder oracle (oracle/attn_oracle.c): embedding lookup, QKV epilogue, attention
core and one full attention step, pinned to the reference.

Anchors:
* the known answers of the reference's tests/test_gpu_kernels.cpp, regenerated from its
  mt19937(12345) stream by oracle/kat_gen.cpp (tests/golden/kat.npz): EmbedLookup row 37
  (:268-292), QKVEpilogue with partial rotary (:649-692), Attention GQA 16/8 window 128
  (:694-741) and Attention across the ring wrap (:804-858). The attention cases' K/V caches are
  drawn again here from the stored generator state;
* digests of one layer run position by position through the reference's own compiled helpers
  (tests/golden/attn_steps.npz);
* live comparisons with oracle/_ref/libgtref.so when it is built.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "tests", "golden")]

import oracle  # noqa: E402
from make_golden import ATTN_CASES, digest  # noqa: E402

needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built (reference tree absent)")


@pytest.fixture(scope="module")
def kat():
    return np.load(os.path.join(ROOT, "tests", "golden", "kat.npz"))


def bits_equal(a, b) -> bool:
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def uniform_stream(state: np.ndarray, n: int) -> np.ndarray:
    """std::uniform_real_distribution<float>(-1.5, 1.5) over std::mt19937 from a saved state:
    libstdc++ draws one 32-bit word per float, u = float(word) / 2^32 (kept below 1), then
    u * 3 + (-1.5), all in float."""
    bg = np.random.MT19937()
    bg.state = {"bit_generator": "MT19937", "state": {"key": state[:624].astype(np.uint32), "pos": int(state[624])}}
    u = bg.random_raw(n).astype(np.float32) / np.float32(4294967296.0)
    u = np.where(u >= np.float32(1.0), np.nextafter(np.float32(1.0), np.float32(0.0)), u).astype(np.float32)
    return (u * np.float32(3.0) + np.float32(-1.5)).astype(np.float32)


def test_embed_known_answer(kat):
    rows, in_dim, bits = (int(v) for v in kat["embed.shape"])
    m = {"w": kat["embed.w"].reshape(rows, in_dim // 2), "s": kat["embed.s"], "b": kat["embed.b"], "rows": rows,
         "in_dim": in_dim}
    assert bits_equal(oracle.embed(m, int(kat["embed.token"][0])), kat["embed.want"])


def test_qkv_epilogue_known_answer(kat):
    head_dim, heads, rotated, position = (int(v) for v in kat["qkv.shape"])
    got = oracle.qkv_epilogue(kat["qkv.vec"], heads, head_dim, kat["qkv.w"], 1e-6, rotated, float(position), 1e6)
    assert bits_equal(got, kat["qkv.want"])


@pytest.mark.parametrize("case", ["attn", "attn_ring"])
def test_attention_known_answer(kat, case):
    q_heads, kv_heads, head_dim, n_pos, window, capacity = (int(v) for v in kat[case + ".shape"])
    nq, nkv = q_heads * head_dim, capacity * kv_heads * head_dim
    xs = uniform_stream(kat[case + ".rng_state"], nq + 2 * nkv)
    q = (xs[:nq] * np.float32(0.1)).astype(np.float32)
    assert bits_equal(q, kat[case + ".q"])   # the replayed stream is the test's stream
    kc = (xs[nq:nq + nkv] * np.float32(0.1)).astype(np.float32)
    vc = xs[nq + nkv:]
    got = oracle.attention_core(q, kc, vc, q_heads, kv_heads, head_dim, n_pos, n_pos - window, capacity)
    assert bits_equal(got, kat[case + ".want"])


def test_attention_steps_golden():
    g = np.load(os.path.join(ROOT, "tests", "golden", "attn_steps.npz"))
    for name, full, win, n, seed in ATTN_CASES:
        w = oracle.AttnWeights(seed, oracle.attn_shape(full, sliding_window=win or 1024))
        xs = np.stack([oracle.synth_x(seed, t) for t in range(n)])
        r = oracle.attention_steps(w, xs)
        assert bits_equal(r["attn"][-1], g[f"{name}.attn_last"]), name
        for k in ("attn", "q", "k", "v"):
            assert np.array_equal(digest(r[k]), g[f"{name}.{k}.sha256"]), (name, k)


def test_window_and_shape_rules():
    swa, full = oracle.attn_shape(False), oracle.attn_shape(True)
    assert (swa.head_dim, swa.kv_heads, swa.rotated_pairs, swa.sliding_window, swa.k_eq_v) == (256, 8, 128, 1024, 0)
    assert (full.head_dim, full.kv_heads, full.rotated_pairs, full.sliding_window, full.k_eq_v) == (512, 2, 64, 0, 1)
    # a window of 1 attends to the current position only: softmax weight 1 on its own V row
    s = oracle.attn_shape(False, sliding_window=1)
    w = oracle.AttnWeights(5, s)
    xs = np.stack([oracle.synth_x(5, t) for t in range(3)])
    r = oracle.attention_steps(w, xs)
    ctx = oracle.attention_core(r["q"][-1], r["k_cache"], r["v_cache"], s.num_heads, s.kv_heads, s.head_dim, 3, 2, 3)
    gqa = s.num_heads // s.kv_heads
    want = np.concatenate([r["v"][-1][(h // gqa) * s.head_dim:(h // gqa + 1) * s.head_dim] for h in range(s.num_heads)])
    assert bits_equal(ctx, want)


def test_rope_position_zero_is_identity():
    v = oracle.synth_logits(3, 512, 1.0)
    assert bits_equal(oracle.rope_neox(v, 512, 256, 0.0, 1e4), v)


@needs_ref
@pytest.mark.parametrize("full,win", [(False, 2), (False, 1024), (True, 0)])
def test_attention_steps_live_against_reference(full, win):
    w = oracle.AttnWeights(7, oracle.attn_shape(full, sliding_window=win or 1024))
    xs = np.stack([oracle.synth_x(7, t) for t in range(5)])
    a, b = oracle.attention_steps(w, xs), oracle.attention_steps(w, xs, impl="ref")
    for k in a:
        assert bits_equal(a[k], b[k]), k


@needs_ref
def test_embed_and_rope_live_against_reference():
    emb = oracle.synth_quant(3, 90, 300, 2816, 0.05)
    for t in (0, 1, 150, 299):
        assert bits_equal(oracle.embed(emb, t), oracle.embed(emb, t, impl="ref"))
    v = oracle.synth_logits(4, 512, 2.0)
    for pos, pairs, theta in ((1.0, 256, 1e4), (777.0, 64, 1e6), (131071.0, 128, 1e4)):
        assert bits_equal(oracle.rope_neox(v, 512, pairs, pos, theta), oracle.rope_neox(v, 512, pairs, pos, theta, "ref"))

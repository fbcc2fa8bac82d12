"""Device embedding lookup, QKV epilogue and decode attention (include/gtmoe_attention.h) against
the reference's kernel-test known answers (tests/golden/kat.npz) and the pinned attention oracle.

Bars: the embedding lookup bit-identical; the epilogue and attention within the rule the
reference's own GPU kernels are held to (numpy allclose, |got - want| <= 1e-5 + 1e-4 |want|,
docs/ARCHITECTURE.md), since device powf/sinf/cosf/expf and a parallel softmax round
differently from the C library and a sequential loop.

"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "turbo-winfare_b200"), os.path.join(ROOT, "tests")]

import oracle  # noqa: E402
from test_attn_oracle import uniform_stream  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kat():
    return np.load(os.path.join(ROOT, "tests", "golden", "kat.npz"))


def close(got, want) -> bool:
    return bool(np.all(np.abs(got - want) <= 1e-5 + 1e-4 * np.abs(want)))


def test_embed_lookup_bit_identical(kat):
    import torch
    from gtmoe import attention
    rows, in_dim, _ = (int(v) for v in kat["embed.shape"])
    w = torch.from_numpy(kat["embed.w"].reshape(rows, in_dim // 2)).cuda()
    s = torch.from_numpy(kat["embed.s"].view(np.int16)).cuda()
    b = torch.from_numpy(kat["embed.b"].view(np.int16)).cuda()
    out = torch.empty(in_dim, device="cuda")
    attention.embed_lookup(w, s, b, int(kat["embed.token"][0]), out)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), kat["embed.want"].view(np.uint32))


@pytest.mark.parametrize("in_place", [False, True])
def test_qkv_epilogue_known_answer(kat, in_place):
    import torch
    from gtmoe import attention
    head_dim, heads, rotated, position = (int(v) for v in kat["qkv.shape"])
    x = torch.from_numpy(kat["qkv.vec"].copy()).cuda()
    w = torch.from_numpy(kat["qkv.w"].view(np.int16)).cuda()
    out = x if in_place else torch.empty_like(x)
    attention.qkv_epilogue(x, heads, head_dim, w, 1e-6, rotated, position, 1e6, out=out)
    assert close(out.cpu().numpy(), kat["qkv.want"])


@pytest.mark.parametrize("case", ["attn", "attn_ring"])
def test_attention_known_answer(kat, case):
    import torch
    from gtmoe import attention
    q_heads, kv_heads, head_dim, n_pos, window, capacity = (int(v) for v in kat[case + ".shape"])
    nq, nkv = q_heads * head_dim, capacity * kv_heads * head_dim
    xs = uniform_stream(kat[case + ".rng_state"], nq + 2 * nkv)
    q = (xs[:nq] * np.float32(0.1)).astype(np.float32)
    kc = (xs[nq:nq + nkv] * np.float32(0.1)).astype(np.float32)
    vc = xs[nq + nkv:].copy()
    att = attention.Attention(q_heads, kv_heads, head_dim, window)
    ctx = torch.empty(nq, device="cuda")
    att(torch.from_numpy(q).cuda(), torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda(), ctx, n_pos,
        n_pos - window, capacity)
    assert close(ctx.cpu().numpy(), kat[case + ".want"])


@pytest.mark.parametrize("full", [False, True])
def test_attention_against_oracle_steps(full):
    """The device core on the oracle's own caches after 6 positions of a real layer shape."""
    import torch
    from gtmoe import attention
    s = oracle.attn_shape(full, sliding_window=4)
    w = oracle.AttnWeights(9, s)
    xs = np.stack([oracle.synth_x(9, t) for t in range(6)])
    r = oracle.attention_steps(w, xs)
    n_pos = 6
    first = 0 if full else n_pos - 4
    want = oracle.attention_core(r["q"][-1], r["k_cache"], r["v_cache"], s.num_heads, s.kv_heads, s.head_dim, n_pos,
                                 first, n_pos)
    att = attention.Attention(s.num_heads, s.kv_heads, s.head_dim, n_pos)
    ctx = torch.empty(s.num_heads * s.head_dim, device="cuda")
    att(torch.from_numpy(r["q"][-1].copy()).cuda(), torch.from_numpy(r["k_cache"]).cuda(),
        torch.from_numpy(r["v_cache"]).cuda(), ctx, n_pos, first, n_pos)
    assert close(ctx.cpu().numpy(), want)


def test_timing_sliding_window_layer():
    import torch
    from gtmoe import attention
    q_heads, kv_heads, hd, window = 16, 8, 256, 1024
    kc = torch.randn(window * kv_heads * hd, device="cuda")
    vc = torch.randn_like(kc)
    q = torch.randn(q_heads * hd, device="cuda")
    ctx = torch.empty_like(q)
    att = attention.Attention(q_heads, kv_heads, hd, window)
    for _ in range(5):
        att(q, kc, vc, ctx, 4096, 4096 - window, window)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(100):
        att(q, kc, vc, ctx, 4096, 4096 - window, window)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 10
    nbytes = 2 * window * kv_heads * hd * 4
    print(f"\nattention window {window}: {us:.1f} us per call, {nbytes / us / 1e3:.0f} GB/s of K/V")

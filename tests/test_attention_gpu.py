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


def test_rows_entries_bit_identical_to_single_rows():
    """The batched-decode entries (gtm_*_rows) on 5 rows with ragged positions, ring wrap, a full
    layer and windows whose chunk counts are not monotonic (37 and 38 positions at 8 kv heads):
    every row equals the single-sequence entry on it, bit for bit."""
    import ctypes as C
    import torch
    import gtmoe
    from gtmoe import attention
    L = gtmoe.lib()
    g = torch.Generator(device="cpu").manual_seed(11)
    D = gtmoe.HIDDEN

    def u32(v):
        return (C.c_uint32 * len(v))(*v)

    def bits(t):
        return t.cpu().numpy().view(np.uint32)

    n = 5
    # embedding rows
    vocab = 300
    w = torch.randint(0, 256, (vocab, D // 2), dtype=torch.uint8, generator=g).cuda()
    s = (torch.rand(vocab, D // 64, generator=g) * 0.02).to(torch.bfloat16).view(torch.int16).cuda()
    b = (-torch.rand(vocab, D // 64, generator=g) * 0.1).to(torch.bfloat16).view(torch.int16).cuda()
    toks = [3, 299, 0, 150, 3]
    out = torch.empty(n, D, device="cuda")
    gtmoe.check(L.gtm_embed_lookup_rows(vocab, D, gtmoe.ptr(w), gtmoe.ptr(s), gtmoe.ptr(b), u32(toks), n, 53.0,
                                        gtmoe.ptr(out), None))
    for i, t in enumerate(toks):
        one = torch.empty(D, device="cuda")
        attention.embed_lookup(w, s, b, t, one, scale=53.0)
        assert np.array_equal(bits(out[i]), bits(one)), i
    assert L.gtm_embed_lookup_rows(vocab, D, gtmoe.ptr(w), gtmoe.ptr(s), gtmoe.ptr(b), u32([1, vocab]), 2, 1.0,
                                   gtmoe.ptr(out), None) == gtmoe.ERR_INVALID

    # rmsnorm, gemv, post_attn rows
    x = torch.randn(n, D, generator=g).cuda()
    nw = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16).view(torch.int16).cuda()
    rn = torch.empty(n, D, device="cuda")
    gtmoe.check(L.gtm_rmsnorm_rows(n, D, gtmoe.ptr(x), gtmoe.ptr(nw), 1e-6, gtmoe.ptr(rn), None))
    rows_w = 512
    wq = torch.randint(0, 256, (rows_w, D // 2), dtype=torch.uint8, generator=g).cuda()
    gv = torch.empty(n, rows_w, device="cuda")
    gtmoe.check(L.gtm_gemv_q4_rows(rows_w, D, n, gtmoe.ptr(wq), gtmoe.ptr(s), gtmoe.ptr(b), gtmoe.ptr(x), gtmoe.ptr(gv),
                                   None))
    att = torch.randn(n, D, generator=g).cuda()
    hout = torch.empty(n, D, device="cuda")
    gtmoe.check(L.gtm_post_attn_rows(n, D, gtmoe.ptr(att), gtmoe.ptr(x), gtmoe.ptr(nw), None, None, 1e-6,
                                     gtmoe.ptr(hout), None, None, None, None))
    for i in range(n):
        one = torch.empty(D, device="cuda")
        gtmoe.rmsnorm(x[i], nw, 1e-6, one)
        assert np.array_equal(bits(rn[i]), bits(one)), i
        og = torch.empty(rows_w, device="cuda")
        gtmoe.gemv_q4(wq, s, b, x[i], og, rows_w, D)
        assert np.array_equal(bits(gv[i]), bits(og)), i
        views = [torch.empty(D, device="cuda") for _ in range(4)]
        gtmoe.post_attn(att[i], x[i], nw, nw, nw, 1e-6, *views)
        assert np.array_equal(bits(hout[i]), bits(views[0])), i

    # epilogue and attention rows over per-sequence ring caches
    for H, KV, hd, window, cap, pos in ((16, 8, 256, 64, 64, [0, 37, 36, 200, 63]),
                                        (16, 2, 512, 0, 300, [0, 5, 299, 150, 37])):
        S = 4
        seqs = [2, 0, 3, 1, 2] if window else [0, 1, 2, 3, 3]
        kw, qw = KV * hd, H * hd
        kc = torch.randn(S, cap, kw, generator=g).cuda()
        vc = torch.randn(S, cap, kw, generator=g).cuda()
        q = torch.randn(n, qw, generator=g).cuda()
        kin = torch.randn(n, kw, generator=g).cuda()
        qn = (1 + 0.1 * torch.randn(hd, generator=g)).to(torch.bfloat16).view(torch.int16).cuda()
        kc_single = kc.clone()
        q_single = q.clone()
        ws_n = L.gtm_attention_rows_workspace_bytes(H, hd, cap, n)
        ws = torch.empty(ws_n // 4 + 64, device="cuda")
        ctx = torch.empty(n, qw, device="cuda")
        # q in place; K into the caches, one row per distinct (sequence, slot), as a decode step has
        gtmoe.check(L.gtm_qkv_epilogue_rows(H, hd, n, gtmoe.ptr(q), gtmoe.ptr(qn), 1e-6, hd // 4, u32(pos), 1e4,
                                            gtmoe.ptr(q), None, 0, 0, None))
        uniq = [i for i in range(n) if (seqs[i], pos[i] % cap) not in
                {(seqs[j], pos[j] % cap) for j in range(i)}]
        m = len(uniq)
        gtmoe.check(L.gtm_qkv_epilogue_rows(KV, hd, m, gtmoe.ptr(kin), gtmoe.ptr(qn), 1e-6, hd // 4,
                                            u32([pos[i] for i in uniq]), 1e4, gtmoe.ptr(kc),
                                            u32([seqs[i] for i in uniq]), S, cap, None))
        gtmoe.check(L.gtm_attention_decode_rows(H, KV, hd, n, window, cap, gtmoe.ptr(q), gtmoe.ptr(kc), gtmoe.ptr(vc),
                                                u32(seqs), S, u32(pos), gtmoe.ptr(ctx), C.c_void_p(ws.data_ptr()),
                                                ws_n, None))
        for i in range(n):
            attention.qkv_epilogue(q_single[i], H, hd, qn, 1e-6, hd // 4, pos[i], 1e4)
            assert np.array_equal(bits(q[i]), bits(q_single[i])), ("q", i)
        for j, i in enumerate(uniq):
            slot = kc_single[seqs[i], pos[i] % cap]
            attention.qkv_epilogue(kin[j], KV, hd, qn, 1e-6, hd // 4, pos[i], 1e4, out=slot)
        assert np.array_equal(bits(kc), bits(kc_single))
        for i in range(n):
            n_pos = pos[i] + 1
            first = n_pos - window if window and n_pos > window else 0
            op = attention.Attention(H, KV, hd, cap)
            one = torch.empty(qw, device="cuda")
            op(q[i], kc[seqs[i]], vc[seqs[i]], one, n_pos, first, cap)
            assert np.array_equal(bits(ctx[i]), bits(one)), ("attention", H, KV, hd, i)

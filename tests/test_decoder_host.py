"""Host orchestration of gtmoe.decoder.DeviceDecoder, checked on the CPU.

DeviceDecoder is host code that sequences C-ABI calls: ring-cache slots, which buffer feeds V on
a full-attention layer, window starts, the per-layer MoE launch, the device-side penalty history,
and the order of every argument. Here each gtm_* entry it reaches is replaced by a stand-in
that does the same arithmetic with the pinned CPU oracle on host memory, and each call's
argument count is checked against the C ABI's signature table. With those stand-ins the
decoder's greedy and sampled tokens must equal the reference's own generate tokens
(tests/golden/decoder.npz): the sequencing is right before the device kernels ever run.
Nothing here touches a GPU.
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "turbo-winfare_b200"), os.path.join(ROOT, "tests", "golden")]

import oracle  # noqa: E402
from make_golden import (BATCH_CASE, BATCH_NEW_TOKENS, DECODER_CASES, DECODER_NEW_TOKENS,  # noqa: E402
                         DECODER_SAMPLING, DECODER_STOPS)


def addr(p) -> int:
    if p is None:
        return 0
    if isinstance(p, int):
        return p
    return C.cast(p, C.c_void_p).value or 0


def view(p, n: int, dtype) -> np.ndarray:
    dt = np.dtype(dtype)
    return np.frombuffer((C.c_char * (n * dt.itemsize)).from_address(addr(p)), dtype=dt)


class OracleLib:
    """The device entries DeviceDecoder uses, done by the oracle on host memory."""

    def __init__(self, real, moe_layers, synth_layers):
        self.real, self.moe_base, self.synth = real, C.addressof(moe_layers), synth_layers
        import gtmoe
        self.sig = gtmoe.SIGNATURES

    def __getattr__(self, name):
        fn = getattr(type(self), "_" + name, None)
        if fn is None:
            return getattr(self.real, name)   # host-only entries (validate, seed_for, errors)

        def call(*args):
            assert len(args) == len(self.sig[name][1]), (name, len(args))
            return fn(self, *args)
        return call

    # sizes: any non-zero workspace is accepted by the stand-ins
    def _gtm_moe_decode_workspace_bytes(self, dims):
        return 256

    def _gtm_lm_head_workspace_bytes(self, rows):
        return 256

    def _gtm_attention_workspace_bytes(self, q_heads, head_dim, window):
        return 256

    def _gtm_sample_workspace_bytes(self, vocab):
        return 256

    def _gtm_moe_decode_check(self, ws, st):
        return 0

    def _gtm_embed_lookup(self, rows, in_dim, w, s, b, token, scale, out, st):
        assert token < rows and np.float32(scale) == np.sqrt(np.float32(in_dim))
        g = in_dim // 64
        m = {"w": view(w, rows * in_dim // 2, np.uint8), "s": view(s, rows * g, np.uint16),
             "b": view(b, rows * g, np.uint16), "rows": rows, "in_dim": in_dim}
        view(out, in_dim, np.float32)[:] = oracle.embed(m, token)
        return 0

    def _gtm_gemv_q4(self, rows, in_dim, w, s, b, x, out, st):
        g = in_dim // 64
        view(out, rows, np.float32)[:] = oracle.matvec(view(w, rows * in_dim // 2, np.uint8),
                                                      view(s, rows * g, np.uint16), view(b, rows * g, np.uint16),
                                                      view(x, in_dim, np.float32), rows, in_dim, 4)
        return 0

    def _gtm_rmsnorm(self, n, x, w, eps, out, st):
        wa = None if addr(w) == 0 else view(w, n, np.uint16)
        view(out, n, np.float32)[:] = oracle.rms_norm(view(x, n, np.float32).copy(), wa, eps)
        return 0

    def _gtm_qkv_epilogue(self, heads, head_dim, inp, w, eps, pairs, position, theta, out, st):
        wa = None if addr(w) == 0 else view(w, head_dim, np.uint16)
        vec = view(inp, heads * head_dim, np.float32).copy()
        view(out, heads * head_dim, np.float32)[:] = oracle.qkv_epilogue(vec, heads, head_dim, wa, eps, pairs,
                                                                         float(position), theta)
        return 0

    def _gtm_attention_decode(self, q_heads, kv_heads, head_dim, n_pos, first, capacity, q, kc, vc, ctx, ws, wsb,
                              st):
        assert first < n_pos and n_pos - first <= capacity
        row = kv_heads * head_dim
        view(ctx, q_heads * head_dim, np.float32)[:] = oracle.attention_core(
            view(q, q_heads * head_dim, np.float32), view(kc, capacity * row, np.float32),
            view(vc, capacity * row, np.float32), q_heads, kv_heads, head_dim, n_pos, first, capacity)
        return 0

    def _gtm_post_attn(self, d, attn, hidden, w_post, w_pre, w_pre2, eps, hidden_out, dense, routed, router, st):
        h = view(hidden, d, np.float32)
        view(hidden_out, d, np.float32)[:] = h + oracle.rms_norm(view(attn, d, np.float32).copy(),
                                                                 view(w_post, d, np.uint16), eps)
        return 0

    def _gtm_moe_decode(self, dims, layers, n, io, ws, wsb, st):
        import gtmoe
        assert n == 1
        layer = (addr(layers) - self.moe_base) // C.sizeof(gtmoe.Layer)
        o = io._obj
        x = view(o.hidden_in_dev, oracle.HIDDEN, np.float32).copy()
        view(o.hidden_out_dev, oracle.HIDDEN, np.float32)[:] = self.synth[layer].block(x)["hidden"]
        return 0

    # the *_rows entries: row i at the stated offsets, each row through the single stand-in
    def _gtm_attention_rows_workspace_bytes(self, q_heads, head_dim, window, n):
        return 256

    def _gtm_embed_lookup_rows(self, rows, in_dim, w, s, b, tokens, n, scale, out, st):
        for i in range(n):
            self._gtm_embed_lookup(rows, in_dim, w, s, b, tokens[i], scale, addr(out) + 4 * i * in_dim, st)
        return 0

    def _gtm_rmsnorm_rows(self, rows, n, x, w, eps, out, st):
        for i in range(rows):
            self._gtm_rmsnorm(n, addr(x) + 4 * i * n, w, eps, addr(out) + 4 * i * n, st)
        return 0

    def _gtm_gemv_q4_rows(self, rows, in_dim, n, w, s, b, x, out, st):
        for i in range(n):
            self._gtm_gemv_q4(rows, in_dim, w, s, b, addr(x) + 4 * i * in_dim, addr(out) + 4 * i * rows, st)
        return 0

    def _gtm_qkv_epilogue_rows(self, heads, head_dim, n, inp, w, eps, pairs, positions, theta, out, seqs, num_seqs,
                               capacity, st):
        width = heads * head_dim
        for i in range(n):
            row = i if capacity == 0 else seqs[i] * capacity + positions[i] % capacity
            assert capacity == 0 or seqs[i] < num_seqs
            self._gtm_qkv_epilogue(heads, head_dim, addr(inp) + 4 * i * width, w, eps, pairs, positions[i], theta,
                                   addr(out) + 4 * row * width, st)
        return 0

    def _gtm_attention_decode_rows(self, q_heads, kv_heads, head_dim, n, window, capacity, q, kc, vc, seqs, num_seqs,
                                   positions, ctx, ws, wsb, st):
        qw, kw = q_heads * head_dim, kv_heads * head_dim
        for i in range(n):
            n_pos = positions[i] + 1
            first = n_pos - window if window and n_pos > window else 0
            cache = 4 * seqs[i] * capacity * kw
            self._gtm_attention_decode(q_heads, kv_heads, head_dim, n_pos, first, capacity, addr(q) + 4 * i * qw,
                                       addr(kc) + cache, addr(vc) + cache, addr(ctx) + 4 * i * qw, ws, wsb, st)
        return 0

    def _gtm_post_attn_rows(self, rows, d, attn, hidden, w_post, w_pre, w_pre2, eps, hout, dense, routed, router, st):
        for i in range(rows):
            o = 4 * i * d
            self._gtm_post_attn(d, addr(attn) + o, addr(hidden) + o, w_post, w_pre, w_pre2, eps, addr(hout) + o, None,
                                None, None, st)
        return 0

    def _gtm_moe_tokens_workspace_bytes(self, dims, n):
        return 256

    def _gtm_moe_tokens_check(self, ws, st):
        return 0

    def _gtm_moe_tokens(self, dims, layer, io, ws, wsb, st):
        import gtmoe
        layer = (addr(layer) - self.moe_base) // C.sizeof(gtmoe.Layer)
        o = io._obj
        assert o.x_dev and not o.x_bf16_dev
        D = oracle.HIDDEN
        xs = view(o.x_dev, o.num_tokens * D, np.float32).copy().reshape(o.num_tokens, D)
        out = view(o.hidden_out_dev, o.num_tokens * D, np.float32).reshape(o.num_tokens, D)
        for t in range(o.num_tokens):
            out[t] = self.synth[layer].block(xs[t])["hidden"]
        return 0

    def _gtm_lm_head_greedy(self, rows, in_dim, w, s, b, x, token, logit, ws, wsb, st):
        g = in_dim // 64
        lg = oracle.matvec(view(w, rows * in_dim // 2, np.uint8), view(s, rows * g, np.uint16),
                           view(b, rows * g, np.uint16), view(x, in_dim, np.float32), rows, in_dim, 4)
        view(token, 1, np.int32)[0] = int(np.argmax(lg))
        return 0

    def _gtm_softcap(self, n, inp, cap, out, st):
        view(out, n, np.float32)[:] = oracle.softcap(view(inp, n, np.float32).copy(), cap)
        return 0

    def _gtm_repetition_penalty(self, logits, vocab, hist, n, penalty, softcap, ws, wsb, st):
        if penalty == 1.0 or n == 0:
            return 0
        lg = view(logits, vocab, np.float32)
        lg[:] = oracle.apply_repetition_penalty(lg.copy(), view(hist, n, np.uint32).copy(), penalty, softcap)
        return 0

    def _gtm_sample_token(self, logits, vocab, p, seed, token, status, ws, wsb, st):
        sp = p._obj
        op = oracle.Sampling(sp.temperature, sp.top_p, sp.top_k, sp.repetition_penalty, sp.has_seed, 0, sp.seed)
        rc, tok = oracle.sample_token(view(logits, vocab, np.float32).copy(), op, seed)
        view(token, 1, np.int32)[0] = tok if rc == 0 else -1
        view(status, 1, np.int32)[0] = 0 if rc == 0 else 1
        return 0


@pytest.fixture
def host_decoder(monkeypatch):
    import torch
    import gtmoe
    from gtmoe import attention, decoder, sampling
    from gtmoe.decoder import AttnLayerWeights, DeviceDecoder

    def make(case, batch=False):
        args, prompts = BATCH_CASE if case == "b4" else DECODER_CASES[case]
        dec = oracle.SynthDecoder(**args)
        moe_layers = (gtmoe.Layer * dec.num_layers)()
        fake = OracleLib(gtmoe.lib(), moe_layers, dec.moe)
        for mod in (gtmoe, attention, decoder, sampling):
            monkeypatch.setattr(mod, "lib", lambda: fake)
            monkeypatch.setattr(mod, "_stream", lambda stream=None: None)

        def quant(m):
            return {"w": torch.from_numpy(np.ascontiguousarray(m["w"])),
                    "s": torch.from_numpy(np.ascontiguousarray(m["s"]).view(np.int16)),
                    "b": torch.from_numpy(np.ascontiguousarray(m["b"]).view(np.int16)),
                    "rows": m["rows"], "in_dim": m["in_dim"]}

        def bf16(v):
            return torch.from_numpy(np.ascontiguousarray(v).view(np.int16))

        layers = []
        for l in range(dec.num_layers):
            a, s = dec.attn[l], dec.attn[l].shape
            full = bool(dec.full_mask[l])
            layers.append(AttnLayerWeights(quant(a.q), quant(a.k), None if full else quant(a.v), quant(a.o),
                                           bf16(a.input_norm), bf16(a.q_norm), bf16(a.k_norm),
                                           bf16(dec.post_attn[l]), s.num_heads, s.kv_heads, s.head_dim,
                                           s.rotated_pairs, s.theta, 0 if full else s.sliding_window))
        max_pos = max(len(p) for p in prompts) + DECODER_NEW_TOKENS + 1
        if batch:
            from gtmoe import batch as gbatch
            monkeypatch.setattr(gbatch, "lib", lambda: fake)
            monkeypatch.setattr(gbatch, "_stream", lambda stream=None: None)
            max_pos = max(len(p) for p in prompts) + BATCH_NEW_TOKENS + 1
            moe = gbatch.LocalMoe(moe_layers, len(prompts), device="cpu")
            return gbatch.BatchDecoder(layers, moe, quant(dec.embed_w), bf16(dec.final_norm), max_pos, len(prompts),
                                       device="cpu"), prompts
        dd = DeviceDecoder(layers, moe_layers, quant(dec.embed_w), bf16(dec.final_norm), max_pos, device="cpu")
        return dd, prompts
    return make


@pytest.mark.parametrize("case", sorted(DECODER_CASES))
def test_greedy_sequencing_reproduces_reference(host_decoder, case):
    g = np.load(os.path.join(ROOT, "tests", "golden", "decoder.npz"))
    dd, prompts = host_decoder(case)
    for i, p in enumerate(prompts):
        assert dd.greedy(p, DECODER_NEW_TOKENS, DECODER_STOPS) == g[f"{case}.prompt{i}.tokens"].tolist(), (case, i)


def test_sampled_sequencing_reproduces_reference(host_decoder):
    from gtmoe.sampling import SamplingParams
    g = np.load(os.path.join(ROOT, "tests", "golden", "decoder.npz"))
    dd, prompts = host_decoder("d3")
    for j, (t, tp, tk, pen, seed) in enumerate(DECODER_SAMPLING):
        sp = SamplingParams(t, tp, tk, pen, seed is not None, 0 if seed is None else seed)
        for i, p in enumerate(prompts):
            assert dd.sample(p, DECODER_NEW_TOKENS, sp, DECODER_STOPS) == g[f"d3.sampled{j}.prompt{i}.tokens"].tolist(), \
                (j, i)


def test_empty_prompt_raises_as_reference(host_decoder):
    """CpuReference::generate rejects an empty prompt (cpu_reference.cpp:546); so do both loops,
    before any launch."""
    from gtmoe.sampling import SamplingParams
    dd, _ = host_decoder("d2")
    with pytest.raises(ValueError, match="empty prompt"):
        dd.greedy([], DECODER_NEW_TOKENS, DECODER_STOPS)
    with pytest.raises(ValueError, match="empty prompt"):
        dd.sample([], DECODER_NEW_TOKENS, SamplingParams(1.0, 1.0, 8, 1.0, True, 3), DECODER_STOPS)


def test_batch_sequencing_reproduces_reference(host_decoder):
    """gtmoe.batch.BatchDecoder's lockstep over sequences of different prompt lengths (prefill
    token by token, the first greedy token after the last prompt token, 64 tokens each) with the
    oracle behind every entry: each sequence's tokens equal the reference's own generate tokens
    (tests/golden/batch_decode.npz)."""
    g = np.load(os.path.join(ROOT, "tests", "golden", "batch_decode.npz"))
    bd, prompts = host_decoder("b4", batch=True)
    got = bd.greedy(prompts, BATCH_NEW_TOKENS, DECODER_STOPS)
    for i in range(len(prompts)):
        assert got[i] == g[f"b4.prompt{i}.tokens"].tolist(), i

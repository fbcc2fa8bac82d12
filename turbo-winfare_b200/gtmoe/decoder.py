"""Batch-1 greedy decode of a whole model on the device, through the C ABI: the per-token
sequence of ForwardRunner::produce_token (src/runner.cpp:487-770) with the MoE section as one
gtm_moe_decode launch per layer.

Per token: gtm_embed_lookup (x sqrt(D)); per layer gtm_rmsnorm (input norm), gtm_gemv_q4 for
q, k and v (full-attention layers: V is the raw k_proj output), gtm_qkv_epilogue for q in place
and for K and V straight into their ring-cache rows (position p in row p % capacity),
gtm_attention_decode, gtm_gemv_q4 for o, gtm_post_attn (the residual), then gtm_moe_decode for
the layer; finally gtm_rmsnorm (final norm) and gtm_lm_head_greedy. Only the 4-byte token comes
back to the host. Sampled decoding (`sample`) instead forms the logits with gtm_gemv_q4 on the
tied embedding, softcaps them (gtm_softcap), applies the repetition penalty over the device-side
history and draws with gtm_sample_token, as the sampled branch of produce_token
(runner.cpp:771-806) and CpuReference::generate (src/cpu_reference.cpp:573-593) do.

The greedy head takes the argmax of the raw logits, as the reference's GPU greedy branch does
(runner.cpp:720-770); the CPU reference takes it after the softcap, which can only differ when
tanh saturation rounds two logits to the same value.

`greedy` and `sample` queue every launch on the caller's stream (torch's current stream when none
is given) and make that stream torch's current one for the whole loop, so the host reads of the
token and the writes into the device-side history are ordered after the kernels that produce and
consume them. An empty prompt raises, as CpuReference::generate does (cpu_reference.cpp:546).
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field

from . import HIDDEN, Decoder, LmHead, _stream, check, lib, ptr
from .attention import Attention


@dataclass
class AttnLayerWeights:
    """One layer's attention weights on the device. Quantised matrices are dicts with w (uint8
    [rows, in_dim/2]), s and b (bf16 bits [rows, in_dim/64]), rows and in_dim; v is None on a
    full-attention layer (V is k_proj's output)."""
    q: dict
    k: dict
    v: dict | None
    o: dict
    input_norm: object
    q_norm: object
    k_norm: object
    post_attn_norm: object
    num_heads: int
    kv_heads: int
    head_dim: int
    rotated_pairs: int
    theta: float
    window: int          # attended positions; 0 = all (full attention)
    caches: list = field(default_factory=list)


class DeviceDecoder:
    SOFTCAP = 30.0   # final_logit_softcap

    def __init__(self, attn_layers: list[AttnLayerWeights], moe_layers, embed: dict, final_norm, max_pos: int,
                 eps: float = 1e-6, device: str = "cuda"):
        import torch
        self.attn, self.embed, self.final_norm, self.eps = attn_layers, embed, final_norm, eps
        self.n = len(attn_layers)
        self.max_pos = max_pos
        self.moe = Decoder(moe_layers, self.n, device=device)
        self.lm = LmHead(embed["rows"], device=device)
        f32 = dict(dtype=torch.float32, device=device)
        self.hidden = torch.zeros(HIDDEN, **f32)
        self.mid = torch.zeros(HIDDEN, **f32)
        self.normed = torch.zeros(HIDDEN, **f32)
        self.attn_out = torch.zeros(HIDDEN, **f32)
        self.views = torch.zeros(3, HIDDEN, **f32)
        self.token = torch.zeros(1, dtype=torch.int32, device=device)
        self.logits = torch.zeros(embed["rows"], **f32)
        self.sampler = None
        for a in attn_layers:
            cap = a.window if a.window > 0 else max_pos
            row = a.kv_heads * a.head_dim
            a.caches = [torch.zeros(cap * row, **f32), torch.zeros(cap * row, **f32)]
            a.q_buf = torch.zeros(a.num_heads * a.head_dim, **f32)
            a.k_buf = torch.zeros(row, **f32)
            a.v_buf = torch.zeros(row, **f32)
            a.ctx = torch.zeros(a.num_heads * a.head_dim, **f32)
            a.op = Attention(a.num_heads, a.kv_heads, a.head_dim, cap, device=device)
        self.scale = float(math.sqrt(float(HIDDEN)))   # sqrt of a float, as cpu_reference.cpp:327

    def _gemv(self, m: dict, x, out, st) -> None:
        check(lib().gtm_gemv_q4(m["rows"], m["in_dim"], ptr(m["w"]), ptr(m["s"]), ptr(m["b"]), ptr(x), ptr(out), st))

    def forward(self, token: int, pos: int, stream=None, logits: bool = False) -> None:
        """One token through every layer, then the greedy head (the token lands in self.token)
        or, with logits=True, the full softcapped logits in self.logits."""
        if pos >= self.max_pos:
            raise ValueError(f"position {pos} beyond max_pos {self.max_pos}")
        st = _stream(stream)
        L = lib()
        e = self.embed
        check(L.gtm_embed_lookup(e["rows"], e["in_dim"], ptr(e["w"]), ptr(e["s"]), ptr(e["b"]), token,
                                 self.scale, ptr(self.hidden), st))
        for l, a in enumerate(self.attn):
            check(L.gtm_rmsnorm(HIDDEN, ptr(self.hidden), ptr(a.input_norm), self.eps, ptr(self.normed), st))
            self._gemv(a.q, self.normed, a.q_buf, st)
            self._gemv(a.k, self.normed, a.k_buf, st)
            if a.v is not None:
                self._gemv(a.v, self.normed, a.v_buf, st)
            v_src = a.v_buf if a.v is not None else a.k_buf
            cap = a.window if a.window > 0 else self.max_pos
            row = a.kv_heads * a.head_dim
            slot = (pos % cap) * row
            kc, vc = a.caches
            check(L.gtm_qkv_epilogue(a.num_heads, a.head_dim, ptr(a.q_buf), ptr(a.q_norm), self.eps, a.rotated_pairs,
                                     pos, a.theta, ptr(a.q_buf), st))
            check(L.gtm_qkv_epilogue(a.kv_heads, a.head_dim, ptr(v_src), None, self.eps, 0, pos, a.theta,
                                     C.c_void_p(vc.data_ptr() + 4 * slot), st))
            check(L.gtm_qkv_epilogue(a.kv_heads, a.head_dim, ptr(a.k_buf), ptr(a.k_norm), self.eps, a.rotated_pairs,
                                     pos, a.theta, C.c_void_p(kc.data_ptr() + 4 * slot), st))
            n_pos = pos + 1
            first = max(0, n_pos - a.window) if a.window > 0 else 0
            a.op(a.q_buf, kc, vc, a.ctx, n_pos, first, cap, stream=stream)
            self._gemv(a.o, a.ctx, self.attn_out, st)
            check(L.gtm_post_attn(HIDDEN, ptr(self.attn_out), ptr(self.hidden), ptr(a.post_attn_norm),
                                  ptr(a.post_attn_norm), ptr(a.post_attn_norm), self.eps, ptr(self.mid),
                                  ptr(self.views[0]), ptr(self.views[1]), ptr(self.views[2]), st))
            self.moe(self.mid, self.hidden, first_layer=l, num_layers=1, norm_between_layers=False, stream=stream)
        check(L.gtm_rmsnorm(HIDDEN, ptr(self.hidden), ptr(self.final_norm), self.eps, ptr(self.normed), st))
        if logits:
            self._gemv(e, self.normed, self.logits, st)   # tie_word_embeddings
            check(L.gtm_softcap(e["rows"], ptr(self.logits), self.SOFTCAP, ptr(self.logits), st))
        else:
            self.lm(e["w"], e["s"], e["b"], self.normed, self.token, stream=stream)

    def _on_stream(self, stream):
        """Makes the caller's stream torch's current one (device tensors only)."""
        import contextlib
        import torch
        if self.hidden.device.type != "cuda":
            return contextlib.nullcontext()
        return torch.cuda.stream(stream if stream is not None else torch.cuda.current_stream(self.hidden.device))

    def greedy(self, prompt, max_tokens: int, stops=(1, 106, 50), stream=None) -> list[int]:
        """CpuReference::generate's loop (src/cpu_reference.cpp:560-593) with greedy tokens."""
        if len(prompt) == 0:
            raise ValueError("empty prompt")   # cpu_reference.cpp:546
        with self._on_stream(stream):
            return self._greedy(prompt, max_tokens, stops)

    def _greedy(self, prompt, max_tokens: int, stops) -> list[int]:
        stream = None   # the caller's stream is torch's current one here
        for a in self.attn:
            for c in a.caches:
                c.zero_()
        for i, t in enumerate(prompt):
            self.forward(int(t), i, stream)
        out, pos = [], len(prompt)
        for step in range(max_tokens):
            nxt = int(self.token.item())
            if nxt in stops:
                break
            out.append(nxt)
            if step + 1 >= max_tokens:
                break
            self.forward(nxt, pos, stream)
            pos += 1
        self.moe.check(stream)
        return out

    def sample(self, prompt, max_tokens: int, p, stops=(1, 106, 50), stream=None) -> list[int]:
        """Sampled decoding (gtmoe.sampling.SamplingParams `p`): CpuReference::generate's loop with
        the penalty, the draw and seed_for(p, position) on the device; one token and its status
        word come back per step. Raises if a draw is degenerate or compared values inside the
        double-exp bound (the status word's NEAR bits)."""
        if len(prompt) == 0:
            raise ValueError("empty prompt")   # cpu_reference.cpp:546
        with self._on_stream(stream):
            return self._sample(prompt, max_tokens, p, stops)

    def _sample(self, prompt, max_tokens: int, p, stops) -> list[int]:
        import torch
        from .sampling import DEGENERATE, Sampler, seed_for, validate_sampling
        stream = None   # the caller's stream is torch's current one here
        validate_sampling(p)
        if self.sampler is None:
            self.sampler = Sampler(self.embed["rows"], device=str(self.hidden.device))
        for a in self.attn:
            for c in a.caches:
                c.zero_()
        hist = torch.zeros(len(prompt) + max_tokens, dtype=torch.int32, device=self.hidden.device)
        n_hist = 0
        if p.repetition_penalty != 1.0:
            hist[:len(prompt)] = torch.tensor([int(t) for t in prompt], dtype=torch.int32)
            n_hist = len(prompt)
        for i, t in enumerate(prompt):
            self.forward(int(t), i, stream, logits=True)
        out, pos = [], len(prompt)
        for step in range(max_tokens):
            self.sampler.apply_repetition_penalty(self.logits, hist[:n_hist] if n_hist else None, p.repetition_penalty,
                                                  self.SOFTCAP, stream=stream)
            tok, status = (int(v) for v in self.sampler.sample_token(self.logits, p, seed_for(p, pos), stream).tolist())
            if status:
                raise RuntimeError(f"sample_token status {status} at position {pos}" +
                                   (" (degenerate distribution)" if status & DEGENERATE else ""))
            if tok in stops:
                break
            out.append(tok)
            if p.repetition_penalty != 1.0:
                hist[n_hist] = tok
                n_hist += 1
            if step + 1 >= max_tokens:
                break
            self.forward(tok, pos, stream, logits=True)
            pos += 1
        self.moe.check(stream)
        return out

"""Greedy decode of many sequences at once: every step advances each live
sequence by one token, and each layer's MoE block runs once over all the step's tokens.

The reference decodes one sequence at a time, a token at a time (ForwardRunner::generate_tokens,
src/runner.cpp:818-949, prompt loop :845-854; CpuReference::generate, src/cpu_reference.cpp:
544-595). Here the sequences are independent exactly as there: each has its own KV ring caches,
positions and tokens, prefills its prompt token by token and stops on max_tokens or a stop id.
What is shared is the step: per layer,

  attention   per sequence, through the C ABI (gtm_rmsnorm, gtm_gemv_q4 for q/k/v, gtm_qkv_epilogue
              writing K and V into the sequence's ring row p % capacity, gtm_attention_decode,
              gtm_gemv_q4 for o, gtm_post_attn) into row i of the step's [n, hidden] block input;
  MoE block   once for the n rows: gtm_moe_tokens (routing, tcgen05 grouped expert GEMMs, combine)
              on one GPU, or expert parallel over NVLink peer memory (gtmoe.ep.ep_layer_peer) with
              the sequences split over the ranks;

then the greedy LM head (gtm_lm_head_greedy) for every sequence past its prompt. Only the step's
token ids come back to the host. Under expert parallelism every rank takes part in every layer's
exchange until all ranks' sequences are done (a rank whose sequences finished joins with none).
"""
from __future__ import annotations

import ctypes as C
import math

from . import HIDDEN, LmHead, TokenBlock, _stream, check, lib, ptr
from .attention import Attention


class LocalMoe:
    """The step's MoE block on this GPU: gtm_moe_tokens over the rows."""

    def __init__(self, moe_layers, max_tokens: int, device: str = "cuda"):
        self.layers = moe_layers
        self.block = TokenBlock(max_tokens, device=device)

    def __call__(self, l: int, x, out) -> None:
        if x.shape[0] > 0:
            self.block(self.layers[l], x, out)

    def check(self) -> None:
        self.block.check()


class PeerEpMoe:
    """The step's MoE block expert parallel over peer memory: `ops` (gtmoe.ep.PeerEpOps, connected)
    serves every layer, `layers[l]` being this rank's shard descriptor of layer l."""

    def __init__(self, ops, barrier, layers):
        self.ops, self.barrier, self.layers = ops, barrier, layers

    def __call__(self, l: int, x, out) -> None:
        from .ep import ep_layer_peer
        self.ops.layer = self.layers[l]
        ep_layer_peer(self.ops, self.barrier, x, out)

    def check(self) -> None:
        self.ops.check()


class BatchDecoder:
    """Up to `max_seqs` sequences through the whole decoder, one token each per step.

    attn_layers: gtmoe.decoder.AttnLayerWeights (weights only; the caches are per sequence here);
    moe: LocalMoe or PeerEpMoe; embed: the tied embedding dict (w, s, b, rows, in_dim); final_norm:
    bf16 bits [hidden]; max_pos: the longest prompt + generated tokens any sequence reaches."""

    SOFTCAP = 30.0

    def __init__(self, attn_layers, moe, embed: dict, final_norm, max_pos: int, max_seqs: int,
                 eps: float = 1e-6, device: str = "cuda", dist=None):
        import torch
        self.attn, self.moe, self.embed, self.final_norm, self.eps = attn_layers, moe, embed, final_norm, eps
        self.max_pos, self.max_seqs, self.dist = max_pos, max_seqs, dist
        f32 = dict(dtype=torch.float32, device=device)
        self.hidden = torch.zeros(max_seqs, HIDDEN, **f32)
        self.mid = torch.zeros(max_seqs, HIDDEN, **f32)
        self.normed = torch.zeros(HIDDEN, **f32)
        self.attn_out = torch.zeros(HIDDEN, **f32)
        self.views = torch.zeros(3, HIDDEN, **f32)
        self.tokens = torch.zeros(max_seqs, dtype=torch.int32, device=device)
        self.lm = LmHead(embed["rows"], device=device)
        self.caches = []    # [layer][seq] -> (k, v)
        self.ops = []
        for a in attn_layers:
            cap = a.window if a.window > 0 else max_pos
            row = a.kv_heads * a.head_dim
            self.caches.append([(torch.zeros(cap * row, **f32), torch.zeros(cap * row, **f32))
                                for _ in range(max_seqs)])
            a.q_buf = torch.zeros(a.num_heads * a.head_dim, **f32)
            a.k_buf = torch.zeros(row, **f32)
            a.v_buf = torch.zeros(row, **f32)
            a.ctx = torch.zeros(a.num_heads * a.head_dim, **f32)
            self.ops.append(Attention(a.num_heads, a.kv_heads, a.head_dim, cap, device=device))
        self.scale = float(math.sqrt(float(HIDDEN)))   # sqrt of a float, as cpu_reference.cpp:327

    def _gemv(self, m: dict, x, out, st) -> None:
        check(lib().gtm_gemv_q4(m["rows"], m["in_dim"], ptr(m["w"]), ptr(m["s"]), ptr(m["b"]), ptr(x), ptr(out), st))

    def _attention(self, l: int, seq: int, row: int, pos: int, st) -> None:
        """Layer l's attention for sequence `seq` at position `pos`: hidden[row] -> mid[row]."""
        L = lib()
        a = self.attn[l]
        hid, mid = self.hidden[row], self.mid[row]
        check(L.gtm_rmsnorm(HIDDEN, ptr(hid), ptr(a.input_norm), self.eps, ptr(self.normed), st))
        self._gemv(a.q, self.normed, a.q_buf, st)
        self._gemv(a.k, self.normed, a.k_buf, st)
        if a.v is not None:
            self._gemv(a.v, self.normed, a.v_buf, st)
        v_src = a.v_buf if a.v is not None else a.k_buf   # full layers: V is k_proj's output
        cap = a.window if a.window > 0 else self.max_pos
        slot = (pos % cap) * a.kv_heads * a.head_dim
        kc, vc = self.caches[l][seq]
        check(L.gtm_qkv_epilogue(a.num_heads, a.head_dim, ptr(a.q_buf), ptr(a.q_norm), self.eps, a.rotated_pairs,
                                 pos, a.theta, ptr(a.q_buf), st))
        check(L.gtm_qkv_epilogue(a.kv_heads, a.head_dim, ptr(v_src), None, self.eps, 0, pos, a.theta,
                                 C.c_void_p(vc.data_ptr() + 4 * slot), st))
        check(L.gtm_qkv_epilogue(a.kv_heads, a.head_dim, ptr(a.k_buf), ptr(a.k_norm), self.eps, a.rotated_pairs,
                                 pos, a.theta, C.c_void_p(kc.data_ptr() + 4 * slot), st))
        n_pos = pos + 1
        first = max(0, n_pos - a.window) if a.window > 0 else 0
        self.ops[l](a.q_buf, kc, vc, a.ctx, n_pos, first, cap)
        self._gemv(a.o, a.ctx, self.attn_out, st)
        check(L.gtm_post_attn(HIDDEN, ptr(self.attn_out), ptr(hid), ptr(a.post_attn_norm), ptr(a.post_attn_norm),
                              ptr(a.post_attn_norm), self.eps, ptr(mid), ptr(self.views[0]), ptr(self.views[1]),
                              ptr(self.views[2]), st))

    def step(self, seqs, toks, positions, heads) -> None:
        """One step: row i carries sequence seqs[i]'s token toks[i] at positions[i]; rows in
        `heads` (the sequences past their prompt) get their greedy next token in self.tokens."""
        st = _stream()
        L = lib()
        e = self.embed
        n = len(seqs)
        for i in range(n):
            check(L.gtm_embed_lookup(e["rows"], e["in_dim"], ptr(e["w"]), ptr(e["s"]), ptr(e["b"]), int(toks[i]),
                                     self.scale, ptr(self.hidden[i]), st))
        for l in range(len(self.attn)):
            for i in range(n):
                self._attention(l, seqs[i], i, positions[i], st)
            self.moe(l, self.mid[:n], self.hidden[:n])
        for i in heads:
            check(L.gtm_rmsnorm(HIDDEN, ptr(self.hidden[i]), ptr(self.final_norm), self.eps, ptr(self.normed), st))
            self.lm(e["w"], e["s"], e["b"], self.normed, self.tokens[i:i + 1])

    def _all_done(self, done: bool) -> bool:
        if self.dist is None:
            return done
        import torch
        flag = torch.tensor([0 if done else 1], dtype=torch.int32, device=self.hidden.device)
        self.dist.all_reduce(flag)
        return int(flag.item()) == 0

    def greedy(self, prompts, max_tokens: int, stops=(1, 106, 50)) -> list[list[int]]:
        """CpuReference::generate's greedy loop for every prompt, advanced together: sequence i
        prefills prompts[i] at positions 0.., then feeds back its argmax token until it has
        max_tokens tokens or meets a stop id."""
        if len(prompts) > self.max_seqs:
            raise ValueError(f"{len(prompts)} prompts > max_seqs {self.max_seqs}")
        if any(len(p) == 0 for p in prompts):
            raise ValueError("empty prompt")   # cpu_reference.cpp:546
        if any(len(p) + max_tokens > self.max_pos for p in prompts):
            raise ValueError(f"a prompt plus {max_tokens} tokens exceeds max_pos {self.max_pos}")
        for per_layer in self.caches:
            for kc, vc in per_layer:
                kc.zero_()
                vc.zero_()
        out = [[] for _ in prompts]
        live = [max_tokens > 0 for _ in prompts]
        step = 0
        while not self._all_done(not any(live)):
            seqs, toks, pos, heads = [], [], [], []
            for i, p in enumerate(prompts):
                if not live[i]:
                    continue
                if step < len(p):
                    t = int(p[step])
                else:
                    t = out[i][-1]
                if step >= len(p) - 1:
                    heads.append(len(seqs))
                seqs.append(i)
                toks.append(t)
                pos.append(step)
            self.step(seqs, toks, pos, heads)
            if heads:
                got = self.tokens[:len(seqs)].cpu().tolist()
                for r in heads:
                    i = seqs[r]
                    nxt = int(got[r])
                    if nxt in stops:
                        live[i] = False
                        continue
                    out[i].append(nxt)
                    if len(out[i]) >= max_tokens:
                        live[i] = False
            step += 1
        self.moe.check()
        return out

"""Greedy decode of many sequences at once: every step advances each live
sequence by one token, and each layer's MoE block runs once over all the step's tokens.

The reference decodes one sequence at a time, a token at a time (ForwardRunner::generate_tokens,
src/runner.cpp:818-949, prompt loop :845-854; CpuReference::generate, src/cpu_reference.cpp:
544-595). Here the sequences are independent exactly as there: each has its own KV ring caches,
positions and tokens, prefills its prompt token by token and stops on max_tokens or a stop id.
What is shared is the step: per layer, one launch per stage covers the n rows of the step,
row i being one sequence's token,

  attention   gtm_rmsnorm_rows, gtm_gemv_q4_rows for q/k/v, gtm_qkv_epilogue_rows writing K and V
              into each sequence's ring row p % capacity, gtm_attention_decode_rows over each
              sequence's own caches, gtm_gemv_q4_rows for o, gtm_post_attn_rows (every row's
              result bit-identical to the single-sequence entries);
  MoE block   gtm_moe_tokens over the n rows (routing, tcgen05 grouped expert GEMMs, combine) on
              one GPU, or expert parallel over NVLink peer memory (gtmoe.ep.ep_layer_peer) with the
              sequences split over the ranks;

then the greedy LM head (gtm_lm_head_greedy) for every sequence past its prompt. Only the step's
token ids come back to the host. Under expert parallelism every rank takes part in every layer's
exchange until all ranks' sequences are done (a rank whose sequences finished joins with none).
"""
from __future__ import annotations

import ctypes as C
import math

from . import HIDDEN, LmHead, TokenBlock, _stream, check, lib, ptr


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

    attn_layers: gtmoe.decoder.AttnLayerWeights (weights only; the caches live here, one K and one
    V tensor per layer laid out [max_seqs][capacity][kv_heads * head_dim]); moe: LocalMoe or
    PeerEpMoe; embed: the tied embedding dict (w, s, b, rows, in_dim); final_norm: bf16 bits
    [hidden]; max_pos: the longest prompt + generated tokens any sequence reaches."""

    SOFTCAP = 30.0

    def __init__(self, attn_layers, moe, embed: dict, final_norm, max_pos: int, max_seqs: int,
                 eps: float = 1e-6, device: str = "cuda", dist=None):
        import torch
        self.attn, self.moe, self.embed, self.final_norm, self.eps = attn_layers, moe, embed, final_norm, eps
        self.max_pos, self.max_seqs, self.dist = max_pos, max_seqs, dist
        f32 = dict(dtype=torch.float32, device=device)
        self.hidden = torch.zeros(max_seqs, HIDDEN, **f32)
        self.mid = torch.zeros(max_seqs, HIDDEN, **f32)
        self.normed = torch.zeros(max_seqs, HIDDEN, **f32)
        self.attn_out = torch.zeros(max_seqs, HIDDEN, **f32)
        self.tokens = torch.zeros(max_seqs, dtype=torch.int32, device=device)
        self.lm = LmHead(embed["rows"], device=device)
        self.caches = []    # [layer] -> (k, v), each [max_seqs][capacity][kv_heads * head_dim]
        qn = max(a.num_heads * a.head_dim for a in attn_layers)
        kn = max(a.kv_heads * a.head_dim for a in attn_layers)
        ws = 0
        for a in attn_layers:
            cap = self.capacity(a)
            row = a.kv_heads * a.head_dim
            self.caches.append((torch.zeros(max_seqs, cap, row, **f32), torch.zeros(max_seqs, cap, row, **f32)))
            ws = max(ws, lib().gtm_attention_rows_workspace_bytes(a.num_heads, a.head_dim, cap, max_seqs))
        # flat scratch, viewed [n, width] with each layer's widths (sliding and full layers differ)
        self.q_buf = torch.zeros(max_seqs * qn, **f32)
        self.k_buf = torch.zeros(max_seqs * kn, **f32)
        self.v_buf = torch.zeros(max_seqs * kn, **f32)
        self.ctx = torch.zeros(max_seqs * qn, **f32)
        self.ws_bytes = ws
        self.workspace = torch.empty(ws // 4 + 64, **f32)
        self.scale = float(math.sqrt(float(HIDDEN)))   # sqrt of a float, as cpu_reference.cpp:327

    def capacity(self, a) -> int:
        return a.window if a.window > 0 else self.max_pos

    @staticmethod
    def _u32(vals):
        return (C.c_uint32 * max(1, len(vals)))(*[int(v) for v in vals])

    def _gemv(self, m: dict, n: int, x, out, st) -> None:
        check(lib().gtm_gemv_q4_rows(m["rows"], m["in_dim"], n, ptr(m["w"]), ptr(m["s"]), ptr(m["b"]), ptr(x), ptr(out),
                                     st))

    def _attention(self, l: int, n: int, seqs, pos, st) -> None:
        """Layer l's attention for the step's n rows: hidden[:n] -> mid[:n]."""
        L = lib()
        a = self.attn[l]
        qn, kn = a.num_heads * a.head_dim, a.kv_heads * a.head_dim
        q, ctx = self.q_buf[:n * qn].view(n, qn), self.ctx[:n * qn].view(n, qn)
        k, v = self.k_buf[:n * kn].view(n, kn), self.v_buf[:n * kn].view(n, kn)
        check(L.gtm_rmsnorm_rows(n, HIDDEN, ptr(self.hidden), ptr(a.input_norm), self.eps, ptr(self.normed), st))
        self._gemv(a.q, n, self.normed, q, st)
        self._gemv(a.k, n, self.normed, k, st)
        if a.v is not None:
            self._gemv(a.v, n, self.normed, v, st)
        v_src = v if a.v is not None else k   # full layers: V is k_proj's output
        cap = self.capacity(a)
        kc, vc = self.caches[l]
        S = self.max_seqs
        check(L.gtm_qkv_epilogue_rows(a.num_heads, a.head_dim, n, ptr(q), ptr(a.q_norm), self.eps, a.rotated_pairs, pos,
                                      a.theta, ptr(q), None, 0, 0, st))
        check(L.gtm_qkv_epilogue_rows(a.kv_heads, a.head_dim, n, ptr(v_src), None, self.eps, 0, pos, a.theta, ptr(vc),
                                      seqs, S, cap, st))
        check(L.gtm_qkv_epilogue_rows(a.kv_heads, a.head_dim, n, ptr(k), ptr(a.k_norm), self.eps, a.rotated_pairs, pos,
                                      a.theta, ptr(kc), seqs, S, cap, st))
        check(L.gtm_attention_decode_rows(a.num_heads, a.kv_heads, a.head_dim, n, a.window, cap, ptr(q), ptr(kc),
                                          ptr(vc), seqs, S, pos, ptr(ctx), C.c_void_p(self.workspace.data_ptr()),
                                          self.ws_bytes, st))
        self._gemv(a.o, n, ctx, self.attn_out, st)
        check(L.gtm_post_attn_rows(n, HIDDEN, ptr(self.attn_out), ptr(self.hidden), ptr(a.post_attn_norm), None, None,
                                   self.eps, ptr(self.mid), None, None, None, st))

    def step(self, seqs, toks, positions, heads) -> None:
        """One step: row i carries sequence seqs[i]'s token toks[i] at positions[i]; rows in
        `heads` (the sequences past their prompt) get their greedy next token in self.tokens."""
        st = _stream()
        L = lib()
        e = self.embed
        n = len(seqs)
        if n:
            check(L.gtm_embed_lookup_rows(e["rows"], e["in_dim"], ptr(e["w"]), ptr(e["s"]), ptr(e["b"]), self._u32(toks),
                                          n, self.scale, ptr(self.hidden), st))
        sq, ps = self._u32(seqs), self._u32(positions)
        for l in range(len(self.attn)):
            if n:
                self._attention(l, n, sq, ps, st)
            self.moe(l, self.mid[:n], self.hidden[:n])
        if heads:
            check(L.gtm_rmsnorm_rows(n, HIDDEN, ptr(self.hidden), ptr(self.final_norm), self.eps, ptr(self.normed), st))
        for i in heads:
            self.lm(e["w"], e["s"], e["b"], self.normed[i], self.tokens[i:i + 1])

    def _all_done(self, done: bool) -> bool:
        if self.dist is None:
            return done
        import torch
        flag = torch.tensor([0 if done else 1], dtype=torch.int32, device=self.hidden.device)
        self.dist.all_reduce(flag)
        return int(flag.item()) == 0

    def greedy(self, prompts, max_tokens: int, stops=(1, 106, 50), on_step=None) -> list[list[int]]:
        """CpuReference::generate's greedy loop for every prompt, advanced together: sequence i
        prefills prompts[i] at positions 0.., then feeds back its argmax token until it has
        max_tokens tokens or meets a stop id. on_step(step) is called after every step."""
        if len(prompts) > self.max_seqs:
            raise ValueError(f"{len(prompts)} prompts > max_seqs {self.max_seqs}")
        if any(len(p) == 0 for p in prompts):
            raise ValueError("empty prompt")   # cpu_reference.cpp:546
        if any(len(p) + max_tokens > self.max_pos for p in prompts):
            raise ValueError(f"a prompt plus {max_tokens} tokens exceeds max_pos {self.max_pos}")
        for kc, vc in self.caches:
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
            if on_step is not None:
                on_step(step)
            step += 1
        self.moe.check()
        return out


# Attention shapes of Gemma-4-26B-A4B (the manifest defaults, include/gturbo/manifest.hpp:22-49):
# sliding-window layers, and every sixth layer full attention with V = k_proj's output.
SWA_SHAPE = dict(num_heads=16, kv_heads=8, head_dim=256, theta=10000.0)
FULL_SHAPE = dict(num_heads=16, kv_heads=2, head_dim=512, theta=1000000.0)


def synth_decoder(num_layers: int = 30, vocab: int = 262144, seed: int = 0, window: int = 1024,
                  full_every: int = 6, device: str = "cuda"):
    """Random-init attention layers, tied embedding and final norm of the Gemma-4-26B-A4B decoder
    shape, generated on the device (gtm_synth_quant / gtm_synth_norm): returns (attn_layers,
    embed, final_norm) for BatchDecoder / DeviceDecoder. Layer l is full attention when
    l % full_every == full_every - 1 (layers 5, 11, 17, 23, 29 of 30), rotating a quarter of its
    head dimension; sliding-window layers attend to the last `window` positions and rotate all."""
    import torch
    from .decoder import AttnLayerWeights
    L, st = lib(), _stream()

    def quant(rows, in_dim, layer, kind):
        w = torch.empty(rows, in_dim // 2, dtype=torch.uint8, device=device)
        s = torch.empty(rows, in_dim // 64, dtype=torch.int16, device=device)
        b = torch.empty_like(s)
        check(L.gtm_synth_quant(seed, layer, kind, kind + 1, rows, in_dim, ptr(w), ptr(s), ptr(b), st))
        return {"w": w, "s": s, "b": b, "rows": rows, "in_dim": in_dim}

    def norm(n, layer, kind):
        v = torch.empty(n, dtype=torch.int16, device=device)
        check(L.gtm_synth_norm(seed, layer, kind, n, ptr(v), st))
        return v

    layers = []
    for l in range(num_layers):
        full = l % full_every == full_every - 1
        d = FULL_SHAPE if full else SWA_SHAPE
        H, KV, hd = d["num_heads"], d["kv_heads"], d["head_dim"]
        pairs = int(hd * 0.25 / 2.0) if full else hd // 2
        layers.append(AttnLayerWeights(quant(H * hd, HIDDEN, l, 32), quant(KV * hd, HIDDEN, l, 34),
                                       None if full else quant(KV * hd, HIDDEN, l, 36), quant(HIDDEN, H * hd, l, 38),
                                       norm(HIDDEN, l, 40), norm(hd, l, 41), norm(hd, l, 42), norm(HIDDEN, l, 43),
                                       H, KV, hd, pairs, d["theta"], 0 if full else window))
    embed = quant(vocab, HIDDEN, 0xFFFE, 44)
    final_norm = norm(HIDDEN, 0xFFFE, 46)
    return layers, embed, final_norm

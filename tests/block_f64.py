"""TEST INFRASTRUCTURE: the MoE block of many tokens at once in float64 (torch, on the device that
holds the weights), used to check every token of a large batch where the exact CPU oracle, one
token at a time, would take minutes.

It restates the oracle's block (oracle/moe_oracle.c orc_moe_block, after the reference's
src/cpu_reference.cpp:422-520) with the routing taken as given: the caller passes the top-8 ids
and weights (the device's own, already checked bit-exact / within 1e-5 against the oracle), so
the restatement checks the expert products, GeGLU, the weighted combine, the shared expert and
the layer tail of every token. Dequantisation is `q * scale + bias` per 64-element group with q
the low nibble first (src/cpu_reference.cpp:55-83); every sum is float64, so the result differs
from the float32 oracle by float32 rounding only (about 1e-6 of the output RMS), far inside the
2e-3 gate. `pin_against_oracle` in the tests checks exactly that on sampled tokens.
"""
from __future__ import annotations

import torch

GROUP = 64


def bf16_at(buf: torch.Tensor, off: int, n: int) -> torch.Tensor:
    """n bf16 values at byte offset `off` of a uint8 device buffer, as float64."""
    return buf[off:off + 2 * n].view(torch.bfloat16).to(torch.float64)


def dequant4(buf: torch.Tensor, w_off: int, s_off: int, b_off: int, rows: int, in_dim: int) -> torch.Tensor:
    """[rows, in_dim] float64 from a packed int4 affine matrix (8 nibbles per uint32, low first)."""
    by = buf[w_off:w_off + rows * in_dim // 2].view(rows, in_dim // 2)
    q = torch.stack([by & 15, by >> 4], dim=-1).view(rows, in_dim).to(torch.float64)
    g = in_dim // GROUP
    s = bf16_at(buf, s_off, rows * g).view(rows, g, 1)
    b = bf16_at(buf, b_off, rows * g).view(rows, g, 1)
    return (q.view(rows, g, GROUP) * s + b).view(rows, in_dim)


def rms(x: torch.Tensor, w: torch.Tensor | None, eps: float) -> torch.Tensor:
    y = x / torch.sqrt((x * x).mean(dim=-1, keepdim=True) + eps)
    return y if w is None else y * w


def gelu_tanh(g: torch.Tensor) -> torch.Tensor:
    return 0.5 * g * (1.0 + torch.tanh(0.7978845608028654 * (g + 0.044715 * g * g * g)))


def block_f64(layer, resident: torch.Tensor, experts: torch.Tensor, x: torch.Tensor, idx: torch.Tensor,
              w: torch.Tensor, *, hidden: int = 2816, moe_inter: int = 704, ffn: int = 2112, eps: float = 1e-6,
              expert_base: int = 0) -> dict[str, torch.Tensor]:
    """layer: a gtmoe.Layer (byte offsets into `resident` and into each expert block of
    `experts`, whose first block is expert `expert_base`); x: [T, hidden] block input;
    idx, w: [T, top_k] routing. Returns h1, h2 and the new hidden state, float64 [T, hidden]."""
    dev = resident.device
    X = x.to(dev, torch.float64)
    T = X.shape[0]
    h = rms(X, None, eps)
    dense = h * bf16_at(resident, layer.pre_ffn_norm, hidden)
    routed = h * bf16_at(resident, layer.pre_ffn_norm_2, hidden)

    def rq(q, rows, in_dim):
        return dequant4(resident, q.weight, q.scales, q.biases, rows, in_dim)

    g = dense @ rq(layer.shared_gate, ffn, hidden).T
    u = dense @ rq(layer.shared_up, ffn, hidden).T
    s = (gelu_tanh(g) * u) @ rq(layer.shared_down, hidden, ffn).T
    h1 = rms(s, bf16_at(resident, layer.post_ffn_norm_1, hidden), eps)

    idx = idx.to(dev, torch.int64)
    wk = w.to(dev, torch.float64)
    h2 = torch.zeros(T, hidden, dtype=torch.float64, device=dev)
    stride = layer.expert_stride
    for e in torch.unique(idx).tolist():
        tok, slot = torch.nonzero(idx == e, as_tuple=True)
        blk = experts[(e - expert_base) * stride:(e - expert_base + 1) * stride]

        def eq(q, rows, in_dim):
            return dequant4(blk, q.weight, q.scales, q.biases, rows, in_dim)

        xe = routed[tok]
        ge = xe @ eq(layer.expert_gate, moe_inter, hidden).T
        ue = xe @ eq(layer.expert_up, moe_inter, hidden).T
        oe = (gelu_tanh(ge) * ue) @ eq(layer.expert_down, hidden, moe_inter).T
        h2.index_add_(0, tok, oe * wk[tok, slot].unsqueeze(1))

    t = rms(h2, bf16_at(resident, layer.post_ffn_norm_2, hidden), eps) + h1
    ls = bf16_at(resident, layer.layer_scalar, 1)
    out = (X + rms(t, bf16_at(resident, layer.post_ffn_norm, hidden), eps)) * ls
    return {"h1": h1, "h2": h2, "hidden": out}


def rel_err_per_token(got: torch.Tensor, ref: torch.Tensor) -> torch.Tensor:
    """max_i |got - ref| / RMS(ref) for every row (float64, on ref's device)."""
    ref = ref.to(torch.float64)
    got = got.to(ref.device, torch.float64)
    den = torch.sqrt((ref * ref).mean(dim=-1))
    return (got - ref).abs().amax(dim=-1) / den


def max_rel(got: torch.Tensor, ref: torch.Tensor) -> float:
    v = rel_err_per_token(got, ref)
    return float(v.max()) if v.numel() else 0.0


"""Batch-1 decode around the MoE block through libgtmoe (include/gtmoe_attention.h): the
reference's EmbedLookup, QKVEpilogue and Attention steps on device tensors, with the KV cache in
the reference's ring layout (position p in row p % capacity, kv_heads * head_dim floats a row).
"""
from __future__ import annotations

import ctypes as C

from . import ERR_INVALID, GtmError, _stream, check, lib, ptr


def embed_lookup(w, s, b, token: int, out, scale: float | None = None, stream=None) -> None:
    """w: uint8 [rows, in_dim/2]; s, b: bf16 bits [rows, in_dim/64]; out: fp32 [in_dim].
    scale defaults to sqrt(in_dim) as a float (cpu_reference.cpp:328)."""
    import numpy as np
    rows, in_dim = w.shape[0], w.shape[1] * 2
    sc = float(np.sqrt(np.float32(in_dim))) if scale is None else scale
    check(lib().gtm_embed_lookup(rows, in_dim, ptr(w), ptr(s), ptr(b), token, sc, ptr(out), _stream(stream)))


def qkv_epilogue(x, heads: int, head_dim: int, w, eps: float, rotated_pairs: int, position: int, theta: float,
                 out=None, stream=None) -> None:
    """In place on x unless out is given; w: bf16 bits [head_dim] or None (no scale)."""
    check(lib().gtm_qkv_epilogue(heads, head_dim, ptr(x), ptr(w), eps, rotated_pairs, position, theta,
                                 ptr(x if out is None else out), _stream(stream)))


class Attention:
    """Decode attention over ring KV caches of up to `max_window` attended positions."""

    def __init__(self, q_heads: int, kv_heads: int, head_dim: int, max_window: int, device: str = "cuda"):
        import torch
        self.q_heads, self.kv_heads, self.head_dim = q_heads, kv_heads, head_dim
        n = lib().gtm_attention_workspace_bytes(q_heads, head_dim, max_window)
        if n == 0:
            raise GtmError(ERR_INVALID, "attention workspace size query failed")
        self.workspace = torch.empty(n // 4 + 64, dtype=torch.float32, device=device)
        self.ws_bytes = n

    def __call__(self, q, k_cache, v_cache, ctx, n_pos: int, first: int, capacity: int, stream=None) -> None:
        check(lib().gtm_attention_decode(self.q_heads, self.kv_heads, self.head_dim, n_pos, first, capacity, ptr(q),
                                         ptr(k_cache), ptr(v_cache), ptr(ctx), C.c_void_p(self.workspace.data_ptr()),
                                         self.ws_bytes, _stream(stream)))

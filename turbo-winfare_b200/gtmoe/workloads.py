"""Synthetic inputs of the benchmark configurations (host-side numpy, seeded).

* config 2: router logits biased so expert popularity follows Zipf(s) over the experts --
  log p_e is added to every token's logits, p_e proportional to rank_e^-s with the ranks a
  fixed random permutation of 1..E (seed 0);
* config 3: uniform-random routing logits U[0, 1) per token and expert, and bf16 activations
  ~ N(0, 1) (the counter-based generator shared with the oracle, rounded to bf16).
"""
from __future__ import annotations

import numpy as np

EXPERTS = 128


def zipf_logit_bias(experts: int = EXPERTS, s: float = 1.1, seed: int = 0) -> np.ndarray:
    rank = np.random.default_rng(seed).permutation(experts).astype(np.float64) + 1.0
    p = rank ** (-s)
    p /= p.sum()
    return np.log(p).astype(np.float32)


def uniform_route_logits(tokens: int, experts: int = EXPERTS, seed: int = 0) -> np.ndarray:
    return np.random.default_rng(seed).random((tokens, experts), dtype=np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 (ties to even), returned as float32 values."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)

"""Token sampling through libgtmoe (include/gtmoe_sampling.h), named after the reference's
include/gturbo/sampling.hpp: ``SamplingParams``, ``validate_sampling``, ``splitmix64``,
``seed_for``, ``apply_repetition_penalty`` and ``sample_token``, with the logits in device
memory. Invalid parameters raise ``GtmError`` carrying the reference's message, where the
reference throws GTurboFormatError.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import ERR_INVALID, GtmError, Sampling, _stream, check, lib, ptr

MAX_TOP_K = 256
DEGENERATE, NEAR_CUT, NEAR_DRAW = 1, 2, 4   # bits of the device status word


@dataclass
class SamplingParams:
    """include/gturbo/sampling.hpp:21-30 (same defaults: greedy, no truncation, no penalty)."""
    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = 0
    repetition_penalty: float = 1.0
    has_seed: bool = False
    seed: int = 0

    def is_greedy(self) -> bool:
        return self.temperature <= 0.0 and self.repetition_penalty == 1.0

    def c(self) -> Sampling:
        return Sampling(self.temperature, self.top_p, self.top_k, self.repetition_penalty, int(self.has_seed), 0,
                        self.seed)


def validate_sampling(p: SamplingParams) -> None:
    """sampling.cpp:32-54; raises GtmError(ERR_INVALID) with the reference's message."""
    c = p.c()
    check(lib().gtm_sampling_validate(C.byref(c)))


def splitmix64(x: int) -> int:
    return lib().gtm_sampling_splitmix64(x)


def seed_for(p: SamplingParams, position: int) -> int:
    c = p.c()
    return lib().gtm_sampling_seed_for(C.byref(c), position)


def softcap(logits, cap: float, out=None, stream=None) -> None:
    """cap * tanh(z / cap) on fp32 device logits, in place unless out is given."""
    check(lib().gtm_softcap(logits.numel(), ptr(logits), cap, ptr(logits if out is None else out), _stream(stream)))


class Sampler:
    """Device sampling over a vocabulary of `vocab` ids, with its own workspace."""

    def __init__(self, vocab: int, device: str = "cuda"):
        import torch
        self.vocab = vocab
        n = lib().gtm_sample_workspace_bytes(vocab)
        if n == 0:
            raise GtmError(ERR_INVALID, f"sampling workspace size query failed for vocab {vocab}")
        self.workspace = torch.empty(n + 256, dtype=torch.uint8, device=device)
        self.ws_ptr = C.c_void_p((self.workspace.data_ptr() + 255) // 256 * 256)
        self.ws_bytes = n
        self.token = torch.zeros(2, dtype=torch.int32, device=device)   # [token, status]

    def apply_repetition_penalty(self, logits, history, penalty: float, softcap: float, stream=None) -> None:
        """sampling.cpp:74-90, in place on fp32 device logits; history: int32/uint32 device ids."""
        n = 0 if history is None else history.numel()
        check(lib().gtm_repetition_penalty(ptr(logits), self.vocab, ptr(history) if n else None, n, penalty, softcap,
                                           self.ws_ptr, self.ws_bytes, _stream(stream)))

    def sample_token(self, logits, p: SamplingParams, seed: int, stream=None):
        """sampling.cpp:92-169 on fp32 device logits. Returns the device tensor [token, status]
        (asynchronous); status carries DEGENERATE / NEAR_CUT / NEAR_DRAW bits."""
        c = p.c()
        check(lib().gtm_sample_token(ptr(logits), self.vocab, C.byref(c), seed, ptr(self.token[0:1]),
                                     ptr(self.token[1:2]), self.ws_ptr, self.ws_bytes, _stream(stream)))
        return self.token

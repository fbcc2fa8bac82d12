"""Host-side checks of the attention C ABI (include/gtmoe_attention.h): arguments the entries
reject before touching the GPU, and the workspace plan. The device parity tests are in
tests/test_attention_gpu.py."""
from __future__ import annotations

import ctypes as C
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "turbo-winfare_b200")]

import gtmoe  # noqa: E402


def test_workspace_plan():
    L = gtmoe.lib()
    assert L.gtm_attention_workspace_bytes(0, 256, 1024) == 0
    assert L.gtm_attention_workspace_bytes(16, 1024, 1024) == 0
    a = L.gtm_attention_workspace_bytes(16, 256, 1024)
    b = L.gtm_attention_workspace_bytes(16, 512, 1 << 17)
    assert a == 16 * 296 * 258 * 4            # at most two CTAs per SM's worth of chunks
    assert b == 16 * (1 << 17) // 256 * 514 * 4   # long contexts: chunks of 256 positions


def test_entries_reject_bad_arguments_before_the_gpu():
    L = gtmoe.lib()
    f = C.c_void_p(256)   # never dereferenced: every case fails its host-side checks
    ws = 1 << 24
    assert L.gtm_attention_decode(16, 8, 256, 10, 0, 16, None, f, f, f, f, ws, None) == gtmoe.ERR_INVALID
    assert L.gtm_attention_decode(16, 3, 256, 10, 0, 16, f, f, f, f, f, ws, None) == gtmoe.ERR_UNSUPPORTED
    assert L.gtm_attention_decode(32, 2, 256, 10, 0, 16, f, f, f, f, f, ws, None) == gtmoe.ERR_UNSUPPORTED  # group 16
    assert L.gtm_attention_decode(16, 8, 192, 10, 0, 16, f, f, f, f, f, ws, None) == gtmoe.ERR_UNSUPPORTED
    assert L.gtm_attention_decode(16, 8, 256, 10, 10, 16, f, f, f, f, f, ws, None) == gtmoe.ERR_INVALID     # empty
    assert L.gtm_attention_decode(16, 8, 256, 300, 0, 128, f, f, f, f, f, ws, None) == gtmoe.ERR_INVALID    # > ring
    assert L.gtm_attention_decode(16, 8, 256, 10, 0, 16, C.c_void_p(260), f, f, f, f, ws, None) == \
        gtmoe.ERR_MISALIGNED
    assert L.gtm_attention_decode(16, 8, 256, 10, 0, 16, f, f, f, f, f, 64, None) == gtmoe.ERR_WORKSPACE
    rc = L.gtm_embed_lookup(64, 2816, f, f, f, 64, 53.0, f, None)
    assert rc == gtmoe.ERR_INVALID and "out of vocabulary" in gtmoe.last_error()
    assert L.gtm_embed_lookup(64, 100, f, f, f, 1, 1.0, f, None) == gtmoe.ERR_INVALID
    assert L.gtm_qkv_epilogue(2, 384, f, None, 1e-6, 0, 0, 1e4, f, None) == gtmoe.ERR_UNSUPPORTED
    assert L.gtm_qkv_epilogue(2, 256, f, None, 1e-6, 129, 0, 1e4, f, None) == gtmoe.ERR_INVALID
    assert L.gtm_qkv_epilogue(2, 256, None, None, 1e-6, 0, 0, 1e4, f, None) == gtmoe.ERR_INVALID

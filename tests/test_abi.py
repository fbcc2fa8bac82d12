"""C-ABI boundary checks that need no GPU: the library loads, exports every entry point the
headers declare, and rejects bad arguments with the documented status and a message."""
import ctypes as C
import os
import re

import pytest

import gtmoe

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in ("gtmoe.h", "gtmoe_synth.h", "gtmoe_bundle.h",
                                                      "gtmoe_sampling.h", "gtmoe_attention.h")]


def declared_symbols():
    names = []
    for h in HEADERS:
        src = open(h).read()
        names += re.findall(r"GTM_API\s+[\w\s\*]+?\b(gtm_\w+)\s*\(", src)
    return names


def test_library_exports_every_declared_symbol():
    L = gtmoe.lib()
    names = declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(gtmoe.SIGNATURES), "Python signature table out of sync with the headers"


def test_version_and_clean_error_state():
    assert b"sm_100a" in gtmoe.lib().gtm_version()


def test_null_pointer_is_invalid_with_message():
    rc = gtmoe.lib().gtm_gemv_q4(96, 2816, None, None, None, None, None, None)
    assert rc == gtmoe.ERR_INVALID
    assert "gtm_gemv_q4" in gtmoe.last_error()


def test_bad_in_dim_rejected():
    p = C.c_void_p(16)  # never dereferenced: validation fails first
    rc = gtmoe.lib().gtm_gemv_q8(128, 100, p, p, p, p, p, None)
    assert rc == gtmoe.ERR_INVALID and "multiple of 64" in gtmoe.last_error()


def test_topk_bounds():
    p = C.c_void_p(16)
    assert gtmoe.lib().gtm_router_topk(128, 0, p, p, p, p, None) == gtmoe.ERR_INVALID
    assert gtmoe.lib().gtm_router_topk(4, 8, p, p, p, p, None) == gtmoe.ERR_INVALID


def test_dispatch_rejects_kernels_off_the_moe_path():
    c = (C.c_uint32 * 16)()
    assert gtmoe.lib().gtm_dispatch(4, None, 0, None, 0, c, 1, None) == gtmoe.ERR_UNSUPPORTED  # QKVEpilogue


def test_decode_rejects_other_shapes_and_small_workspace():
    L = gtmoe.lib()
    d = gtmoe.default_dims()
    assert L.gtm_moe_decode_workspace_bytes(C.byref(d)) > 0
    bad = gtmoe.Dims(4096, 704, 2112, 128, 8, 1e-6)
    assert L.gtm_moe_decode_workspace_bytes(C.byref(bad)) == 0
    layers = (gtmoe.Layer * 1)()
    io = gtmoe.DecodeIO()
    assert L.gtm_moe_decode(C.byref(bad), layers, 1, C.byref(io), None, 0, None) == gtmoe.ERR_UNSUPPORTED
    io.hidden_in_dev = 256
    io.hidden_out_dev = 512
    rc = L.gtm_moe_decode(C.byref(d), layers, 1, C.byref(io), C.c_void_p(4096), 16, None)
    assert rc == gtmoe.ERR_WORKSPACE
    assert L.gtm_moe_decode(C.byref(d), layers, 0, C.byref(io), None, 0, None) == gtmoe.ERR_INVALID
    assert L.gtm_moe_decode(C.byref(d), layers, gtmoe.MAX_LAYERS + 1, C.byref(io), None, 0, None) == gtmoe.ERR_INVALID


def test_expert_block_layout_matches_gturbo():
    # converter order, packed tight, 16 KB stride (tools/convert_hf_to_gturbo.py:379-419;
    # include/gturbo/manifest.hpp:144-147 expert_stride 3,358,720)
    off, stride = gtmoe.expert_layout()
    assert off == [0, 991232, 1053184, 1115136, 2106368, 2168320, 2230272, 3221504, 3283456]
    assert stride == 3358720


def test_resident_layout_is_16k_aligned():
    off, total = gtmoe.resident_layout()
    assert all(o % 16384 == 0 for o in off) and total % 16384 == 0


@pytest.mark.parametrize("field,size", [("Layer", 8 + 24 + 16 + 72 + 48 + 8 + 8 + 72), ("DecodeIO", 9 * 8 + 8),
                                        ("TokensIO", 8 + 10 * 8 + 8)])
def test_struct_sizes(field, size):
    assert C.sizeof(getattr(gtmoe, field)) == size


def test_ep_peer_config_bounds_and_argument_checks():
    # peer-memory expert parallelism: world divides 128 and is at most 8; world x max_tokens <= 65536
    L = gtmoe.lib()
    d = gtmoe.default_dims()
    sizes = {}
    for world, max_tokens in [(1, 64), (2, 64), (8, 64), (8, 8192)]:
        sizes[world, max_tokens] = L.gtm_moe_ep_peer_workspace_bytes(C.byref(d), C.byref(gtmoe.EpConfig(world, 0, max_tokens, 0)))
        assert sizes[world, max_tokens] > 0, (world, max_tokens)
    assert sizes[2, 64] > sizes[1, 64] and sizes[8, 64] > sizes[2, 64]
    for world, rank, max_tokens in [(3, 0, 64), (16, 0, 64), (2, 2, 64), (8, 0, 8193), (2, 0, 0)]:
        cfg = gtmoe.EpConfig(world, rank, max_tokens, 0)
        assert L.gtm_moe_ep_peer_workspace_bytes(C.byref(d), C.byref(cfg)) == 0, (world, rank, max_tokens)
    cfg = gtmoe.EpConfig(2, 0, 64, 0)
    layer, io = gtmoe.Layer(), gtmoe.TokensIO()
    assert L.gtm_moe_ep_peer_experts(C.byref(d), C.byref(layer), C.byref(cfg), None, 0, None) == gtmoe.ERR_INVALID
    peers = gtmoe.EpPeers()
    rc = L.gtm_moe_ep_peer_experts(C.byref(d), C.byref(layer), C.byref(cfg), C.byref(peers), 1 << 40, None)
    assert rc == gtmoe.ERR_WORKSPACE and "gtm_moe_ep_peer_experts" in gtmoe.last_error()
    peers.workspace_dev[0] = 4096
    rc = L.gtm_moe_ep_peer_dispatch(C.byref(d), C.byref(layer), C.byref(io), C.byref(cfg), C.byref(peers), 16, None)
    assert rc == gtmoe.ERR_WORKSPACE
    assert L.gtm_moe_ep_peer_dispatch(C.byref(d), C.byref(layer), C.byref(io), C.byref(cfg), None, 16, None) == gtmoe.ERR_INVALID


def test_ipc_argument_checks():
    L = gtmoe.lib()
    p = C.c_void_p()
    h = (C.c_uint8 * gtmoe.IPC_HANDLE_BYTES)()
    assert L.gtm_ipc_alloc(0, C.byref(p), h) == gtmoe.ERR_INVALID
    assert L.gtm_ipc_alloc(256, None, h) == gtmoe.ERR_INVALID
    assert L.gtm_ipc_open(None, C.byref(p)) == gtmoe.ERR_INVALID
    assert L.gtm_ipc_close(None) == gtmoe.ERR_INVALID
    assert L.gtm_ipc_free(None) == gtmoe.ERR_INVALID
    assert C.sizeof(gtmoe.EpPeers) == 8 * gtmoe.EP_PEER_MAX_WORLD


def test_phase_events_argument_checks():
    L = gtmoe.lib()
    assert L.gtm_set_phase_events(None, 0) == gtmoe.OK   # off
    assert L.gtm_set_phase_events(None, 3) == gtmoe.ERR_INVALID
    arr = (C.c_void_p * 7)()
    assert L.gtm_set_phase_events(arr, 7) == gtmoe.ERR_INVALID and "0..6" in gtmoe.last_error()
    assert L.gtm_set_phase_events(arr, 2) == gtmoe.ERR_INVALID and "NULL" in gtmoe.last_error()
    assert L.gtm_set_phase_events(None, 0) == gtmoe.OK

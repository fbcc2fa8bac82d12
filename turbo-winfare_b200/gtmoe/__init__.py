"""Host side of the B200 MoE block: ctypes bindings to libgtmoe.so (include/gtmoe.h).

PyTorch is used only for device memory and streams; every computation goes through the C ABI
and the sm_100a kernels in libgtmoe.so. There is no fallback: if the library or a CUDA device
is missing, calls raise.

The classes mirror the reference's MoE section of ForwardRunner::produce_token
(src/runner.cpp:549-716) for the batch-1 decode path, with all experts resident in HBM:

* ``SynthModel`` -- random-init weights of the Gemma-4-26B-A4B MoE shape in the .gturbo byte
  layouts (per-layer expert image + resident tensors), generated on the device;
* ``Decoder`` -- one token through N MoE layers in one fused launch (gtm_moe_decode);
* ``TokenBlock`` -- T > 1 tokens through one MoE layer: routing, tcgen05 grouped expert
  products and combine (gtm_moe_tokens), replacing the reference's token-at-a-time prefill
  loop (src/runner.cpp:845-854).
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG, "libgtmoe.so")

HIDDEN, MOE_INTER, FFN, EXPERTS, TOP_K, EPS = 2816, 704, 2112, 128, 8, 1e-6
MAX_LAYERS = 64
NORM_BETWEEN_LAYERS = 1
DECODE_TEST_WAIT_RUNS_OUT = 0x100   # GTM_DECODE_TEST_WAIT_RUNS_OUT (include/gtmoe.h)
TOKENS_TEST_WAIT_RUNS_OUT = 0x100   # GTM_TOKENS_TEST_WAIT_RUNS_OUT (include/gtmoe.h)

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT, ERR_WORKSPACE, ERR_MISALIGNED = 0, -1, -2, -3, -4, -5, -6

KERNEL_RMSNORMK, KERNEL_GEMV_INT4, KERNEL_GEMV_INT8 = 1, 2, 3
KERNEL_ROUTER_TOPK, KERNEL_GEGLU, KERNEL_POST_ATTN, KERNEL_LAYER_TAIL = 6, 7, 8, 9
KERNEL_SCALE_ACCUM, KERNEL_MUL_BF16 = 11, 12


class GtmError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"[{status}] {msg}")
        self.status = status


class Quant(C.Structure):
    _fields_ = [("weight", C.c_uint64), ("scales", C.c_uint64), ("biases", C.c_uint64)]


class Layer(C.Structure):
    _fields_ = [("resident_dev", C.c_void_p), ("router", Quant), ("router_scale", C.c_uint64),
                ("per_expert_scale", C.c_uint64), ("shared_gate", Quant), ("shared_up", Quant),
                ("shared_down", Quant), ("pre_ffn_norm", C.c_uint64), ("pre_ffn_norm_2", C.c_uint64),
                ("post_ffn_norm_1", C.c_uint64), ("post_ffn_norm_2", C.c_uint64), ("post_ffn_norm", C.c_uint64),
                ("layer_scalar", C.c_uint64), ("experts_dev", C.c_void_p), ("expert_stride", C.c_uint64),
                ("expert_gate", Quant), ("expert_up", Quant), ("expert_down", Quant)]


class Dims(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("moe_inter", C.c_uint32), ("ffn_inter", C.c_uint32),
                ("num_experts", C.c_uint32), ("top_k", C.c_uint32), ("eps", C.c_float)]


class DecodeIO(C.Structure):
    _fields_ = [("hidden_in_dev", C.c_void_p), ("hidden_out_dev", C.c_void_p), ("topk_idx_dev", C.c_void_p),
                ("topk_w_dev", C.c_void_p), ("logits_dev", C.c_void_p), ("h1_dev", C.c_void_p),
                ("h2_dev", C.c_void_p), ("hidden_layers_dev", C.c_void_p), ("logit_bias_dev", C.c_void_p),
                ("flags", C.c_uint32)]


class TokensIO(C.Structure):
    _fields_ = [("num_tokens", C.c_uint32), ("x_dev", C.c_void_p), ("x_bf16_dev", C.c_void_p),
                ("hidden_out_dev", C.c_void_p), ("topk_idx_dev", C.c_void_p), ("topk_w_dev", C.c_void_p),
                ("logits_dev", C.c_void_p), ("h1_dev", C.c_void_p), ("h2_dev", C.c_void_p),
                ("logit_bias_dev", C.c_void_p), ("route_logits_dev", C.c_void_p), ("flags", C.c_uint32)]


class EpConfig(C.Structure):
    _fields_ = [("world", C.c_uint32), ("rank", C.c_uint32), ("max_tokens", C.c_uint32),
                ("max_recv_rows", C.c_uint32)]


EP_PEER_MAX_WORLD = 8
IPC_HANDLE_BYTES = 64


class EpPeers(C.Structure):
    _fields_ = [("workspace_dev", C.c_void_p * EP_PEER_MAX_WORLD)]


class BundleInfo(C.Structure):
    _fields_ = [("num_layers", C.c_uint32), ("experts_per_layer", C.c_uint32), ("hidden", C.c_uint32),
                ("moe_inter", C.c_uint32), ("ffn_inter", C.c_uint32), ("top_k", C.c_uint32),
                ("rms_norm_eps", C.c_float), ("resident_entries", C.c_uint32), ("expert_stride", C.c_uint64),
                ("resident_bytes", C.c_uint64), ("resident_index_bytes", C.c_uint64),
                ("layer_file_bytes", C.c_uint64)]


class Sampling(C.Structure):
    """GtmSampling (include/gtmoe_sampling.h), the reference's SamplingParams
    (include/gturbo/sampling.hpp:21-30)."""
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int32),
                ("repetition_penalty", C.c_float), ("has_seed", C.c_int32), ("reserved", C.c_uint32),
                ("seed", C.c_uint64)]


_lib = None

# (name, restype, argtypes) for every entry point in include/gtmoe.h, include/gtmoe_synth.h,
# include/gtmoe_bundle.h, include/gtmoe_sampling.h and include/gtmoe_attention.h
_P, _U32, _U64, _I, _F, _SZ = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int, C.c_float, C.c_size_t
SIGNATURES = {
    "gtm_last_error": (C.c_char_p, []),
    "gtm_version": (C.c_char_p, []),
    "gtm_ctx_create": (_I, [_I, C.POINTER(_P)]),
    "gtm_ctx_destroy": (_I, [_P]),
    "gtm_ctx_stream": (_P, [_P]),
    "gtm_buffer_alloc": (_I, [_P, _U64, C.POINTER(_P)]),
    "gtm_buffer_free": (_I, [_P, _P]),
    "gtm_buffer_upload": (_I, [_P, _P, _U64, _P, _U64]),
    "gtm_buffer_download": (_I, [_P, _P, _P, _U64, _U64]),
    "gtm_submit": (_I, [_P, C.POINTER(_U64)]),
    "gtm_wait": (_I, [_P, _U64, _U32]),
    "gtm_gemv_q4": (_I, [_U32, _U32, _P, _P, _P, _P, _P, _P]),
    "gtm_gemv_q8": (_I, [_U32, _U32, _P, _P, _P, _P, _P, _P]),
    "gtm_router_topk": (_I, [_U32, _U32, _P, _P, _P, _P, _P]),
    "gtm_geglu": (_I, [_U32, _P, _P, _P, _P]),
    "gtm_scale_accum": (_I, [_U32, _P, _P, _U32, _I, _P, _P]),
    "gtm_mul_bf16": (_I, [_U32, _P, _P, _F, _P, _P]),
    "gtm_rmsnorm": (_I, [_U32, _P, _P, _F, _P, _P]),
    "gtm_post_attn": (_I, [_U32, _P, _P, _P, _P, _P, _F, _P, _P, _P, _P, _P]),
    "gtm_layer_tail": (_I, [_U32, _P, _P, _P, _P, _P, _F, _F, _P, _P]),
    "gtm_dispatch": (_I, [_I, C.POINTER(_P), _I, C.POINTER(_P), _I, C.POINTER(_U32), _U32, _P]),
    "gtm_moe_decode_workspace_bytes": (_SZ, [C.POINTER(Dims)]),
    "gtm_moe_decode": (_I, [C.POINTER(Dims), C.POINTER(Layer), _I, C.POINTER(DecodeIO), _P, _SZ, _P]),
    "gtm_moe_decode_check": (_I, [_P, _P]),
    "gtm_moe_decode_noalloc": (_I, [C.POINTER(Dims), C.POINTER(Layer), _I, C.POINTER(DecodeIO), _P]),
    "gtm_moe_tokens_workspace_bytes": (_SZ, [C.POINTER(Dims), _U32]),
    "gtm_moe_tokens": (_I, [C.POINTER(Dims), C.POINTER(Layer), C.POINTER(TokensIO), _P, _SZ, _P]),
    "gtm_moe_tokens_check": (_I, [_P, _P]),
    "gtm_set_phase_events": (_I, [C.POINTER(_P), _I]),
    "gtm_lm_head_workspace_bytes": (_SZ, [_U32]),
    "gtm_lm_head_greedy": (_I, [_U32, _U32, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "gtm_lm_head_candidates": (_I, [_P, _P, C.POINTER(C.c_int32)]),
    "gtm_moe_ep_workspace_bytes": (_SZ, [C.POINTER(Dims), C.POINTER(EpConfig)]),
    "gtm_moe_ep_dispatch": (_I, [C.POINTER(Dims), C.POINTER(Layer), C.POINTER(TokensIO), C.POINTER(EpConfig),
                                 _P, _P, _P, _P, _SZ, _P]),
    "gtm_moe_ep_shared": (_I, [C.POINTER(Dims), C.POINTER(Layer), C.POINTER(TokensIO), C.POINTER(EpConfig),
                               _P, _SZ, _P]),
    "gtm_moe_ep_experts": (_I, [C.POINTER(Dims), C.POINTER(Layer), C.POINTER(EpConfig), _P, _P, _U32, _P,
                                _P, _SZ, _P]),
    "gtm_moe_ep_combine": (_I, [C.POINTER(Dims), C.POINTER(Layer), C.POINTER(TokensIO), C.POINTER(EpConfig),
                                _P, _P, _SZ, _P]),
    "gtm_moe_ep_check": (_I, [_P, _P]),
    "gtm_moe_ep_peer_workspace_bytes": (_SZ, [C.POINTER(Dims), C.POINTER(EpConfig)]),
    "gtm_moe_ep_peer_dispatch": (_I, [C.POINTER(Dims), C.POINTER(Layer), C.POINTER(TokensIO), C.POINTER(EpConfig),
                                      C.POINTER(EpPeers), _SZ, _P]),
    "gtm_moe_ep_peer_shared": (_I, [C.POINTER(Dims), C.POINTER(Layer), C.POINTER(TokensIO), C.POINTER(EpConfig),
                                    _P, _SZ, _P]),
    "gtm_moe_ep_peer_experts": (_I, [C.POINTER(Dims), C.POINTER(Layer), C.POINTER(EpConfig), C.POINTER(EpPeers),
                                     _SZ, _P]),
    "gtm_moe_ep_peer_combine": (_I, [C.POINTER(Dims), C.POINTER(Layer), C.POINTER(TokensIO), C.POINTER(EpConfig),
                                     _P, _SZ, _P]),
    "gtm_ipc_alloc": (_I, [_SZ, C.POINTER(_P), _P]),
    "gtm_ipc_open": (_I, [_P, C.POINTER(_P)]),
    "gtm_ipc_close": (_I, [_P]),
    "gtm_ipc_free": (_I, [_P]),
    "gtm_bundle_open": (_I, [C.c_char_p, C.POINTER(_P)]),
    "gtm_bundle_close": (_I, [_P]),
    "gtm_bundle_info": (_I, [_P, C.POINTER(BundleInfo)]),
    "gtm_bundle_load_resident": (_I, [_P, _P, _U64]),
    "gtm_bundle_load_experts": (_I, [_P, _U32, _U32, _U32, _P, _U64]),
    "gtm_bundle_layer_desc": (_I, [_P, _U32, _P, _P, C.POINTER(Layer)]),
    "gtm_embed_lookup": (_I, [_U32, _U32, _P, _P, _P, _U32, _F, _P, _P]),
    "gtm_qkv_epilogue": (_I, [_U32, _U32, _P, _P, _F, _U32, _U32, _F, _P, _P]),
    "gtm_attention_workspace_bytes": (_SZ, [_U32, _U32, _U32]),
    "gtm_attention_decode": (_I, [_U32, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, _P, _P, _SZ, _P]),
    "gtm_gemv_q4_rows": (_I, [_U32, _U32, _U32, _P, _P, _P, _P, _P, _P]),
    "gtm_rmsnorm_rows": (_I, [_U32, _U32, _P, _P, _F, _P, _P]),
    "gtm_post_attn_rows": (_I, [_U32, _U32, _P, _P, _P, _P, _P, _F, _P, _P, _P, _P, _P]),
    "gtm_embed_lookup_rows": (_I, [_U32, _U32, _P, _P, _P, C.POINTER(_U32), _U32, _F, _P, _P]),
    "gtm_qkv_epilogue_rows": (_I, [_U32, _U32, _U32, _P, _P, _F, _U32, C.POINTER(_U32), _F, _P, C.POINTER(_U32), _U32,
                                   _U32, _P]),
    "gtm_attention_rows_workspace_bytes": (_SZ, [_U32, _U32, _U32, _U32]),
    "gtm_attention_decode_rows": (_I, [_U32, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, C.POINTER(_U32), _U32,
                                       C.POINTER(_U32), _P, _P, _SZ, _P]),
    "gtm_sampling_validate": (_I, [C.POINTER(Sampling)]),
    "gtm_sampling_splitmix64": (_U64, [_U64]),
    "gtm_sampling_seed_for": (_U64, [C.POINTER(Sampling), _I]),
    "gtm_softcap": (_I, [_U32, _P, _F, _P, _P]),
    "gtm_sample_workspace_bytes": (_SZ, [_U32]),
    "gtm_repetition_penalty": (_I, [_P, _U32, _P, _U32, _F, _F, _P, _SZ, _P]),
    "gtm_sample_token": (_I, [_P, _U32, C.POINTER(Sampling), _U64, _P, _P, _P, _SZ, _P]),
    "gtm_synth_expert_layout": (_I, [_U32, _U32, C.POINTER(_U64), C.POINTER(_U64)]),
    "gtm_synth_resident_layout": (_I, [_U32, _U32, _U32, C.POINTER(_U64), C.POINTER(_U64)]),
    "gtm_synth_experts": (_I, [_U64, _U32, _U32, _U32, _U32, _U32, _P, _P]),
    "gtm_synth_resident": (_I, [_U64, _U32, _U32, _U32, _U32, _P, _P]),
    "gtm_synth_x": (_I, [_U64, _U32, _U32, _U32, _P, _P]),
    "gtm_synth_layer_desc": (_I, [_U32, _U32, _U32, _U32, _P, _P, C.POINTER(Layer)]),
    "gtm_synth_quant": (_I, [_U64, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, _P]),
    "gtm_synth_norm": (_I, [_U64, _U32, _U32, _U32, _P, _P]),
}


def lib():
    """Loads libgtmoe.so. Raises if it has not been built -- there is no fallback path."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libgtmoe.so not built at {LIB_PATH}; run python turbo-winfare_b200/build.py")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().gtm_last_error().decode()


def check(rc: int) -> None:
    if rc != OK:
        raise GtmError(rc, last_error())


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def ptr(t) -> C.c_void_p | None:
    return None if t is None else C.c_void_p(t.data_ptr())


def default_dims() -> Dims:
    return Dims(HIDDEN, MOE_INTER, FFN, EXPERTS, TOP_K, EPS)


# ---- single kernels (the reference's dispatch set) ----------------------------------------------

def gemv_q4(w, s, b, x, out, rows: int, in_dim: int, stream=None):
    check(lib().gtm_gemv_q4(rows, in_dim, ptr(w), ptr(s), ptr(b), ptr(x), ptr(out), _stream(stream)))


def gemv_q8(w, s, b, x, out, rows: int, in_dim: int, stream=None):
    check(lib().gtm_gemv_q8(rows, in_dim, ptr(w), ptr(s), ptr(b), ptr(x), ptr(out), _stream(stream)))


def router_topk(logits, pes, idx, w, k: int, stream=None):
    check(lib().gtm_router_topk(logits.numel(), k, ptr(logits), ptr(pes), ptr(idx), ptr(w), _stream(stream)))


def geglu(g, u, out, stream=None):
    check(lib().gtm_geglu(g.numel(), ptr(g), ptr(u), ptr(out), _stream(stream)))


def scale_accum(inp, weights, w_index: int, accumulate: bool, out, stream=None):
    check(lib().gtm_scale_accum(inp.numel(), ptr(inp), ptr(weights), w_index, int(accumulate), ptr(out), _stream(stream)))


def mul_bf16(inp, w, scale: float, out, stream=None):
    check(lib().gtm_mul_bf16(inp.numel(), ptr(inp), ptr(w), scale, ptr(out), _stream(stream)))


def rmsnorm(x, w, eps: float, out, stream=None):
    check(lib().gtm_rmsnorm(x.numel(), ptr(x), ptr(w), eps, ptr(out), _stream(stream)))


def post_attn(attn, hidden, w_post, w_pre, w_pre2, eps, hidden_out, dense, routed, router, stream=None):
    check(lib().gtm_post_attn(attn.numel(), ptr(attn), ptr(hidden), ptr(w_post), ptr(w_pre), ptr(w_pre2), eps,
                              ptr(hidden_out), ptr(dense), ptr(routed), ptr(router), _stream(stream)))


def layer_tail(h2, h1, hidden, w_pf2, w_pf, eps, layer_scalar, hidden_out, stream=None):
    check(lib().gtm_layer_tail(h2.numel(), ptr(h2), ptr(h1), ptr(hidden), ptr(w_pf2), ptr(w_pf), eps, layer_scalar,
                               ptr(hidden_out), _stream(stream)))


def dispatch(kernel: int, srvs, uavs, constants, grid_x: int = 1, stream=None):
    """gtm_dispatch: the reference's (srv, uav, 16 root constants) convention."""
    srv = (C.c_void_p * max(1, len(srvs)))(*[t.data_ptr() for t in srvs])
    uav = (C.c_void_p * max(1, len(uavs)))(*[t.data_ptr() for t in uavs])
    c = (C.c_uint32 * 16)(*(list(constants) + [0] * (16 - len(constants))))
    check(lib().gtm_dispatch(kernel, srv, len(srvs), uav, len(uavs), c, grid_x, _stream(stream)))


# ---- synthetic model --------------------------------------------------------------------------

def expert_layout(hidden=HIDDEN, inter=MOE_INTER):
    off = (C.c_uint64 * 9)()
    stride = C.c_uint64()
    check(lib().gtm_synth_expert_layout(hidden, inter, off, C.byref(stride)))
    return list(off), stride.value


def resident_layout(hidden=HIDDEN, ffn=FFN, experts=EXPERTS):
    off = (C.c_uint64 * 20)()
    total = C.c_uint64()
    check(lib().gtm_synth_resident_layout(hidden, ffn, experts, off, C.byref(total)))
    return list(off), total.value


class SynthModel:
    """`num_layers` random-init MoE layers resident in HBM in the .gturbo byte layouts."""

    def __init__(self, num_layers: int, seed: int = 0, device: str = "cuda", stream=None):
        import torch
        self.num_layers, self.seed = num_layers, seed
        _, stride = expert_layout()
        _, rtotal = resident_layout()
        self.expert_stride = stride
        self.resident = []
        self.experts = []
        self.layers = (Layer * num_layers)()
        for l in range(num_layers):
            r = torch.empty(rtotal, dtype=torch.uint8, device=device)
            e = torch.empty(EXPERTS * stride, dtype=torch.uint8, device=device)
            check(lib().gtm_synth_resident(seed, l, HIDDEN, FFN, EXPERTS, ptr(r), _stream(stream)))
            check(lib().gtm_synth_experts(seed, l, HIDDEN, MOE_INTER, 0, EXPERTS, ptr(e), _stream(stream)))
            check(lib().gtm_synth_layer_desc(HIDDEN, MOE_INTER, FFN, EXPERTS, ptr(r), ptr(e), C.byref(self.layers[l])))
            self.resident.append(r)
            self.experts.append(e)

    def weight_bytes(self) -> int:
        return sum(t.numel() for t in self.resident) + sum(t.numel() for t in self.experts)


class LmHead:
    """Tied LM head with greedy argmax (gtm_lm_head_greedy) over `rows` vocabulary rows."""

    def __init__(self, rows: int, device: str = "cuda"):
        import torch
        self.rows = rows
        n = lib().gtm_lm_head_workspace_bytes(rows)
        if n == 0:
            raise GtmError(ERR_INVALID, "LM head workspace size query failed")
        self.workspace = torch.empty(n + 256, dtype=torch.uint8, device=device)
        self.ws_ptr = C.c_void_p((self.workspace.data_ptr() + 255) // 256 * 256)
        self.ws_bytes = n

    def __call__(self, w, s, b, x, token, logit=None, stream=None):
        """w: uint8 [rows, hidden/2]; s, b: bf16 bits (int16/uint16) [rows, hidden/64]; x: fp32 [hidden];
        token: int32/uint32 [1] on the device; logit: fp32 [1] or None."""
        check(lib().gtm_lm_head_greedy(self.rows, x.numel(), ptr(w), ptr(s), ptr(b), ptr(x), ptr(token), ptr(logit),
                                       self.ws_ptr, self.ws_bytes, _stream(stream)))

    def candidates(self, stream=None) -> int:
        n = C.c_int32()
        check(lib().gtm_lm_head_candidates(self.ws_ptr, _stream(stream), C.byref(n)))
        return n.value


def synth_x(seed: int, token0: int, count: int, out, stream=None):
    check(lib().gtm_synth_x(seed, token0, count, HIDDEN, ptr(out), _stream(stream)))


class Decoder:
    """Batch-1 decode through a stack of MoE layers: one fused launch per token."""

    def __init__(self, layers, num_layers: int | None = None, device: str = "cuda"):
        import torch
        self.layers = layers
        self.num_layers = num_layers if num_layers is not None else len(layers)
        self.dims = default_dims()
        n = lib().gtm_moe_decode_workspace_bytes(C.byref(self.dims))
        if n == 0:
            raise GtmError(ERR_UNSUPPORTED, "decode workspace size query failed")
        self.workspace = torch.zeros(n + 256, dtype=torch.uint8, device=device)  # zeroed once, as required
        base = self.workspace.data_ptr()
        self.ws_ptr = C.c_void_p((base + 255) // 256 * 256)
        self.ws_bytes = n

    def __call__(self, hidden_in, hidden_out, *, topk_idx=None, topk_w=None, logits=None, h1=None, h2=None,
                 hidden_layers=None, logit_bias=None, norm_between_layers=True, stream=None, first_layer: int = 0,
                 num_layers: int | None = None, extra_flags: int = 0):
        n = num_layers if num_layers is not None else self.num_layers
        layer_arr = C.cast(C.addressof(self.layers) + first_layer * C.sizeof(Layer), C.POINTER(Layer))
        io = DecodeIO(hidden_in.data_ptr(), hidden_out.data_ptr(), ptr(topk_idx), ptr(topk_w), ptr(logits), ptr(h1),
                      ptr(h2), ptr(hidden_layers), ptr(logit_bias),
                      (NORM_BETWEEN_LAYERS if norm_between_layers else 0) | extra_flags)
        check(lib().gtm_moe_decode(C.byref(self.dims), layer_arr, n, C.byref(io), self.ws_ptr, self.ws_bytes,
                                   _stream(stream)))

    def check(self, stream=None):
        check(lib().gtm_moe_decode_check(self.ws_ptr, _stream(stream)))


class TokenBlock:
    """T > 1 tokens through one MoE layer (gtm_moe_tokens), workspace sized for `max_tokens`."""

    def __init__(self, max_tokens: int, device: str = "cuda"):
        import torch
        self.dims = default_dims()
        self.max_tokens = max_tokens
        n = lib().gtm_moe_tokens_workspace_bytes(C.byref(self.dims), max_tokens)
        if n == 0:
            raise GtmError(ERR_UNSUPPORTED, f"tokens workspace size query failed for {max_tokens} tokens")
        self.workspace = torch.zeros(n + 256, dtype=torch.uint8, device=device)  # zeroed once, as required
        base = self.workspace.data_ptr()
        self.ws_ptr = C.c_void_p((base + 255) // 256 * 256)
        self.ws_bytes = n

    def __call__(self, layer: Layer, x, hidden_out, *, topk_idx=None, topk_w=None, logits=None, h1=None, h2=None,
                 logit_bias=None, route_logits=None, stream=None, extra_flags=0):
        """x: [T, hidden] float32 or bfloat16 on the device; hidden_out: [T, hidden] float32."""
        import torch
        T = x.shape[0]
        xf = x if x.dtype == torch.float32 else None
        xb = x if x.dtype == torch.bfloat16 else None
        if xf is None and xb is None:
            raise TypeError("x must be float32 or bfloat16")
        io = TokensIO(T, ptr(xf), ptr(xb), hidden_out.data_ptr(), ptr(topk_idx), ptr(topk_w), ptr(logits), ptr(h1),
                      ptr(h2), ptr(logit_bias), ptr(route_logits), extra_flags)
        check(lib().gtm_moe_tokens(C.byref(self.dims), C.byref(layer), C.byref(io), self.ws_ptr, self.ws_bytes,
                                   _stream(stream)))

    def check(self, stream=None):
        check(lib().gtm_moe_tokens_check(self.ws_ptr, _stream(stream)))



PHASE_EVENTS = 6
PHASE_NAMES = ("views_router", "routing", "gemm_gate_up", "gemm_down", "combine")


def set_phase_events(events) -> None:
    """Stage timing of this thread's next gtm_moe_tokens calls (gtm_set_phase_events): `events`
    are up to PHASE_EVENTS torch.cuda.Event(enable_timing=True) objects, recorded once on the
    current stream first so their handles exist; an empty list turns it off."""
    arr = (C.c_void_p * max(1, len(events)))(*[e.cuda_event for e in events])
    check(lib().gtm_set_phase_events(arr, len(events)))


def decode_noalloc(layers, hidden_in, hidden_out, *, num_layers: int | None = None, first_layer: int = 0,
                   topk_idx=None, topk_w=None, logits=None, h1=None, h2=None, hidden_layers=None, logit_bias=None,
                   norm_between_layers=True, stream=None):
    """gtm_moe_decode_noalloc: the batch-1 decode using the library's static per-device scratch,
    for callers that cannot allocate a workspace (see include/gtmoe.h)."""
    n = num_layers if num_layers is not None else len(layers) - first_layer
    layer_arr = C.cast(C.addressof(layers) + first_layer * C.sizeof(Layer), C.POINTER(Layer))
    io = DecodeIO(hidden_in.data_ptr(), hidden_out.data_ptr(), ptr(topk_idx), ptr(topk_w), ptr(logits), ptr(h1),
                  ptr(h2), ptr(hidden_layers), ptr(logit_bias), NORM_BETWEEN_LAYERS if norm_between_layers else 0)
    dims = default_dims()
    check(lib().gtm_moe_decode_noalloc(C.byref(dims), layer_arr, n, C.byref(io), _stream(stream)))


def decode_noalloc_check(stream=None):
    """Reads and clears the static scratch's device-side error word (synchronises the stream)."""
    check(lib().gtm_moe_decode_noalloc(None, None, 0, None, _stream(stream)))

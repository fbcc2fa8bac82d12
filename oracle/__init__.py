"""TEST INFRASTRUCTURE ONLY -- the CPU checker for the CUDA MoE path.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may import this
package; the product path never does.

Two CPU implementations are exposed:

* ``liboracle.so`` -- the restated MoE block (oracle/moe_oracle.c), which follows the
  reference's scalar FP32 forward (src/cpu_reference.cpp:422-520) operation by operation, the
  restated token sampling (oracle/sampling_oracle.c, src/sampling.cpp:1-171), and the embedding
  lookup and attention step (oracle/attn_oracle.c, src/cpu_reference.cpp:108-140, 322-417);
* ``_ref/libgtref.so`` -- the reference's own src/cpu_reference.cpp helpers and src/sampling.cpp
  compiled from its sources (built only where the reference tree is present; it travels as a
  prebuilt .so).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libgtref.so")

HIDDEN, MOE_INTER, FFN, EXPERTS, TOP_K, EPS = 2816, 704, 2112, 128, 8, 1e-6


def reference_dir(ref_dir: str | None = None) -> str | None:
    """The reference checkout: the argument, else $GTM_REFERENCE_DIR, else a directory named
    `reference` beside this repository; None when none of them holds src/cpu_reference.cpp."""
    cands = [ref_dir] if ref_dir else [os.environ.get("GTM_REFERENCE_DIR"),
                                       os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")]
    for c in cands:
        if c and os.path.isfile(os.path.join(c, "src", "cpu_reference.cpp")):
            return os.path.abspath(c)
    return None


def build(ref_dir: str | None = None) -> None:
    """Builds liboracle.so, and _ref/libgtref.so when the reference sources are present."""
    subprocess.check_call(["make", "-s", "-C", HERE, "oracle"])
    ref = reference_dir(ref_dir)
    if ref is not None:
        subprocess.check_call(["make", "-s", "-C", HERE, "ref", f"REF={ref}"])


class QT(C.Structure):
    _fields_ = [("data", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p),
                ("rows", C.c_uint32), ("in_dim", C.c_uint32), ("bits", C.c_int)]


class Layer(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("moe_inter", C.c_uint32), ("ffn_inter", C.c_uint32),
                ("num_experts", C.c_uint32), ("top_k", C.c_uint32), ("eps", C.c_float),
                ("router", QT), ("router_scale", C.c_void_p), ("per_expert_scale", C.c_void_p),
                ("sh_gate", QT), ("sh_up", QT), ("sh_down", QT),
                ("w_pre", C.c_void_p), ("w_pre2", C.c_void_p), ("w_pf1", C.c_void_p),
                ("w_pf2", C.c_void_p), ("w_pf", C.c_void_p), ("layer_scalar", C.c_uint16),
                ("experts", C.c_void_p), ("expert_stride", C.c_uint64),
                ("sub_off", C.c_uint64 * 9)]


class Sampling(C.Structure):
    """orc_sampling / gtref_sampling (include/gturbo/sampling.hpp:21-30 SamplingParams)."""
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int32),
                ("repetition_penalty", C.c_float), ("has_seed", C.c_int32), ("pad_", C.c_uint32),
                ("seed", C.c_uint64)]


def sampling_params(temperature=0.0, top_p=1.0, top_k=0, repetition_penalty=1.0, seed=None) -> Sampling:
    return Sampling(temperature, top_p, top_k, repetition_penalty, 0 if seed is None else 1, 0,
                    0 if seed is None else seed)


class AttnShape(C.Structure):
    """orc_attn_shape / gtref_attn_shape."""
    _fields_ = [("hidden", C.c_uint32), ("num_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("kv_heads", C.c_uint32), ("rotated_pairs", C.c_uint32), ("theta", C.c_float),
                ("sliding_window", C.c_int32), ("k_eq_v", C.c_int32), ("eps", C.c_float)]


class AttnLayer(C.Structure):
    """orc_attn_layer / gtref_attn_layer."""
    _fields_ = [("q", QT), ("k", QT), ("v", QT), ("o", QT), ("input_norm", C.c_void_p), ("q_norm", C.c_void_p),
                ("k_norm", C.c_void_p)]


class BlockOut(C.Structure):
    _fields_ = [("hidden_out", C.c_void_p), ("h1", C.c_void_p), ("h2", C.c_void_p),
                ("logits", C.c_void_p), ("top_idx", C.c_void_p), ("top_w", C.c_void_p)]


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.orc_bf16.restype = C.c_float
        L.orc_bf16.argtypes = [C.c_uint16]
        L.orc_gelu_tanh.restype = C.c_float
        L.orc_gelu_tanh.argtypes = [C.c_float]
        L.orc_rms_norm.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_float, C.c_void_p]
        L.orc_matvec.argtypes = [C.POINTER(QT), C.c_void_p, C.c_void_p]
        L.orc_topk.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_moe_block.argtypes = [C.POINTER(Layer), C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(BlockOut)]
        L.orc_synth_resident.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p]
        L.orc_synth_expert.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p]
        L.orc_synth_x.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_void_p]
        L.orc_synth_layer_create.restype = C.c_void_p
        L.orc_synth_layer_create.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                             C.c_uint32, C.c_uint32, C.c_float]
        L.orc_synth_layer_destroy.argtypes = [C.c_void_p]
        L.orc_synth_layer_view.restype = C.POINTER(Layer)
        L.orc_synth_layer_view.argtypes = [C.c_void_p]
        L.orc_synth_layer_ensure.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32]
        L.orc_synth_layer_block.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(BlockOut)]
        L.orc_synth_layer_route.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_synth_stack.argtypes = [C.POINTER(C.c_void_p), C.c_uint32, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_embed.argtypes = [C.POINTER(QT), C.c_uint32, C.c_void_p]
        L.orc_rope_neox.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_float, C.c_float]
        L.orc_qkv_epilogue.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_float, C.c_uint32,
                                       C.c_float, C.c_float]
        L.orc_attention_core.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32,
                                         C.c_int, C.c_int, C.c_uint32, C.c_void_p]
        L.orc_attention_step.restype = C.c_int
        L.orc_attention_step.argtypes = [C.POINTER(AttnShape), C.POINTER(AttnLayer), C.c_int, C.c_void_p,
                                         C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_softcap.argtypes = [C.c_void_p, C.c_size_t, C.c_float]
        L.orc_validate_sampling.restype = C.c_int
        L.orc_validate_sampling.argtypes = [C.POINTER(Sampling)]
        L.orc_splitmix64.restype = C.c_uint64
        L.orc_splitmix64.argtypes = [C.c_uint64]
        L.orc_seed_for.restype = C.c_uint64
        L.orc_seed_for.argtypes = [C.POINTER(Sampling), C.c_int]
        L.orc_apply_repetition_penalty.argtypes = [C.c_void_p, C.c_uint32, C.c_void_p, C.c_size_t, C.c_float,
                                                   C.c_float]
        L.orc_sample_token.restype = C.c_int
        L.orc_sample_token.argtypes = [C.c_void_p, C.c_uint32, C.POINTER(Sampling), C.c_uint64,
                                       C.POINTER(C.c_uint32)]
        L.orc_sample_shortlist.restype = C.c_int
        L.orc_sample_shortlist.argtypes = [C.c_void_p, C.c_uint32, C.POINTER(Sampling), C.c_void_p,
                                           C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref():
    """The reference's own compiled helpers (oracle/_ref/libgtref.so)."""
    global _ref
    if _ref is None:
        R = C.CDLL(REF_PATH)
        R.gtref_bf16.restype = C.c_float
        R.gtref_bf16.argtypes = [C.c_uint16]
        R.gtref_gelu_tanh.restype = C.c_float
        R.gtref_gelu_tanh.argtypes = [C.c_float]
        R.gtref_rms_norm.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_float, C.c_void_p]
        R.gtref_matvec.argtypes = [C.POINTER(QT), C.c_void_p, C.c_void_p]
        R.gtref_moe_block.argtypes = [C.POINTER(Layer), C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(BlockOut)]
        R.gtref_embed.argtypes = [C.POINTER(QT), C.c_uint32, C.c_void_p]
        R.gtref_rope_neox.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_float, C.c_float]
        R.gtref_attention_step.restype = C.c_int
        R.gtref_attention_step.argtypes = [C.POINTER(AttnShape), C.POINTER(AttnLayer), C.c_int, C.c_void_p,
                                           C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        R.gtref_generate.restype = C.c_int
        R.gtref_generate.argtypes = [C.c_char_p, C.c_void_p, C.c_uint32, C.c_int, C.c_char_p, C.POINTER(Sampling),
                                     C.c_void_p, C.POINTER(C.c_uint32), C.c_char_p, C.c_size_t]
        R.gtref_validate_sampling.restype = C.c_int
        R.gtref_validate_sampling.argtypes = [C.POINTER(Sampling)]
        R.gtref_splitmix64.restype = C.c_uint64
        R.gtref_splitmix64.argtypes = [C.c_uint64]
        R.gtref_seed_for.restype = C.c_uint64
        R.gtref_seed_for.argtypes = [C.POINTER(Sampling), C.c_int]
        R.gtref_apply_repetition_penalty.argtypes = [C.c_void_p, C.c_uint32, C.c_void_p, C.c_size_t, C.c_float,
                                                     C.c_float]
        R.gtref_sample_token.restype = C.c_int
        R.gtref_sample_token.argtypes = [C.c_void_p, C.c_uint32, C.POINTER(Sampling), C.c_uint64,
                                         C.POINTER(C.c_uint32)]
        _ref = R
    return _ref


# ---- numpy-facing helpers ------------------------------------------------------------------

def matvec(w: np.ndarray, s: np.ndarray, b: np.ndarray, x: np.ndarray, rows: int, in_dim: int,
           bits: int, impl: str = "oracle") -> np.ndarray:
    """out[r] = sum_c (q[r][c] * s + b) * x[c] in the reference's accumulation order."""
    w = np.ascontiguousarray(w); s = np.ascontiguousarray(s, dtype=np.uint16)
    b = np.ascontiguousarray(b, dtype=np.uint16); x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(rows, np.float32)
    qt = QT(w.ctypes.data, s.ctypes.data, b.ctypes.data, rows, in_dim, bits)
    if impl == "ref":
        ref().gtref_matvec(C.byref(qt), _ptr(x), _ptr(out))
    else:
        lib().orc_matvec(C.byref(qt), _ptr(x), _ptr(out))
    return out


def rms_norm(x: np.ndarray, w: np.ndarray | None, eps: float = EPS, impl: str = "oracle") -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    wa = None if w is None else np.ascontiguousarray(w, dtype=np.uint16)
    out = np.zeros_like(x)
    f = ref().gtref_rms_norm if impl == "ref" else lib().orc_rms_norm
    f(_ptr(x), _ptr(wa), x.size, eps, _ptr(out))
    return out


def gelu_tanh(x: np.ndarray, impl: str = "oracle") -> np.ndarray:
    f = ref().gtref_gelu_tanh if impl == "ref" else lib().orc_gelu_tanh
    return np.array([f(float(v)) for v in np.asarray(x, np.float32)], np.float32)


def topk(logits: np.ndarray, k: int, per_expert_scale: np.ndarray):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    pes = np.ascontiguousarray(per_expert_scale, dtype=np.uint16)
    idx = np.zeros(k, np.uint32)
    w = np.zeros(k, np.float32)
    lib().orc_topk(_ptr(logits), logits.size, k, _ptr(pes), _ptr(idx), _ptr(w))
    return idx, w


def synth_x(seed: int, token: int, hidden: int = HIDDEN) -> np.ndarray:
    x = np.zeros(hidden, np.float32)
    lib().orc_synth_x(seed, token, hidden, _ptr(x))
    return x


class SynthLayer:
    """One synthetic MoE layer on the host, generated by the same counter RNG as the GPU side."""

    def __init__(self, seed: int, layer: int, hidden=HIDDEN, moe_inter=MOE_INTER, ffn=FFN,
                 experts=EXPERTS, top_k=TOP_K, eps=EPS):
        self.hidden, self.top_k, self.experts, self.eps = hidden, top_k, experts, eps
        self.h = lib().orc_synth_layer_create(seed, layer, hidden, moe_inter, ffn, experts, top_k, eps)
        if not self.h:
            raise MemoryError("orc_synth_layer_create failed")

    def close(self):
        if self.h:
            lib().orc_synth_layer_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def view(self):
        return lib().orc_synth_layer_view(self.h)

    def ensure(self, experts):
        e = np.ascontiguousarray(np.asarray(experts, dtype=np.uint32))
        lib().orc_synth_layer_ensure(self.h, _ptr(e), e.size)

    def route(self, hidden_in, logit_bias=None, route_logits=None) -> np.ndarray:
        """Views, router and top-k only (the selected experts are generated): the top-k ids."""
        x = np.ascontiguousarray(hidden_in, dtype=np.float32)
        lb = None if logit_bias is None else np.ascontiguousarray(logit_bias, dtype=np.float32)
        rl = None if route_logits is None else np.ascontiguousarray(route_logits, dtype=np.float32)
        idx = np.zeros(self.top_k, np.uint32)
        lib().orc_synth_layer_route(self.h, _ptr(x), _ptr(lb), _ptr(rl), _ptr(idx))
        return idx

    def block(self, hidden_in, logit_bias=None, route_logits=None, impl: str = "oracle"):
        """Runs the MoE block for one token. impl='ref' runs the reference's compiled helpers."""
        D, K = self.hidden, self.top_k
        x = np.ascontiguousarray(hidden_in, dtype=np.float32)
        lb = None if logit_bias is None else np.ascontiguousarray(logit_bias, dtype=np.float32)
        rl = None if route_logits is None else np.ascontiguousarray(route_logits, dtype=np.float32)
        res = {"hidden": np.zeros(D, np.float32), "h1": np.zeros(D, np.float32), "h2": np.zeros(D, np.float32),
               "logits": np.zeros(self.experts, np.float32), "idx": np.zeros(K, np.uint32),
               "w": np.zeros(K, np.float32)}
        out = BlockOut(res["hidden"].ctypes.data, res["h1"].ctypes.data, res["h2"].ctypes.data,
                       res["logits"].ctypes.data, res["idx"].ctypes.data, res["w"].ctypes.data)
        if impl == "ref":
            # route first (views + router only) to learn which experts to materialise
            lib().orc_synth_layer_route(self.h, _ptr(x), _ptr(lb), _ptr(rl), None)
            ref().gtref_moe_block(self.view(), _ptr(x), _ptr(lb), _ptr(rl), C.byref(out))
        else:
            lib().orc_synth_layer_block(self.h, _ptr(x), _ptr(lb), _ptr(rl), C.byref(out))
        return res


def synth_stack(layers: list[SynthLayer], hidden_in: np.ndarray):
    """A stack of synthetic layers with a weightless RMSNorm between layers."""
    n = len(layers)
    D, K = layers[0].hidden, layers[0].top_k
    arr = (C.c_void_p * n)(*[l.h for l in layers])
    x = np.ascontiguousarray(hidden_in, dtype=np.float32)
    out = np.zeros(D, np.float32)
    per = np.zeros((n, D), np.float32)
    idx = np.zeros((n, K), np.uint32)
    w = np.zeros((n, K), np.float32)
    lib().orc_synth_stack(arr, n, _ptr(x), _ptr(out), _ptr(per), _ptr(idx), _ptr(w))
    return {"hidden": out, "hidden_per_layer": per, "idx": idx, "w": w}


# ---- token sampling (src/sampling.cpp) ------------------------------------------------------

def _slib(impl: str):
    return (lib(), "orc_") if impl == "oracle" else (ref(), "gtref_")


def validate_sampling(p: Sampling, impl: str = "oracle") -> int:
    """0 when accepted; otherwise the oracle's rule code, or 1 from the reference."""
    L, pre = _slib(impl)
    return getattr(L, pre + "validate_sampling")(C.byref(p))


def splitmix64(x: int, impl: str = "oracle") -> int:
    L, pre = _slib(impl)
    return getattr(L, pre + "splitmix64")(x)


def seed_for(p: Sampling, position: int, impl: str = "oracle") -> int:
    L, pre = _slib(impl)
    return getattr(L, pre + "seed_for")(C.byref(p), position)


def apply_repetition_penalty(logits: np.ndarray, history, penalty: float, softcap: float,
                             impl: str = "oracle") -> np.ndarray:
    """Returns a penalised copy of fp32 logits."""
    L, pre = _slib(impl)
    out = np.ascontiguousarray(logits, dtype=np.float32).copy()
    h = np.ascontiguousarray(history, dtype=np.uint32)
    getattr(L, pre + "apply_repetition_penalty")(_ptr(out), out.size, _ptr(h) if h.size else None, h.size,
                                                 penalty, softcap)
    return out


def sample_token(logits: np.ndarray, p: Sampling, seed: int, impl: str = "oracle") -> tuple[int, int]:
    """(status, token): status 0 with a token, else the failure code (token -1)."""
    L, pre = _slib(impl)
    x = np.ascontiguousarray(logits, dtype=np.float32)
    tok = C.c_uint32(0)
    rc = getattr(L, pre + "sample_token")(_ptr(x) if x.size else None, x.size, C.byref(p), seed, C.byref(tok))
    return rc, (tok.value if rc == 0 else -1)


def sample_shortlist(logits: np.ndarray, p: Sampling) -> tuple[int, np.ndarray, int]:
    """(status, shortlist ids in candidate order, survivors after the nucleus and top-k cuts)."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    ids = np.zeros(256, dtype=np.uint32)
    n, cut = C.c_uint32(0), C.c_uint32(0)
    rc = lib().orc_sample_shortlist(_ptr(x) if x.size else None, x.size, C.byref(p), _ptr(ids), C.byref(n),
                                    C.byref(cut))
    return rc, ids[:n.value].copy(), cut.value


def synth_logits(seed: int, vocab: int, scale: float = 4.0, step: float = 0.0) -> np.ndarray:
    """Deterministic fp32 logits from integer arithmetic only (splitmix64 per index, four 24-bit
    uniforms summed: roughly normal with std ~`scale`), so a fixture can name them by (seed,
    vocab, scale, step) instead of storing them. step > 0 rounds to multiples of step, which makes
    many exact ties."""
    i = np.arange(vocab, dtype=np.uint64)
    acc = np.zeros(vocab, dtype=np.float64)
    with np.errstate(over="ignore"):
        for j in range(4):
            z = i * np.uint64(4) + np.uint64(j) + np.uint64(seed) * np.uint64(0x9E3779B97F4A7C15)
            z = z + np.uint64(0x9E3779B97F4A7C15)
            z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
            z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
            z = z ^ (z >> np.uint64(31))
            acc += (z >> np.uint64(40)).astype(np.float64) * 2.0 ** -24 - 0.5
    v = acc * (scale * 3.0 ** 0.5)   # sum of 4 U(-1/2, 1/2) has variance 1/3
    if step > 0:
        v = np.round(v / step) * step
    return v.astype(np.float32)


# ---- embedding lookup and attention step (src/cpu_reference.cpp:108-140, 322-417) -------------

SWA_SHAPE = dict(num_heads=16, head_dim=256, kv_heads=8, theta=10000.0, k_eq_v=0)        # sliding-window layers
FULL_SHAPE = dict(num_heads=16, head_dim=512, kv_heads=2, theta=1000000.0, k_eq_v=1)     # layers 5, 11, 17, 23, 29


def attn_shape(full: bool, sliding_window: int = 1024, hidden: int = HIDDEN, **over) -> AttnShape:
    """The manifest's defaults (include/gturbo/manifest.hpp:22-49): full layers rotate
    head_dim * 0.25 / 2 pairs and attend to every position; sliding layers rotate all pairs."""
    d = dict(FULL_SHAPE if full else SWA_SHAPE)
    d.update(over)
    pairs = int(d["head_dim"] * 0.25 / 2.0) if full else d["head_dim"] // 2
    return AttnShape(hidden, d["num_heads"], d["head_dim"], d["kv_heads"], pairs, d["theta"],
                     0 if full else sliding_window, d["k_eq_v"], EPS)


def _synth_u64(seed: int, n: int, stream: int) -> np.ndarray:
    i = np.arange(n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = i + np.uint64(seed) * np.uint64(0x9E3779B97F4A7C15) + np.uint64(stream) * np.uint64(0xD1B54A32D192ED03)
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


def synth_quant(seed: int, stream: int, rows: int, in_dim: int, scale: float) -> dict:
    """A deterministic int4 MLX-affine matrix (integer arithmetic only): packed bytes, and bf16
    scales / biases of about `scale` so a row's outputs stay O(1)."""
    g = in_dim // 64
    w = (_synth_u64(seed, rows * in_dim // 2, stream) & np.uint64(0xFF)).astype(np.uint8).reshape(rows, in_dim // 2)
    r = _synth_u64(seed, 2 * rows * g, stream + 1)
    u = (r >> np.uint64(40)).astype(np.float64) * 2.0 ** -24
    s = _bf16_bits((scale * (0.5 + u[:rows * g])).reshape(rows, g))
    b = _bf16_bits((-7.5 * scale * (0.5 + u[rows * g:])).reshape(rows, g))
    return {"w": w, "s": s, "b": b, "rows": rows, "in_dim": in_dim}


def synth_norm(seed: int, stream: int, n: int) -> np.ndarray:
    u = (_synth_u64(seed, n, stream) >> np.uint64(40)).astype(np.float64) * 2.0 ** -24
    return _bf16_bits(0.5 + u)


class AttnWeights:
    """Synthetic weights of one attention layer with the shape `s` (q/k/v/o int4, bf16 norms)."""

    def __init__(self, seed: int, s: AttnShape):
        D, hd, H, KV = s.hidden, s.head_dim, s.num_heads, s.kv_heads
        self.shape = s
        self.q = synth_quant(seed, 10, H * hd, D, 0.02)
        self.k = synth_quant(seed, 20, KV * hd, D, 0.02)
        self.v = synth_quant(seed, 30, KV * hd, D, 0.02)
        self.o = synth_quant(seed, 40, D, H * hd, 0.01)
        self.input_norm = synth_norm(seed, 50, D)
        self.q_norm = synth_norm(seed, 60, hd)
        self.k_norm = synth_norm(seed, 70, hd)

    @staticmethod
    def _qt(m: dict) -> QT:
        return QT(_ptr(m["w"]), _ptr(m["s"]), _ptr(m["b"]), m["rows"], m["in_dim"], 4)

    def view(self) -> AttnLayer:
        return AttnLayer(self._qt(self.q), self._qt(self.k), self._qt(self.v), self._qt(self.o),
                         _ptr(self.input_norm), _ptr(self.q_norm), _ptr(self.k_norm))


def attention_steps(w: AttnWeights, hiddens: np.ndarray, impl: str = "oracle") -> dict:
    """Runs positions 0..n-1 through one layer (each row of `hiddens` is that position's input);
    returns the per-position attn outputs and q/k/v vectors, and the final caches."""
    s = w.shape
    n = hiddens.shape[0]
    kn, qn = s.kv_heads * s.head_dim, s.num_heads * s.head_dim
    kc = np.zeros((n, kn), np.float32)
    vc = np.zeros((n, kn), np.float32)
    out = {"attn": np.zeros((n, s.hidden), np.float32), "q": np.zeros((n, qn), np.float32),
           "k": np.zeros((n, kn), np.float32), "v": np.zeros((n, kn), np.float32)}
    L, fn = (lib(), "orc_attention_step") if impl == "oracle" else (ref(), "gtref_attention_step")
    view = w.view()
    for p in range(n):
        x = np.ascontiguousarray(hiddens[p], dtype=np.float32)
        getattr(L, fn)(C.byref(s), C.byref(view), p, _ptr(x), _ptr(kc), _ptr(vc), _ptr(out["attn"][p]),
                       _ptr(out["q"][p]), _ptr(out["k"][p]), _ptr(out["v"][p]))
    out["k_cache"], out["v_cache"] = kc, vc
    return out


def embed(m: dict, token: int, impl: str = "oracle") -> np.ndarray:
    out = np.zeros(m["in_dim"], np.float32)
    L, fn = (lib(), "orc_embed") if impl == "oracle" else (ref(), "gtref_embed")
    qt = AttnWeights._qt(m)
    getattr(L, fn)(C.byref(qt), token, _ptr(out))
    return out


def rope_neox(vec: np.ndarray, head_dim: int, pairs: int, position: float, theta: float, impl: str = "oracle"):
    out = np.ascontiguousarray(vec, dtype=np.float32).copy()
    L, fn = (lib(), "orc_rope_neox") if impl == "oracle" else (ref(), "gtref_rope_neox")
    getattr(L, fn)(_ptr(out), head_dim, pairs, position, theta)
    return out


def qkv_epilogue(vec: np.ndarray, heads: int, head_dim: int, w, eps: float, pairs: int, position: float,
                 theta: float) -> np.ndarray:
    out = np.ascontiguousarray(vec, dtype=np.float32).copy()
    lib().orc_qkv_epilogue(_ptr(out), heads, head_dim, _ptr(w), eps, pairs, position, theta)
    return out


def attention_core(q, k_cache, v_cache, q_heads: int, kv_heads: int, head_dim: int, n_pos: int, first: int,
                   capacity: int) -> np.ndarray:
    ctx = np.zeros(q_heads * head_dim, np.float32)
    q, k_cache, v_cache = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k_cache, v_cache))
    lib().orc_attention_core(_ptr(q), _ptr(k_cache), _ptr(v_cache), q_heads, kv_heads, head_dim, n_pos, first,
                             capacity, _ptr(ctx))
    return ctx


def softcap(z: np.ndarray, cap: float) -> np.ndarray:
    out = np.ascontiguousarray(z, dtype=np.float32).copy()
    lib().orc_softcap(_ptr(out), out.size, cap)
    return out


def ref_generate(model_dir: str, prompt, max_tokens: int, dump_dir: str | None = None,
                 sampling: Sampling | None = None) -> list[int]:
    """The reference's CpuReference::generate on a bundle directory: greedy, or with `sampling`
    (a seed of 0 means none there, as CpuGenerationOptions has it); with dump_dir, its per-stage
    tensors of the first prompt token are written there."""
    p = np.ascontiguousarray(prompt, dtype=np.uint32)
    out = np.zeros(max_tokens + 1, np.uint32)
    n = C.c_uint32(0)
    err = C.create_string_buffer(512)
    dd = None if dump_dir is None else dump_dir.encode()
    sp = None if sampling is None else C.byref(sampling)
    if ref().gtref_generate(model_dir.encode(), _ptr(p), p.size, max_tokens, dd, sp, _ptr(out), C.byref(n), err,
                            512) != 0:
        raise RuntimeError("reference generate failed: " + err.value.decode())
    return [int(t) for t in out[:n.value]]


# ---- the whole decoder: embedding, per layer attention + MoE block, final norm, LM head ------

class SynthDecoder:
    """A synthetic Gemma-4-shaped decoder on the host, composed from the oracle's pieces in the
    order of CpuReference::forward (src/cpu_reference.cpp:313-540): embedding x sqrt(D); per
    layer the attention step, the post-attention norm added to the residual, and the MoE block;
    then the final norm, the tied LM head and the softcap. Greedy decoding follows
    CpuReference::generate (:544-595). Layer l is full-attention when full_mask[l] is 1."""

    SOFTCAP = 30.0

    def __init__(self, num_layers: int = 2, vocab: int = 1024, sliding_window: int = 3, seed: int = 0,
                 full_mask=None, embed_scale: float = 0.002):
        self.num_layers, self.vocab, self.window, self.seed = num_layers, vocab, sliding_window, seed
        self.full_mask = list(full_mask) if full_mask is not None else [l % 2 for l in range(num_layers)]
        self.moe = [SynthLayer(seed, l) for l in range(num_layers)]
        self.attn = [AttnWeights(1000 + 37 * seed + l, attn_shape(bool(self.full_mask[l]), sliding_window))
                     for l in range(num_layers)]
        self.post_attn = [synth_norm(seed, 2000 + l, HIDDEN) for l in range(num_layers)]
        # small embedding values, so that the layers and not the token's own row decide the argmax
        self.embed_w = synth_quant(seed, 3000, vocab, HIDDEN, embed_scale)
        self.final_norm = synth_norm(seed, 3001, HIDDEN)
        self.used = [set() for _ in range(num_layers)]
        self.reset(64)

    def reset(self, max_pos: int) -> None:
        self.caches = []
        for a in self.attn:
            kn = a.shape.kv_heads * a.shape.head_dim
            self.caches.append((np.zeros((max_pos, kn), np.float32), np.zeros((max_pos, kn), np.float32)))

    def forward(self, token: int, pos: int, trace: dict | None = None) -> np.ndarray:
        """Softcapped logits; `trace` receives the stages the reference dumps (embed,
        layerN_hidden, final_norm, logits)."""
        hidden = embed(self.embed_w, token)
        if trace is not None:
            trace["embed"] = hidden.copy()
        for l in range(self.num_layers):
            a = self.attn[l]
            kc, vc = self.caches[l]
            attn = np.zeros(HIDDEN, np.float32)
            view = a.view()
            lib().orc_attention_step(C.byref(a.shape), C.byref(view), pos, _ptr(hidden), _ptr(kc), _ptr(vc),
                                     _ptr(attn), None, None, None)
            hidden = (hidden + rms_norm(attn, self.post_attn[l])).astype(np.float32)
            r = self.moe[l].block(hidden)
            self.used[l].update(int(e) for e in r["idx"])
            hidden = r["hidden"]
            if trace is not None:
                trace[f"layer{l}_hidden"] = hidden.copy()
        normed = rms_norm(hidden, self.final_norm)
        e = self.embed_w
        logits = softcap(matvec(e["w"], e["s"], e["b"], normed, e["rows"], e["in_dim"], 4), self.SOFTCAP)
        if trace is not None:
            trace["final_norm"], trace["logits"] = normed, logits
        return logits

    def sample(self, prompt, max_tokens: int, p: Sampling, stops=(1, 106, 50)) -> list[int]:
        """CpuReference::generate with sampling (src/cpu_reference.cpp:544-595): the penalty over
        the prompt and the tokens so far on the softcapped logits, then sample_token with the
        generator state seed_for(p, position of the next token)."""
        assert validate_sampling(p) == 0
        self.reset(len(prompt) + max_tokens + 1)
        logits = None
        for i, t in enumerate(prompt):
            logits = self.forward(int(t), i)
        history = [int(t) for t in prompt] if p.repetition_penalty != 1.0 else []
        out, pos = [], len(prompt)
        for step in range(max_tokens):
            pen = apply_repetition_penalty(logits, history, p.repetition_penalty, self.SOFTCAP)
            rc, nxt = sample_token(pen, p, seed_for(p, pos))
            if rc != 0:
                raise ValueError(f"sample_token failed ({rc})")
            if nxt in stops:
                break
            out.append(nxt)
            if p.repetition_penalty != 1.0:
                history.append(nxt)
            if step + 1 >= max_tokens:
                break
            logits = self.forward(nxt, pos)
            pos += 1
        return out

    def greedy(self, prompt, max_tokens: int, stops=(1, 106, 50), trace: dict | None = None) -> list[int]:
        """Prompt prefilled token by token, then greedy tokens (argmax, ties to the lower id)
        until max_tokens or a stop id, as CpuReference::generate does; `trace` gets the first
        prompt token's stages."""
        self.reset(len(prompt) + max_tokens + 1)
        logits = None
        for i, t in enumerate(prompt):
            logits = self.forward(int(t), i, trace if i == 0 else None)
        out, pos = [], len(prompt)
        for step in range(max_tokens):
            nxt = int(np.argmax(logits))
            if nxt in stops:
                break
            out.append(nxt)
            if step + 1 >= max_tokens:
                break
            logits = self.forward(nxt, pos)
            pos += 1
        return out

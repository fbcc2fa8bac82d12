"""`.gturbo` bundles through the C ABI (include/gtmoe_bundle.h): open and validate a bundle
directory, load resident.bin and a layer's experts straight into device memory, and describe a
layer for the MoE kernels.

    b = Bundle("/models/gemma-4-26b-a4b.gturbo")
    resident = b.load_resident()                   # uint8 device tensor, resident.bin as is
    experts = b.load_experts(layer=0)              # all 128 experts of layer 0 (or a rank's range)
    layer = b.layer_desc(0, resident, experts)     # gtmoe.Layer for TokenBlock / Decoder / EP ops

This replaces the engine's bundle upload (src/runner.cpp:248-292) and its NVMe expert streamer
(src/streamer.cpp) for the MoE path: every expert is resident in HBM.
"""
from __future__ import annotations

import ctypes as C

from . import BundleInfo, GtmError, Layer, check, lib


class Bundle:
    def __init__(self, path: str):
        self._h = C.c_void_p()
        check(lib().gtm_bundle_open(str(path).encode(), C.byref(self._h)))
        self.info = BundleInfo()
        check(lib().gtm_bundle_info(self._h, C.byref(self.info)))

    def close(self):
        if self._h:
            check(lib().gtm_bundle_close(self._h))
            self._h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _need_open(self):
        if not self._h:
            raise GtmError(-1, "bundle is closed")

    def load_resident(self, out=None, device: str = "cuda"):
        """resident.bin into a uint8 device tensor (allocated when `out` is None). Blocking."""
        import torch
        self._need_open()
        n = self.info.resident_bytes
        if out is None:
            out = torch.empty(n, dtype=torch.uint8, device=device)
        check(lib().gtm_bundle_load_resident(self._h, C.c_void_p(out.data_ptr()), out.numel() * out.element_size()))
        return out

    def load_experts(self, layer: int, first: int = 0, count: int | None = None, out=None, device: str = "cuda"):
        """Experts [first, first + count) of `layer`, expert e at (e - first) * stride. Blocking."""
        import torch
        self._need_open()
        if count is None:
            count = self.info.experts_per_layer - first
        n = count * self.info.expert_stride
        if out is None:
            out = torch.empty(n, dtype=torch.uint8, device=device)
        check(lib().gtm_bundle_load_experts(self._h, layer, first, count, C.c_void_p(out.data_ptr()),
                                            out.numel() * out.element_size()))
        return out

    def layer_desc(self, layer: int, resident, experts) -> Layer:
        """GtmLayer for `layer` over the loaded resident image and the layer's loaded experts."""
        self._need_open()
        L = Layer()
        check(lib().gtm_bundle_layer_desc(self._h, layer, C.c_void_p(resident.data_ptr()),
                                          C.c_void_p(experts.data_ptr()), C.byref(L)))
        return L

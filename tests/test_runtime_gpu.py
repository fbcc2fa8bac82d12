"""Device context / buffer / fence entry points (the D3D12Context replacement) through the C ABI."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import gtmoe  # noqa: E402


def test_context_buffers_and_fences_round_trip():
    L = gtmoe.lib()
    ctx = C.c_void_p()
    gtmoe.check(L.gtm_ctx_create(0, C.byref(ctx)))
    try:
        assert L.gtm_ctx_stream(ctx)
        n = 1 << 20
        host = np.random.default_rng(0).integers(0, 255, n, dtype=np.uint8)
        back = np.zeros(n, np.uint8)
        dev = C.c_void_p()
        gtmoe.check(L.gtm_buffer_alloc(ctx, 2 * n, C.byref(dev)))
        gtmoe.check(L.gtm_buffer_upload(ctx, dev, n, host.ctypes.data, n))     # at a byte offset
        gtmoe.check(L.gtm_buffer_download(ctx, back.ctypes.data, dev, n, n))
        t = C.c_uint64()
        gtmoe.check(L.gtm_submit(ctx, C.byref(t)))
        assert t.value == 1
        gtmoe.check(L.gtm_wait(ctx, t.value, 10000))
        assert np.array_equal(back, host)
        # many tickets: old ones (past the kept fences) still wait correctly
        for _ in range(100):
            gtmoe.check(L.gtm_submit(ctx, C.byref(t)))
        gtmoe.check(L.gtm_wait(ctx, 2, 10000))
        gtmoe.check(L.gtm_wait(ctx, t.value, 10000))
        # a ticket that was never issued is an error, not a hang
        assert L.gtm_wait(ctx, t.value + 5, 10) == gtmoe.ERR_INVALID
        assert "not issued" in gtmoe.last_error()
        gtmoe.check(L.gtm_buffer_free(ctx, dev))
    finally:
        gtmoe.check(L.gtm_ctx_destroy(ctx))


def test_context_rejects_bad_device():
    L = gtmoe.lib()
    ctx = C.c_void_p()
    assert L.gtm_ctx_create(10_000, C.byref(ctx)) == gtmoe.ERR_INVALID

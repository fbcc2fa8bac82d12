"""GPU parity of the reference's MoE kernels through the C ABI (libgtmoe.so), on the
known-answer cases of the reference's tests/test_gpu_kernels.cpp.

Tolerance: that test's allclose (ATOL 1e-5, RTOL 1e-4; test_gpu_kernels.cpp:80-81). Where the
CUDA kernel evaluates the same float operations in the same order as src/cpu_reference.cpp
(GEMVs, norms, MulBF16, ScaleAccum, PostAttn, LayerTail) the result must also be bit-identical
with the CPU oracle; GeGLU and the routing softmax use CUDA's tanhf/expf and are checked by
tolerance only. Router indices are exact, including the forced 11/70 tie.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import gtmoe  # noqa: E402

ATOL, RTOL = 1e-5, 1e-4


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda()
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).cuda()
    return torch.from_numpy(a).cuda()


def host(t, dtype=np.float32):
    torch.cuda.synchronize()
    return t.cpu().numpy().view(dtype)


def assert_allclose(got, want):
    got = np.asarray(got, np.float64); want = np.asarray(want, np.float64)
    excess = np.abs(got - want) - (ATOL + RTOL * np.abs(want))
    assert excess.max() <= 0, f"max abs err {np.abs(got - want).max()}"


@pytest.mark.parametrize("name", ["gemv_int4", "gemv_int8"])
def test_gemv(golden, name):
    k = golden["kat"]
    rows, in_dim, bits = (int(v) for v in k[name + ".shape"])
    w, s, b, x = dev(k[name + ".w"]), dev(k[name + ".s"]), dev(k[name + ".b"]), dev(k[name + ".x"])
    out = torch.full((rows,), np.nan, dtype=torch.float32, device="cuda")
    (gtmoe.gemv_q4 if bits == 4 else gtmoe.gemv_q8)(w, s, b, x, out, rows, in_dim)
    got = host(out)
    assert_allclose(got, k[name + ".want"])
    assert np.array_equal(got, golden["ref"][name + ".ref_out"]), "not bit-identical with the CPU reference"


def test_gemv_through_dispatch_with_byte_offsets(golden):
    """GemvInt4 through gtm_dispatch: one raw buffer with byte offsets, like the runner's RES."""
    k = golden["kat"]
    rows, in_dim, _ = (int(v) for v in k["gemv_int4.shape"])
    parts = [k["gemv_int4.w"].view(np.uint8), k["gemv_int4.s"].view(np.uint8), k["gemv_int4.b"].view(np.uint8)]
    offs, blob = [], bytearray()
    for p in parts:
        blob += b"\0" * ((-len(blob)) % 256)
        offs.append(len(blob))
        blob += p.tobytes()
    res = dev(np.frombuffer(bytes(blob), np.uint8).copy())
    x = dev(k["gemv_int4.x"])
    out = torch.zeros(rows + 16, dtype=torch.float32, device="cuda")
    # two chunks through row_base, as the runner does for > 65535 rows (runner.cpp:431-442)
    for base, cnt in ((0, 50), (50, rows - 50)):
        gtmoe.dispatch(gtmoe.KERNEL_GEMV_INT4, [res, res, res, x], [out],
                       [rows, in_dim, offs[0], offs[1], offs[2], 0, 16 * 4, base], grid_x=cnt)
    got = host(out)[16:16 + rows]
    assert np.array_equal(got, golden["ref"]["gemv_int4.ref_out"])


def test_rmsnorm(golden):
    k = golden["kat"]
    x, w = dev(k["rmsnorm.x"]), dev(k["rmsnorm.w"])
    out = torch.empty_like(x)
    gtmoe.rmsnorm(x, None, 1e-6, out)
    assert_allclose(host(out), k["rmsnorm.want_nw"])
    assert np.array_equal(host(out), k["rmsnorm.want_nw"])
    gtmoe.rmsnorm(x, w, 1e-6, out)
    assert np.array_equal(host(out), golden["ref"]["rmsnorm.ref_w"])


def test_rmsnorm_through_dispatch(golden):
    k = golden["kat"]
    x, w = dev(k["rmsnorm.x"]), dev(k["rmsnorm.w"])
    out = torch.empty_like(x)
    eps_bits = int(np.array([1e-6], np.float32).view(np.uint32)[0])
    gtmoe.dispatch(gtmoe.KERNEL_RMSNORMK, [x, w], [out], [x.numel(), 0, 0, 0, 1, eps_bits])
    assert np.array_equal(host(out), golden["ref"]["rmsnorm.ref_w"])


def test_geglu(golden):
    k = golden["kat"]
    g, u = dev(k["geglu.g"]), dev(k["geglu.u"])
    out = torch.empty_like(g)
    gtmoe.geglu(g, u, out)
    assert_allclose(host(out), k["geglu.want"])


def test_mul_bf16(golden):
    k = golden["kat"]
    x, w = dev(k["mulbf16.x"]), dev(k["mulbf16.w"])
    out = torch.empty_like(x)
    gtmoe.mul_bf16(x, w, float(k["mulbf16.scale"][0]), out)
    assert np.array_equal(host(out), k["mulbf16.want"])


def test_scale_accum_first_write_overwrites(golden):
    k = golden["kat"]
    ins = k["scaleaccum.in"].reshape(8, -1)
    weights = dev(k["scaleaccum.weights"])
    out = torch.full((ins.shape[1],), 12345.0, dtype=torch.float32, device="cuda")   # pre-dirtied
    for j in range(8):
        gtmoe.scale_accum(dev(ins[j]), weights, j, j > 0, out)
    assert_allclose(host(out), k["scaleaccum.want"])
    assert np.array_equal(host(out), k["scaleaccum.want"])


def test_router_topk_tie_to_lower_index(golden):
    k = golden["kat"]
    logits, pes = dev(k["topk.logits"]), dev(k["topk.pes"])
    idx = torch.zeros(8, dtype=torch.int32, device="cuda")
    w = torch.zeros(8, dtype=torch.float32, device="cuda")
    gtmoe.router_topk(logits, pes, idx, w, 8)
    assert np.array_equal(host(idx, np.uint32), k["topk.want_idx"])
    assert_allclose(host(w), k["topk.want_w"])


def test_post_attn(golden):
    k = golden["kat"]
    attn, hid = dev(k["postattn.attn"]), dev(k["postattn.hidden"])
    outs = [torch.empty_like(attn) for _ in range(4)]
    gtmoe.post_attn(attn, hid, dev(k["postattn.w_post"]), dev(k["postattn.w_pre"]), dev(k["postattn.w_pre2"]), 1e-6,
                    *outs)
    for o, key in zip(outs, ("hidden", "dense", "routed", "router")):
        want = k["postattn.want_" + key]
        assert_allclose(host(o), want)
        assert np.array_equal(host(o), want), key


def test_post_attn_in_place_hidden(golden):
    """The runner binds the residual as both input and output (runner.cpp:543-546)."""
    k = golden["kat"]
    attn, hid = dev(k["postattn.attn"]), dev(k["postattn.hidden"])
    d, r, x = torch.empty_like(attn), torch.empty_like(attn), torch.empty_like(attn)
    gtmoe.post_attn(attn, hid, dev(k["postattn.w_post"]), dev(k["postattn.w_pre"]), dev(k["postattn.w_pre2"]), 1e-6,
                    hid, d, r, x)
    assert np.array_equal(host(hid), k["postattn.want_hidden"])
    assert np.array_equal(host(x), k["postattn.want_router"])


def test_layer_tail(golden):
    k = golden["kat"]
    out = torch.empty(2816, dtype=torch.float32, device="cuda")
    gtmoe.layer_tail(dev(k["layertail.h2"]), dev(k["layertail.h1"]), dev(k["layertail.hidden"]),
                     dev(k["layertail.w_pf2"]), dev(k["layertail.w_pf"]), 1e-6, float(k["layertail.scalar"][0]), out)
    assert_allclose(host(out), k["layertail.want"])
    assert np.array_equal(host(out), k["layertail.want"])

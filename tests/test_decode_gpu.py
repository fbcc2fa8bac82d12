"""GPU parity of the fused batch-1 MoE decode (gtm_moe_decode) against the CPU oracle.

Gates (north star): top-8 expert indices bit-exact (ties to the lower index) and router logits
bit-identical given the same block input; routing weights within 1e-5 relative; h1, h2 and the
new residual within max|y - ref| <= 2e-3 * RMS(ref).

Configurations: BASELINE config 0 (one layer, seed 0, several tokens) and config 1 (30 layers
with a weightless RMSNorm between layers). For the stack, routing exactness is checked per layer
on the layer's actual input (the GPU's own residual after the previous layer, fed to the oracle
layer), and the free-running final residual is compared with the oracle's free run.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import gtmoe  # noqa: E402
import oracle  # noqa: E402

D, E, K = gtmoe.HIDDEN, gtmoe.EXPERTS, gtmoe.TOP_K
TOL = 2e-3


def rel_max(got, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.abs(np.asarray(got, np.float64) - ref).max() / np.sqrt(np.mean(ref ** 2)))


def run(dec, x, nl, **kw):
    o = {"hidden": torch.empty(D, device="cuda"), "idx": torch.empty(nl * K, dtype=torch.int32, device="cuda"),
         "w": torch.empty(nl * K, device="cuda"), "logits": torch.empty(nl * E, device="cuda"),
         "h1": torch.empty(nl * D, device="cuda"), "h2": torch.empty(nl * D, device="cuda"),
         "layers": torch.empty(nl * D, device="cuda")}
    dec(x, o["hidden"], topk_idx=o["idx"], topk_w=o["w"], logits=o["logits"], h1=o["h1"], h2=o["h2"],
        hidden_layers=o["layers"], num_layers=nl, **kw)
    dec.check()
    torch.cuda.synchronize()
    out = {k: v.cpu().numpy() for k, v in o.items()}
    out["idx"] = out["idx"].view(np.uint32).reshape(nl, K)
    out["w"] = out["w"].reshape(nl, K)
    out["logits"] = out["logits"].reshape(nl, E)
    for k in ("h1", "h2", "layers"):
        out[k] = out[k].reshape(nl, D)
    return out


@pytest.fixture(scope="module")
def model1():
    m = gtmoe.SynthModel(1, seed=0)
    torch.cuda.synchronize()
    return m


def test_device_weights_byte_identical_with_oracle(model1):
    ref = oracle.SynthLayer(0, 0)
    roff, rtotal = gtmoe.resident_layout()
    img = np.zeros(rtotal, np.uint8)
    oracle.lib().orc_synth_resident(0, 0, D, gtmoe.FFN, E, img.ctypes.data)
    assert np.array_equal(model1.resident[0].cpu().numpy(), img)
    _, stride = gtmoe.expert_layout()
    for e in (0, 17, 127):
        blk = np.zeros(stride, np.uint8)
        oracle.lib().orc_synth_expert(0, 0, e, D, gtmoe.MOE_INTER, blk.ctypes.data)
        got = model1.experts[0][e * stride:(e + 1) * stride].cpu().numpy()
        assert np.array_equal(got, blk), e
    xs = torch.empty(3 * D, device="cuda")
    gtmoe.synth_x(0, 0, 3, xs)
    xs = xs.cpu().numpy().reshape(3, D)
    for t in range(3):
        assert np.array_equal(xs[t], oracle.synth_x(0, t))
    del ref


@pytest.mark.parametrize("tok", range(6))
def test_config0_single_layer(model1, tok):
    dec = gtmoe.Decoder(model1.layers, 1)
    x = torch.from_numpy(oracle.synth_x(0, tok)).cuda()
    g = run(dec, x, 1, norm_between_layers=False)
    want = oracle.SynthLayer(0, 0).block(oracle.synth_x(0, tok))
    assert np.array_equal(g["logits"][0], want["logits"]), "router logits not bit-identical"
    assert np.array_equal(g["idx"][0], want["idx"])
    np.testing.assert_allclose(g["w"][0], want["w"], rtol=1e-5, atol=0)
    for key, gv in (("h1", g["h1"][0]), ("h2", g["h2"][0]), ("hidden", g["hidden"])):
        assert rel_max(gv, want[key]) <= TOL, (key, rel_max(gv, want[key]))
    assert np.array_equal(g["layers"][0], g["hidden"])


def test_config0_logit_bias_skews_routing(model1):
    """The benchmark's Zipf skew knob: a bias vector added to the logits before selection."""
    dec = gtmoe.Decoder(model1.layers, 1)
    rng = np.random.default_rng(0)
    bias = rng.normal(0, 2.0, size=E).astype(np.float32)
    x = oracle.synth_x(0, 9)
    g = run(dec, torch.from_numpy(x).cuda(), 1, logit_bias=torch.from_numpy(bias).cuda(), norm_between_layers=False)
    want = oracle.SynthLayer(0, 0).block(x, logit_bias=bias)
    assert np.array_equal(g["logits"][0], want["logits"])
    assert np.array_equal(g["idx"][0], want["idx"])
    assert rel_max(g["hidden"], want["hidden"]) <= TOL


def test_config0_repeat_calls_identical(model1):
    dec = gtmoe.Decoder(model1.layers, 1)
    x = torch.from_numpy(oracle.synth_x(0, 3)).cuda()
    a = run(dec, x, 1)
    b = run(dec, x, 1)
    for k in a:
        assert np.array_equal(a[k], b[k]), k


def test_config1_thirty_layer_stack():
    nl = 30
    m = gtmoe.SynthModel(nl, seed=0)
    dec = gtmoe.Decoder(m.layers, nl)
    x0 = oracle.synth_x(0, 0)
    g = run(dec, torch.from_numpy(x0).cuda(), nl)
    layers = [oracle.SynthLayer(0, l) for l in range(nl)]
    # per layer, on the GPU's own layer input: exact routing, outputs within tolerance
    cur = x0
    for l in range(nl):
        o = layers[l].block(cur)
        assert np.array_equal(g["logits"][l], o["logits"]), f"layer {l}: logits"
        assert np.array_equal(g["idx"][l], o["idx"]), f"layer {l}: top-8"
        assert rel_max(g["h2"][l], o["h2"]) <= TOL, l
        assert rel_max(g["h1"][l], o["h1"]) <= TOL, l
        ref_next = oracle.rms_norm(o["hidden"], None) if l < nl - 1 else o["hidden"]
        assert rel_max(g["layers"][l], ref_next) <= TOL, l
        cur = g["layers"][l]
    # free-running end to end
    free = oracle.synth_stack(layers, x0)
    assert rel_max(g["hidden"], free["hidden"]) <= TOL
    assert np.array_equal(g["idx"], free["idx"])


def test_bounded_wait_runs_out_then_workspace_recovers(model1):
    """A grid-barrier wait that can never be satisfied (GTM_DECODE_TEST_WAIT_RUNS_OUT: the first
    wait's epoch is one no CTA arrives with, under a 2 ms limit) ends in GTM_ERR_TIMEOUT read back
    by gtm_moe_decode_check, with the context usable; the next launch on the same workspace is
    exact again."""
    import time
    dec = gtmoe.Decoder(model1.layers, 1)
    x = torch.from_numpy(oracle.synth_x(0, 3)).cuda()
    out = torch.empty(D, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    dec(x, out, num_layers=1, norm_between_layers=False, extra_flags=gtmoe.DECODE_TEST_WAIT_RUNS_OUT)
    with pytest.raises(gtmoe.GtmError) as e:
        dec.check()
    assert e.value.status == gtmoe.ERR_TIMEOUT and "timed out" in str(e.value)
    assert time.perf_counter() - t0 < 1.0
    dec.check()   # the sticky word was cleared by the failing check
    g = run(dec, x, 1, norm_between_layers=False)
    want = oracle.SynthLayer(0, 0).block(oracle.synth_x(0, 3))
    assert np.array_equal(g["idx"][0], want["idx"])
    assert rel_max(g["hidden"], want["hidden"]) <= TOL


@pytest.mark.parametrize("case", ["zero_group", "outlier", "tiny", "mixed_scale"])
def test_config0_activation_ranges(model1, case):
    """The decode carries each 64-element group of an activation as three 7-bit limbs under a
    power-of-two group scale: a group of zeros, one element 1e4 times its neighbours, values near
    the float minimum and groups of very different magnitude keep exact routing and the 2e-3 gate."""
    x = oracle.synth_x(0, 11).copy()
    if case == "zero_group":
        x[64:128] = 0.0
        x[1000:1064] = 0.0
    elif case == "outlier":
        x[70] = 1.0e4
        x[2000] = -3.0e3
    elif case == "tiny":
        x[:704] *= 1.0e-30
    else:
        x *= np.repeat(np.float32(10.0) ** np.arange(-3, 3, 6 / 44, dtype=np.float32)[:44], 64)
    dec = gtmoe.Decoder(model1.layers, 1)
    g = run(dec, torch.from_numpy(x).cuda(), 1, norm_between_layers=False)
    want = oracle.SynthLayer(0, 0).block(x)
    assert np.array_equal(g["logits"][0], want["logits"]), "router logits not bit-identical"
    assert np.array_equal(g["idx"][0], want["idx"])
    for key, gv in (("h1", g["h1"][0]), ("h2", g["h2"][0]), ("hidden", g["hidden"])):
        assert rel_max(gv, want[key]) <= TOL, (key, rel_max(gv, want[key]))

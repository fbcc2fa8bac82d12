"""Pins the CPU oracle (oracle/moe_oracle.c) before anything is checked against it.

* Against the known-answer cases of the reference's tests/test_gpu_kernels.cpp (kat.npz), with
  that test's own tolerance (numpy allclose, ATOL 1e-5, RTOL 1e-4, test_gpu_kernels.cpp:80-81)
  and exact top-8 indices including the forced 11/70 tie (:489-490).
* Bit for bit against the reference's own compiled helpers (ref_block.npz, produced from
  oracle/_ref/libgtref.so): matvec, rms_norm, gelu_tanh and the whole MoE block.
* Live against oracle/_ref when that library is present (this container).
"""
import numpy as np
import pytest

import oracle

ATOL, RTOL = 1e-5, 1e-4


def allclose(got, want):
    got = np.asarray(got, np.float64); want = np.asarray(want, np.float64)
    excess = np.abs(got - want) - (ATOL + RTOL * np.abs(want))
    return float(excess.max()) <= 0.0, float(np.abs(got - want).max())


@pytest.mark.parametrize("name", ["gemv_int4", "gemv_int8"])
def test_matvec_known_answer(golden, name):
    k = golden["kat"]
    rows, in_dim, bits = (int(v) for v in k[name + ".shape"])
    got = oracle.matvec(k[name + ".w"], k[name + ".s"], k[name + ".b"], k[name + ".x"], rows, in_dim, bits)
    ok, err = allclose(got, k[name + ".want"])
    assert ok, f"{name}: max abs err {err}"
    # and bit-identical with the reference's own matvec order
    assert np.array_equal(got, golden["ref"][name + ".ref_out"])


def test_rmsnorm_known_answer(golden):
    k = golden["kat"]
    assert allclose(oracle.rms_norm(k["rmsnorm.x"], None), k["rmsnorm.want_nw"])[0]
    got = oracle.rms_norm(k["rmsnorm.x"], k["rmsnorm.w"])
    assert allclose(got, k["rmsnorm.want_w"])[0]
    assert np.array_equal(got, golden["ref"]["rmsnorm.ref_w"])


def test_geglu_known_answer(golden):
    k = golden["kat"]
    got = oracle.gelu_tanh(k["geglu.g"]) * k["geglu.u"]
    assert allclose(got, k["geglu.want"])[0]
    assert np.array_equal(oracle.gelu_tanh(k["geglu.g"]), golden["ref"]["geglu.ref_gelu"])


def test_topk_known_answer_with_tie(golden):
    k = golden["kat"]
    idx, w = oracle.topk(k["topk.logits"], 8, k["topk.pes"])
    assert np.array_equal(idx, k["topk.want_idx"])
    assert 11 in idx and 70 in idx and list(idx).index(11) < list(idx).index(70)
    assert allclose(w, k["topk.want_w"])[0]


def test_scale_accum_known_answer(golden):
    k = golden["kat"]
    ins = k["scaleaccum.in"].reshape(8, -1)
    acc = np.zeros(ins.shape[1], np.float32)
    for j in range(8):
        acc = (acc + np.float32(k["scaleaccum.weights"][j]) * ins[j]).astype(np.float32)
    assert allclose(acc, k["scaleaccum.want"])[0]


@pytest.mark.parametrize("tok", [0, 1])
def test_block_bit_identical_with_reference(golden, tok):
    r = golden["ref"]
    layer = oracle.SynthLayer(0, 0)
    x = oracle.synth_x(0, tok)
    assert np.array_equal(x, r[f"block{tok}.x"]), "synthetic generator drifted"
    got = layer.block(x)
    for key in ("hidden", "h1", "h2", "logits", "idx", "w"):
        assert np.array_equal(got[key], r[f"block{tok}.{key}"]), key


def test_block_router_tie_goes_to_lower_index(golden):
    r = golden["ref"]
    assert int(r["tie.exact"][0]) == 1
    layer = oracle.SynthLayer(0, 0)
    got = layer.block(r["tie.x"], logit_bias=r["tie.bias"])
    lo, hi = (int(v) for v in r["tie.pair"])
    idx = list(got["idx"])
    assert idx.index(lo) < idx.index(hi)
    for key in ("hidden", "h1", "h2", "idx", "w"):
        assert np.array_equal(got[key], r[f"tie.{key}"]), key


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built here")
def test_block_live_against_reference_more_tokens():
    layer = oracle.SynthLayer(7, 3)
    for tok in range(3):
        x = oracle.synth_x(7, tok)
        a = layer.block(x)
        b = layer.block(x, impl="ref")
        for key in a:
            assert np.array_equal(a[key], b[key]), (tok, key)


def test_stack_matches_blockwise_composition():
    layers = [oracle.SynthLayer(0, l) for l in range(3)]
    x = oracle.synth_x(0, 0)
    s = oracle.synth_stack(layers, x)
    cur = x
    for l, L in enumerate(layers):
        o = L.block(cur)
        assert np.array_equal(o["idx"], s["idx"][l])
        cur = oracle.rms_norm(o["hidden"], None) if l < 2 else o["hidden"]
        assert np.array_equal(cur, s["hidden_per_layer"][l])
    assert np.array_equal(cur, s["hidden"])

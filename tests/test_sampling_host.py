"""Host side of the sampling C ABI (include/gtmoe_sampling.h) against the pinned sampling oracle.

gtm_sampling_validate, gtm_sampling_splitmix64 and gtm_sampling_seed_for run on the host, so
they are checked here without a GPU: the same outcomes as the reference's compiled
sampling.cpp (tests/golden/sampling.npz) and its messages. The device entry points are only
checked for the argument errors they report before touching the GPU.
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "turbo-winfare_b200")]

import gtmoe  # noqa: E402
from gtmoe import sampling  # noqa: E402

GOLDEN = os.path.join(ROOT, "tests", "golden", "sampling.npz")


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN)


def sp(t, tp, tk, pen=1.0, seed=None):
    return sampling.SamplingParams(float(t), float(tp), int(tk), float(pen), seed is not None,
                                   0 if seed is None else int(seed))


def test_splitmix64_matches_reference(g):
    for x, want in zip(g["splitmix.in"], g["splitmix.out"]):
        assert sampling.splitmix64(int(x)) == int(want)
    assert sampling.splitmix64(0) == 0xE220A8397B1DCDAF   # tests/test_sampling.cpp:118


def test_seed_for_matches_reference(g):
    for has, seed, pos, want in zip(g["seed.has"], g["seed.seed"], g["seed.pos"], g["seed.out"]):
        assert sampling.seed_for(sp(0.7, 1.0, 0, seed=int(seed) if has else None), int(pos)) == int(want)


def test_validate_matches_reference(g):
    for (t, tp, tk, pen), rej in zip(g["validate.params"], g["validate.rejects"]):
        p = sp(t, tp, tk, pen)
        if rej:
            with pytest.raises(gtmoe.GtmError) as e:
                sampling.validate_sampling(p)
            assert e.value.status == gtmoe.ERR_INVALID
        else:
            sampling.validate_sampling(p)


def test_validate_messages():
    # sampling.cpp:49-53: the rule that looks like an oversight, with the reference's wording
    with pytest.raises(gtmoe.GtmError, match="requires top_k in 1..256; full-vocabulary nucleus sampling is not"):
        sampling.validate_sampling(sp(0.7, 0.9, 0))
    with pytest.raises(gtmoe.GtmError, match="top_k must be in 0..256"):
        sampling.validate_sampling(sp(0.2, 0.95, 257))
    with pytest.raises(gtmoe.GtmError, match="temperature must be finite and >= 0"):
        sampling.validate_sampling(sp(float("nan"), 1.0, 0))
    assert sp(0.0, 1.0, 0).is_greedy() and not sp(0.0, 1.0, 0, pen=1.1).is_greedy()


def test_workspace_sizes():
    L = gtmoe.lib()
    assert L.gtm_sample_workspace_bytes(0) == 0
    assert L.gtm_sample_workspace_bytes((1 << 22) + 1) == 0
    small, full = L.gtm_sample_workspace_bytes(8), L.gtm_sample_workspace_bytes(262144)
    assert 0 < small < full and full % 256 == 0
    assert L.gtm_sample_workspace_bytes(1 << 22) > full


def test_device_entries_reject_bad_arguments_before_the_gpu():
    L = gtmoe.lib()
    fake = C.c_void_p(256)   # never dereferenced: every case below fails its host-side checks
    ok = sp(1.0, 0.9, 8).c()
    bad = sp(0.7, 0.9, 0).c()
    rc = L.gtm_sample_token(fake, 0, C.byref(ok), 1, fake, fake, fake, 1 << 20, None)
    assert rc == gtmoe.ERR_INVALID and "empty vocabulary" in gtmoe.last_error()
    assert L.gtm_sample_token(fake, 100, C.byref(bad), 1, fake, fake, fake, 1 << 20, None) == gtmoe.ERR_INVALID
    assert L.gtm_sample_token(None, 100, C.byref(ok), 1, fake, fake, fake, 1 << 20, None) == gtmoe.ERR_INVALID
    assert L.gtm_sample_token(fake, (1 << 22) + 1, C.byref(ok), 1, fake, fake, fake, 1 << 30, None) == \
        gtmoe.ERR_UNSUPPORTED
    assert L.gtm_sample_token(fake, 100, C.byref(ok), 1, fake, fake, fake, 16, None) == gtmoe.ERR_WORKSPACE
    assert L.gtm_sample_token(C.c_void_p(258), 100, C.byref(ok), 1, fake, fake, fake, 1 << 20, None) == \
        gtmoe.ERR_MISALIGNED
    assert L.gtm_repetition_penalty(fake, 100, None, 3, 1.3, 30.0, fake, 1 << 20, None) == gtmoe.ERR_INVALID
    assert L.gtm_repetition_penalty(fake, 100, fake, 3, 0.0, 30.0, fake, 1 << 20, None) == gtmoe.ERR_INVALID
    assert L.gtm_repetition_penalty(fake, 100, fake, 3, 1.3, 30.0, fake, 16, None) == gtmoe.ERR_WORKSPACE
    assert L.gtm_softcap(16, fake, 0.0, fake, None) == gtmoe.ERR_INVALID
    assert L.gtm_softcap(16, None, 30.0, fake, None) == gtmoe.ERR_INVALID
    assert L.gtm_softcap(0, None, 30.0, None, None) == gtmoe.OK
    # penalty 1 or an empty history is a no-op (sampling.cpp:77): nothing is launched
    assert L.gtm_repetition_penalty(fake, 100, fake, 3, 1.0, 30.0, None, 0, None) == gtmoe.OK
    assert L.gtm_repetition_penalty(fake, 100, None, 0, 2.0, 30.0, None, 0, None) == gtmoe.OK

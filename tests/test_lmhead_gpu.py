"""Tied LM head with greedy argmax (gtm_lm_head_greedy) against the CPU oracle's matvec
(cpu_reference.cpp:55-83 order): the token and its logit must be bit-identical to the
reference's argmax (ties to the lower row; LMHeadGreedy.hlsl:12, ArgmaxReduce.hlsl:33-34) at the
model's full vocabulary (262,144 x 2816 int4, ~415 MB), including forced exact ties, a near tie
below the approximate pass's resolution, and an all-zero input where every row ties."""
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import gtmoe  # noqa: E402
import oracle  # noqa: E402

D = gtmoe.HIDDEN
G = D // 64


def make_head(rows, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randint(0, 256, (rows, D // 2), dtype=torch.uint8, device="cuda", generator=g)
    sc = (torch.randn(rows, G, device="cuda", generator=g).abs() * 0.02 + 1e-3).to(torch.bfloat16)
    bi = (-8.0 * sc.float() * (1.0 + 0.05 * torch.randn(rows, G, device="cuda", generator=g))).to(torch.bfloat16)
    return w, sc.view(torch.int16), bi.view(torch.int16)


def oracle_logits(w, s, b, x):
    return oracle.matvec(w.cpu().numpy(), s.cpu().numpy().view(np.uint16), b.cpu().numpy().view(np.uint16),
                         x.cpu().numpy(), w.shape[0], D, 4)


def run(head, w, s, b, x):
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    logit = torch.zeros(1, device="cuda")
    head(w, s, b, x, tok, logit)
    torch.cuda.synchronize()
    return int(tok.item()), logit.cpu().numpy()[0], head.candidates()


def expect(ref):
    t = int(np.argmax(ref))   # first occurrence: ties go to the lower row
    return t, ref[t]


@pytest.fixture(scope="module")
def full():
    rows = 262144
    w, s, b = make_head(rows, 1)
    x = torch.randn(D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(2))
    x = x / x.pow(2).mean().sqrt()
    ref = oracle_logits(w, s, b, x)
    return w, s, b, x, ref


def test_full_vocabulary_matches_the_oracle_bit_for_bit(full):
    w, s, b, x, ref = full
    head = gtmoe.LmHead(w.shape[0])
    tok, val, n = run(head, w, s, b, x)
    t, v = expect(ref)
    assert tok == t
    assert np.float32(val).tobytes() == np.float32(v).tobytes()
    assert 1 <= n <= 64, n
    if oracle.ref_available():   # the reference's own compiled CPU code, same answer
        rref = oracle.matvec(w.cpu().numpy(), s.cpu().numpy().view(np.uint16), b.cpu().numpy().view(np.uint16),
                             x.cpu().numpy(), w.shape[0], D, 4, impl="ref")
        assert np.array_equal(rref, ref)
    # timing: weights, scales and biases once per call (cold L2: 415 MB > 126 MB)
    tokt = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(3):
        head(w, s, b, x, tokt)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        head(w, s, b, x, tokt)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 20
    nbytes = w.numel() + 2 * s.numel() * 2
    print(f"\nlm head {w.shape[0]} x {D}: {ms * 1e3:.1f} us per token = {nbytes / ms / 1e6:.0f} GB/s, "
          f"{n} rows recomputed exactly")


def test_exact_ties_go_to_the_lower_row(full):
    w, s, b, x, ref = full
    t, _ = expect(ref)
    lo, hi = t // 2, min(t + 12345, w.shape[0] - 1)
    w2, s2, b2 = w.clone(), s.clone(), b.clone()
    for r in (lo, hi):
        w2[r], s2[r], b2[r] = w[t], s[t], b[t]
    head = gtmoe.LmHead(w.shape[0])
    tok, val, n = run(head, w2, s2, b2, x)
    assert tok == lo and np.float32(val).tobytes() == np.float32(ref[t]).tobytes()
    assert n >= 3


def test_near_tie_below_the_fast_pass_resolution(full):
    w, s, b, x, ref = full
    t, _ = expect(ref)
    xs = x.cpu().numpy()
    # nudge one weight where |x| is small but the change still exceeds the logit's fp32 ulp:
    # the two rows then differ by ~1e-4, far inside the fast pass's error bound
    ax = np.where(np.abs(xs) >= 0.01, np.abs(xs), np.inf)
    k = int(np.argmin(ax))
    byte = w[t, k // 2].item()
    nib = (byte >> 4) if k % 2 else (byte & 15)
    new = nib + 1 if nib < 15 else nib - 1
    nb = ((byte & 15) | (new << 4)) if k % 2 else ((byte & 0xF0) | new)
    lo = t // 3
    w2, s2, b2 = w.clone(), s.clone(), b.clone()
    w2[lo], s2[lo], b2[lo] = w[t], s[t], b[t]
    w2[lo, k // 2] = nb
    ref2 = ref.copy()
    ref2[lo] = oracle_logits(w2[lo:lo + 1], s2[lo:lo + 1], b2[lo:lo + 1], x)[0]
    assert ref2[lo] != ref2[t] and abs(ref2[lo] - ref2[t]) < 1e-3
    head = gtmoe.LmHead(w.shape[0])
    tok, val, _ = run(head, w2, s2, b2, x)
    et, ev = expect(ref2)
    assert tok == et and np.float32(val).tobytes() == np.float32(ev).tobytes()


@pytest.mark.parametrize("rows", [1, 17, 1000, 4099])
def test_ragged_row_counts(rows):
    w, s, b = make_head(rows, 10 + rows)
    x = torch.randn(D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(rows))
    ref = oracle_logits(w, s, b, x)
    tok, val, _ = run(gtmoe.LmHead(rows), w, s, b, x)
    t, v = expect(ref)
    assert tok == t and np.float32(val).tobytes() == np.float32(v).tobytes()


def test_zero_input_every_row_ties():
    rows = 20000
    w, s, b = make_head(rows, 7)
    x = torch.zeros(D, device="cuda")
    tok, val, n = run(gtmoe.LmHead(rows), w, s, b, x)
    assert tok == 0 and val == 0.0 and n == rows


def test_rejects_other_shapes_and_small_workspace():
    L = gtmoe.lib()
    p = torch.zeros(64, device="cuda")
    ptr = gtmoe.ptr(p)
    assert L.gtm_lm_head_greedy(10, 4096, ptr, ptr, ptr, ptr, ptr, None, ptr, 1 << 20, None) == gtmoe.ERR_UNSUPPORTED
    assert L.gtm_lm_head_greedy(10, D, ptr, ptr, ptr, ptr, ptr, None, ptr, 16, None) == gtmoe.ERR_WORKSPACE
    assert L.gtm_lm_head_greedy(0, D, ptr, ptr, ptr, ptr, ptr, None, ptr, 1 << 20, None) == gtmoe.ERR_INVALID

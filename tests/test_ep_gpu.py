"""GPU parity of the expert-parallel MoE layer (gtm_moe_ep_* and gtm_moe_ep_peer_* phases).

P ranks are emulated in one process on one GPU (gtmoe.ep.ep_layer_local: the same phases and
the same split bookkeeping as the NCCL path, the all-to-all replaced by tensor slicing). Each
rank holds only its own experts. Checked against the single-GPU path on the full token set
(expert rows are computed independently of which other rows share a tile, so the results agree
to the last bit) and against the CPU oracle on sampled tokens (top-8 bit-exact, outputs within
2e-3 x RMS). Configurations: BASELINE config 3 shape (bf16 tokens, uniform routing logits) at
P = 2, 4, 8, and config 2 (router GEMV, Zipf logit bias) at P = 2.
"""
import os
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import gtmoe  # noqa: E402
from gtmoe import ep, workloads  # noqa: E402
import oracle  # noqa: E402
from block_f64 import block_f64, rel_err_per_token  # noqa: E402

D, E, K = gtmoe.HIDDEN, gtmoe.EXPERTS, gtmoe.TOP_K
TOL = 2e-3


def rel_max(got, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.abs(np.asarray(got, np.float64) - ref).max() / np.sqrt(np.mean(ref ** 2)))


@pytest.fixture(scope="module")
def full_model():
    m = gtmoe.SynthModel(1, seed=0)
    torch.cuda.synchronize()
    return m


@pytest.fixture(scope="module")
def ref_layer():
    return oracle.SynthLayer(0, 0)


def run_ep(P, x, route_logits=None, logit_bias=None):
    T = x.shape[0]
    Tp = T // P
    shards = [ep.EpShardModel(0, r, P) for r in range(P)]
    ops = [ep.CudaEpOps(shards[r].layer, r, P, max_tokens=Tp, max_recv_rows=T * K) for r in range(P)]
    xs = [x[r * Tp:(r + 1) * Tp] for r in range(P)]
    outs = [torch.empty(Tp, D, device="cuda") for _ in range(P)]
    idx = [torch.empty(Tp, K, dtype=torch.int32, device="cuda") for _ in range(P)]
    kw = []
    for r in range(P):
        d = {"topk_idx": idx[r]}
        if route_logits is not None:
            d["route_logits"] = route_logits[r * Tp:(r + 1) * Tp]
        if logit_bias is not None:
            d["logit_bias"] = logit_bias
        kw.append(d)
    recv = ep.ep_layer_local(ops, ep.LocalExchange(P), xs, outs, kw)
    for o in ops:
        o.check()
    torch.cuda.synchronize()
    return torch.cat(outs).cpu().numpy(), torch.cat(idx).cpu().numpy().view(np.uint32), recv


def run_single(model, x, **kw):
    T = x.shape[0]
    blk = gtmoe.TokenBlock(T)
    out = torch.empty(T, D, device="cuda")
    idx = torch.empty(T, K, dtype=torch.int32, device="cuda")
    blk(model.layers[0], x, out, topk_idx=idx, **kw)
    blk.check()
    torch.cuda.synchronize()
    return out.cpu().numpy(), idx.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("P", [2, 4, 8])
def test_ep_prefill_matches_single_gpu_and_oracle(full_model, ref_layer, P):
    T = 1024
    x32 = torch.empty(T * D, device="cuda")
    gtmoe.synth_x(0, 0, T, x32)
    x = x32.view(T, D).to(torch.bfloat16)
    rl = torch.from_numpy(workloads.uniform_route_logits(T)).cuda()
    got, gidx, recv = run_ep(P, x, route_logits=rl)
    assert sum(recv) == T * K
    single, sidx = run_single(full_model, x, route_logits=rl)
    assert np.array_equal(gidx, sidx)
    assert np.array_equal(got, single), f"max diff {np.abs(got - single).max()}"
    xs = x.float().cpu().numpy()
    rls = rl.cpu().numpy()
    for t in (0, T // P, T - 1):
        ref = ref_layer.block(xs[t], route_logits=rls[t])
        assert np.array_equal(gidx[t], ref["idx"])
        assert rel_max(got[t], ref["hidden"]) <= TOL


def test_ep_router_zipf_two_ranks(full_model, ref_layer):
    T = 64
    x32 = torch.empty(T * D, device="cuda")
    gtmoe.synth_x(0, 0, T, x32)
    x = x32.view(T, D)
    bias = workloads.zipf_logit_bias()
    lb = torch.from_numpy(bias).cuda()
    got, gidx, _ = run_ep(2, x, logit_bias=lb)
    single, sidx = run_single(full_model, x, logit_bias=lb)
    assert np.array_equal(gidx, sidx)
    assert np.array_equal(got, single)
    xs = x.cpu().numpy()
    for t in (0, 31, 63):
        ref = ref_layer.block(xs[t], logit_bias=bias)
        assert np.array_equal(gidx[t], ref["idx"])
        assert rel_max(got[t], ref["hidden"]) <= TOL


# ---- expert parallelism over peer memory (gtm_moe_ep_peer_*) ---------------------------------------
# The ranks are emulated in one process: every rank's workspace is device memory of this process,
# so the kernels' "peer" loads and stores are local ones, but they follow the same pointers,
# entry order and barriers (stream order here) as the multi-GPU run.

def make_peer_ops(P, max_tokens):
    shards = [ep.EpShardModel(0, r, P) for r in range(P)]
    ops = [ep.PeerEpOps(shards[r].layer, r, P, max_tokens=max_tokens) for r in range(P)]
    for o in ops:
        o.connect_local(ops)
    return shards, ops


def run_peer(ops, xs, route_logits=None, logit_bias=None, h2=None, extra=None):
    """h2: list that receives the routed sums (combine input) of all ranks' tokens; extra: dict
    that receives h1, h2 and the routing weights of all ranks' tokens."""
    P = len(ops)
    outs = [torch.empty(x.shape[0], D, device="cuda") for x in xs]
    idx = [torch.empty(x.shape[0], K, dtype=torch.int32, device="cuda") for x in xs]
    h2s = [torch.empty(x.shape[0], D, device="cuda") for x in xs]
    h1s = [torch.empty(x.shape[0], D, device="cuda") for x in xs]
    ws = [torch.empty(x.shape[0], K, device="cuda") for x in xs]
    kw, off = [], 0
    for r in range(P):
        n = xs[r].shape[0]
        d = {"topk_idx": idx[r], "h2": h2s[r] if (h2 is not None or extra is not None) else None}
        if extra is not None:
            d["h1"], d["topk_w"] = h1s[r], ws[r]
        if route_logits is not None:
            d["route_logits"] = route_logits[off:off + n]
        if logit_bias is not None:
            d["logit_bias"] = logit_bias
        kw.append(d)
        off += n
    ep.ep_layer_peer_local(ops, xs, outs, kw)
    for o in ops:
        o.check()
    torch.cuda.synchronize()
    if h2 is not None:
        h2.append(torch.cat(h2s).cpu().numpy())
    if extra is not None:
        extra.update(h1=torch.cat(h1s), h2=torch.cat(h2s), w=torch.cat(ws))
    return torch.cat(outs).cpu().numpy(), torch.cat(idx).cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("P", [1, 2, 4, 8])
def test_ep_peer_matches_single_gpu_and_oracle(full_model, ref_layer, P):
    T = 1024
    x32 = torch.empty(T * D, device="cuda")
    gtmoe.synth_x(0, 0, T, x32)
    x = x32.view(T, D).to(torch.bfloat16)
    rl = torch.from_numpy(workloads.uniform_route_logits(T)).cuda()
    _, ops = make_peer_ops(P, T // P)
    try:
        got, gidx = run_peer(ops, list(x.split(T // P)), route_logits=rl)
    finally:
        for o in ops:
            o.close()
    single, sidx = run_single(full_model, x, route_logits=rl)
    assert np.array_equal(gidx, sidx)
    assert np.array_equal(got, single), f"max diff {np.abs(got - single).max()}"
    xs = x.float().cpu().numpy()
    rls = rl.cpu().numpy()
    for t in (0, (T // P) % T, T - 1):
        ref = ref_layer.block(xs[t], route_logits=rls[t])
        assert np.array_equal(gidx[t], ref["idx"])
        assert rel_max(got[t], ref["hidden"]) <= TOL


def test_ep_peer_ragged_ranks_and_stale_entries(full_model, ref_layer):
    """Ranks with different token counts (one with none) after a call with full ranks: entries
    past a rank's current count are stale and must be ignored. Each expert sees the same rows in
    the same order as on one GPU, so the routed sum h2 is bit-identical; the shared expert runs
    per rank, and a rank's token tiles of <= 64 rows take the stacked high/low operand (the
    high and low products summed after the MMAs, not in one accumulator), so the layer output
    agrees to rounding there."""
    P, MT = 4, 128
    counts = [100, 1, 37, 0]
    n_all = P * MT
    x32 = torch.empty(n_all * D, device="cuda")
    gtmoe.synth_x(0, 0, n_all, x32)
    x = x32.view(n_all, D)
    bias = torch.from_numpy(workloads.zipf_logit_bias()).cuda()
    _, ops = make_peer_ops(P, MT)
    try:
        full_got, _ = run_peer(ops, list(x.split(MT)), logit_bias=bias)
        xr = x[:sum(counts)]
        h2 = []
        got, gidx = run_peer(ops, list(xr.split(counts)), logit_bias=bias, h2=h2)
    finally:
        for o in ops:
            o.close()
    single_full, _ = run_single(full_model, x, logit_bias=bias)
    assert np.array_equal(full_got, single_full)
    sh2 = torch.empty(sum(counts), D, device="cuda")
    single, sidx = run_single(full_model, xr, logit_bias=bias, h2=sh2)
    assert np.array_equal(gidx, sidx)
    assert np.array_equal(h2[0], sh2.cpu().numpy())
    assert np.array_equal(got[:counts[0]], single[:counts[0]])   # rank 0: > 64 rows in both
    assert rel_max(got, single) <= 1e-5
    xs = xr.cpu().numpy()
    b = bias.cpu().numpy()
    for t in (0, counts[0], counts[0] + counts[1] + counts[2] - 1):
        ref = ref_layer.block(xs[t], logit_bias=b)
        assert np.array_equal(gidx[t], ref["idx"])
        assert rel_max(got[t], ref["hidden"]) <= TOL


def test_ep_peer_eight_ranks_every_token_config3(full_model):
    """BASELINE config 3 at emulated P = 8 (4096 bf16 tokens, 512 per rank, 16 experts per rank):
    every token's top-8 against the oracle's selection, and h1, h2 and the new residual of every
    token against the float64 whole-batch restatement (tests/block_f64.py) fed the device's
    routing."""
    P, T = 8, 4096
    x32 = torch.empty(T * D, device="cuda")
    gtmoe.synth_x(0, 0, T, x32)
    x = x32.view(T, D).to(torch.bfloat16)
    rl_np = workloads.uniform_route_logits(T)
    rl = torch.from_numpy(rl_np).cuda()
    _, ops = make_peer_ops(P, T // P)
    ex = {}
    try:
        got, gidx = run_peer(ops, list(x.split(T // P)), route_logits=rl, extra=ex)
    finally:
        for o in ops:
            o.close()
    res = full_model.resident[0].cpu().numpy()
    o = full_model.layers[0].per_expert_scale
    pes = res[o:o + 2 * E].view(np.uint16)
    for t in range(T):
        idx, _ = oracle.topk(rl_np[t], K, pes)
        assert np.array_equal(gidx[t], idx), f"token {t}"
    ref = block_f64(full_model.layers[0], full_model.resident[0], full_model.experts[0], x.float(),
                    torch.from_numpy(gidx.astype(np.int64)), ex["w"])
    for k, v in (("h1", ex["h1"]), ("h2", ex["h2"]), ("hidden", torch.from_numpy(got))):
        e = rel_err_per_token(v, ref[k])
        assert float(e.max()) <= TOL, f"{k}: token {int(e.argmax())} at {float(e.max()):.3e}"

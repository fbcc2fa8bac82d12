"""Expert-parallel exchange protocol on CPU: two gloo ranks run gtmoe.ep.ep_layer (the function
the product runs over NCCL) with stand-in phase ops whose result is known in closed form.

The stand-in ops follow the CUDA dispatch contract: one row per (token, slot), grouped by
destination rank in (token, slot) order, metadata (expert, weight), counts per destination;
experts return rows in received order; combine sums the returned rows per token in router
order. Checked: rows reach the rank that owns their expert, uneven and empty splits, and every
token's combined output equals the single-process value.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
dist = pytest.importorskip("torch.distributed")

from gtmoe import ep  # noqa: E402

D, E, K = 16, 8, 2


def expert_fn(e, w, row):
    return row * np.float32(e + 1) * np.float32(w)


def route(x, skew):
    """Deterministic stand-in router: top-K of a fixed projection, ties to the lower index."""
    rng = np.random.default_rng(5)
    P = rng.standard_normal((D, E)).astype(np.float32)
    logits = x @ P + skew
    idx = np.argsort(-logits, axis=1, kind="stable")[:, :K]
    w = np.exp(np.take_along_axis(logits, idx, 1) - logits[np.arange(len(x)), idx[:, 0]][:, None])
    w = (w / w.sum(1, keepdims=True)).astype(np.float32)
    return idx.astype(np.int64), w


class StandInOps:
    def __init__(self, rank, world, skew):
        self.rank, self.world, self.skew = rank, world, skew
        self.e0, self.e1 = ep.experts_of(rank, world, E)
        self.seen_experts = set()

    def dispatch(self, x):
        xs = x.numpy()
        idx, w = route(xs, self.skew)
        epr = E // self.world
        order = sorted(range(len(xs) * K), key=lambda i: (idx.flat[i] // epr, i))
        self.send_pos = np.empty(len(order), np.int64)
        rows = np.zeros((len(order), D), np.float32)
        meta = np.zeros((len(order), 2), np.int32)
        for r, i in enumerate(order):
            self.send_pos[i] = r
            rows[r] = xs[i // K]
            meta[r, 0] = idx.flat[i]
            meta[r, 1] = np.float32(w.flat[i]).view(np.int32)
        counts = np.bincount(idx.reshape(-1) // epr, minlength=self.world).astype(np.int32)
        return torch.from_numpy(rows), torch.from_numpy(meta), torch.from_numpy(counts)

    def shared(self, x):
        self.shared_out = 2.0 * x.numpy()

    def experts(self, rows, meta, n):
        rows, meta = rows.numpy(), meta.numpy()
        out = np.zeros_like(rows)
        for j in range(n):
            e, wgt = int(meta[j, 0]), meta[j, 1:2].view(np.float32)[0]
            assert self.e0 <= e < self.e1, "row sent to a rank that does not own its expert"
            self.seen_experts.add(e)
            out[j] = expert_fn(e, wgt, rows[j])
        return torch.from_numpy(out)

    def combine(self, x, hidden_out, back):
        b = back.numpy()
        T = x.shape[0]
        res = self.shared_out.copy()
        for t in range(T):
            for k in range(K):
                res[t] += b[self.send_pos[t * K + k]]
        hidden_out.copy_(torch.from_numpy(res))


def expected(x, skew):
    idx, w = route(x, skew)
    out = 2.0 * x
    for t in range(len(x)):
        for k in range(K):
            out[t] += expert_fn(idx[t, k], w[t, k], x[t])
    return out


def worker(rank, world, port, tokens_per_rank, skews, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        xch = ep.NcclExchange()
        results = []
        for skew in skews:
            rng = np.random.default_rng(100 + rank)
            x = rng.standard_normal((tokens_per_rank, D)).astype(np.float32)
            ops = StandInOps(rank, world, np.asarray(skew, np.float32))
            out = torch.zeros(tokens_per_rank, D)
            n_send, n_recv = ep.ep_layer(ops, xch, torch.from_numpy(x), out)
            err = float(np.abs(out.numpy() - expected(x, np.asarray(skew, np.float32))).max())
            results.append((n_send, n_recv, err))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, results, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_ep_protocol_two_gloo_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, T = 2, 6
    skews = [
        [0.0] * E,                                    # mixed routing
        [60.0, 60.0, 60.0, 60.0, 0.0, 0.0, 0.0, 0.0],  # everything to rank 0's experts: empty splits
        [0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 60.0, 60.0],  # everything to rank 1
    ]
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, T, skews, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, res, err = q.get(timeout=120)
        assert err is None, f"rank {rank}: {err}"
        out[rank] = res
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for case in range(len(skews)):
        sent = sum(out[r][case][0] for r in range(world))
        recv = sum(out[r][case][1] for r in range(world))
        assert sent == recv == world * T * K
        for r in range(world):
            assert out[r][case][2] < 1e-5, (case, r, out[r][case])
    # the skewed cases really produced empty splits
    assert out[1][1][1] == 0 and out[0][2][1] == 0


def test_local_exchange_matches_protocol():
    """LocalExchange (one-process emulation used by the GPU tests) routes like all_to_all."""
    xch = ep.LocalExchange(3)
    sends = [torch.arange(6).view(6, 1) + 10 * s for s in range(3)]
    splits = [[1, 2, 3], [0, 6, 0], [2, 2, 2]]
    recv_splits = [[splits[s][d] for s in range(3)] for d in range(3)]
    got = xch.rows(sends, splits, recv_splits)
    assert got[0].view(-1).tolist() == [0, 20, 21]
    assert got[1].view(-1).tolist() == [1, 2, 10, 11, 12, 13, 14, 15, 22, 23]
    assert got[2].view(-1).tolist() == [3, 4, 5, 24, 25]
    counts = xch.counts([torch.tensor(s, dtype=torch.int32) for s in splits])
    assert [c.tolist() for c in counts] == recv_splits


# ---- the peer-memory protocol (ep_layer_peer) ------------------------------------------------------
# Stand-in ops keep each rank's "workspace" as files in a directory shared by the processes: the
# dispatch stores every token's top-K into each rank's directory and its row into the directories
# of the ranks that own one of its experts; the experts phase reads only its own directory and
# stores each unweighted result into the token's rank; the combine reads its own results. Without
# the two barriers a rank would read files a peer has not written yet.

class StandInPeerOps:
    def __init__(self, rank, world, root, skew):
        self.rank, self.world, self.root, self.skew = rank, world, root, skew
        self.e0, self.e1 = ep.experts_of(rank, world, E)
        self.layer = 0

    def _ws(self, r):
        return os.path.join(self.root, f"ws{r}")

    def dispatch(self, x):
        xs = x.numpy()
        idx, w = route(xs, self.skew) if len(xs) else (np.zeros((0, K), np.int64), np.zeros((0, K), np.float32))
        self.w = w
        epr = E // self.world
        for r in range(self.world):
            owns = [t for t in range(len(xs)) if any(idx[t, k] // epr == r for k in range(K))]
            np.savez(os.path.join(self._ws(r), f"L{self.layer}_from{self.rank}.npz"), idx=idx,
                     rows=xs[owns] if owns else np.zeros((0, D), np.float32), owns=np.asarray(owns, np.int64))

    def shared(self, x):
        self.shared_out = 2.0 * x.numpy()

    def experts(self):
        for s in range(self.world):
            z = np.load(os.path.join(self._ws(self.rank), f"L{self.layer}_from{s}.npz"))
            idx, rows, owns = z["idx"], z["rows"], list(z["owns"])
            ret = {}
            for t in range(len(idx)):
                for k in range(K):
                    e = int(idx[t, k])
                    if self.e0 <= e < self.e1:
                        ret[t * K + k] = expert_fn(e, np.float32(1.0), rows[owns.index(t)])
            np.savez(os.path.join(self._ws(s), f"L{self.layer}_ret{self.rank}.npz"),
                     pos=np.asarray(list(ret.keys()), np.int64),
                     val=np.asarray(list(ret.values()), np.float32).reshape(-1, D))

    def combine(self, x, hidden_out):
        T = x.shape[0]
        got = np.full((T * K, D), np.nan, np.float32)
        for r in range(self.world):
            z = np.load(os.path.join(self._ws(self.rank), f"L{self.layer}_ret{r}.npz"))
            for p, v in zip(z["pos"], z["val"]):
                got[p] = v
        res = self.shared_out.copy()
        for t in range(T):
            for k in range(K):
                res[t] += self.w[t, k] * got[t * K + k]
        hidden_out.copy_(torch.from_numpy(res))
        self.layer += 1


def peer_worker(rank, world, port, root, counts, skews, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        bar = ep.NcclBarrier(device="cpu")
        errs = []
        ops = StandInPeerOps(rank, world, root, None)
        for case, (n, skew) in enumerate(zip(counts, skews)):
            ops.skew = np.asarray(skew, np.float32)
            rng = np.random.default_rng(200 + 10 * case + rank)
            x = rng.standard_normal((n[rank], D)).astype(np.float32)
            out = torch.zeros(n[rank], D)
            ep.ep_layer_peer(ops, bar, torch.from_numpy(x), out)
            exp = expected(x, ops.skew) if len(x) else np.zeros((0, D), np.float32)
            errs.append(float(np.abs(out.numpy() - exp).max()) if len(x) else 0.0)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, errs, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))


def test_ep_peer_protocol_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 2
    for r in range(world):
        os.makedirs(tmp_path / f"ws{r}")
    counts = [(6, 6), (5, 0), (0, 3), (7, 2)]   # ragged ranks, empty ranks
    skews = [[0.0] * E, [0.0] * E, [60.0] * 4 + [0.0] * 4, [0.0] * 6 + [60.0] * 2]
    port = free_port()
    procs = [ctx.Process(target=peer_worker, args=(r, world, port, str(tmp_path), counts, skews, q))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, errs, err = q.get(timeout=120)
        assert err is None, f"rank {rank}: {err}"
        out[rank] = errs
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert max(out[r]) < 1e-5, out[r]


def leave_worker(rank, world, port, q):
    """Both ranks run one layer; then rank 1 leaves (the process ends without a word to the group)
    and rank 0 starts the next layer, whose first exchange must fail within the group's timeout."""
    import time
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        xch = ep.NcclExchange()
        x = np.random.default_rng(300 + rank).standard_normal((4, D)).astype(np.float32)
        ops = StandInOps(rank, world, np.zeros(E, np.float32))
        out = torch.zeros(4, D)
        ep.ep_layer(ops, xch, torch.from_numpy(x), out)
        err = float(np.abs(out.numpy() - expected(x, np.zeros(E, np.float32))).max())
        if rank == 1:
            q.put((rank, err, None, 0.0))
            q.close()
            q.join_thread()   # the message is sent before the process ends abruptly
            os._exit(0)
        time.sleep(0.5)   # the peer is gone before the next step starts
        t0 = time.perf_counter()
        try:
            ep.ep_layer(ops, xch, torch.from_numpy(x), out)
            q.put((rank, err, "second layer completed without its peer", time.perf_counter() - t0))
        except Exception as e:   # the expected outcome
            q.put((rank, err, "raised: " + type(e).__name__, time.perf_counter() - t0))
    except Exception as e:
        q.put((rank, None, "setup: " + repr(e), 0.0))


def test_ep_rank_leaving_between_steps_is_reported():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=leave_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        rank, err, msg, dt = q.get(timeout=120)
        got[rank] = (err, msg, dt)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[1][0] is not None and got[1][0] < 1e-5          # the first layer was right on both
    assert got[0][0] is not None and got[0][0] < 1e-5
    assert got[0][1].startswith("raised"), got[0]              # the survivor learned of it ...
    assert got[0][2] < 30.0, got[0]                            # ... within a bounded time

"""Expert-parallel MoE layer: one process per GPU, experts sharded across ranks, tokens
data-parallel, NCCL all-to-all over NVLink for the dispatch and the combine.

Rank r of P owns experts [r*E/P, (r+1)*E/P) and its own tokens. One layer:

  1. dispatch   own tokens: views, router, top-k; one routed_x row per (token, slot), grouped
                by destination rank in (token, slot) order (gtm_moe_ep_dispatch)
  2. counts     all-to-all of the per-destination row counts
  3. rows       all-to-all of the rows and their (expert, weight) metadata
  4. shared     shared expert of the own tokens, issued while the exchange runs (gtm_moe_ep_shared)
  5. experts    received rows through the local experts, results in received order
                (gtm_moe_ep_experts)
  6. return     all-to-all back with the split sizes reversed
  7. combine    sum over the slots in router order, layer tail (gtm_moe_ep_combine)

`ep_layer` runs that protocol over an `exchange` and an `ops` object. The product uses
`NcclExchange` (torch.distributed) and `CudaEpOps` (the C ABI); the CPU tests drive the same
function with gloo and stand-in ops. The reference has no multi-GPU path; this replaces its
token-at-a-time prefill (src/runner.cpp:845-854) for a layer sharded over GPUs.

Over peer memory (`PeerEpOps`, `ep_layer_peer`) the ranks map each other's workspaces (CUDA
IPC) and the kernels move the rows themselves with plain NVLink stores: the dispatch stores each
token's top-8 ids into every rank and its routed view into the ranks that own one of its
experts, the experts phase reads only its own workspace and stores each expert output row into
its token's rank. The only collectives are two one-element all-reduces used as stream-ordered
barriers:

  1. dispatch   own tokens: views, router, top-k, pushes to the peers (gtm_moe_ep_peer_dispatch)
  2. shared     on a second stream (gtm_moe_ep_peer_shared)
     -- barrier --
  3. experts    this rank's experts over all ranks' entries (gtm_moe_ep_peer_experts)
     -- barrier --
  4. combine    after the shared expert (gtm_moe_ep_peer_combine)
"""
from __future__ import annotations

import ctypes as C

from . import (ERR_UNSUPPORTED, EXPERTS, HIDDEN, IPC_HANDLE_BYTES, MOE_INTER, TOP_K, EpConfig, EpPeers, GtmError,
               Layer, TokensIO, _stream, check, default_dims, expert_layout, lib, ptr, resident_layout)


META_WORDS = 2   # GtmEpMeta = (uint32 expert, float weight)


def experts_of(rank: int, world: int, experts: int = EXPERTS) -> tuple[int, int]:
    per = experts // world
    return rank * per, (rank + 1) * per


# ---- exchange ----------------------------------------------------------------------------------

class NcclExchange:
    """all-to-all over a torch.distributed process group (NCCL on GPUs, gloo on CPU)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def counts(self, send_counts):
        """send_counts: int32 tensor [world] -> recv_counts (same device)."""
        import torch
        recv = torch.empty_like(send_counts)
        self.dist.all_to_all_single(recv, send_counts, group=self.group)
        return recv

    def rows(self, send, send_splits: list[int], recv_splits: list[int]):
        """send: [sum(send_splits), ...] -> [sum(recv_splits), ...]."""
        import torch
        recv = torch.empty((sum(recv_splits),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        self.dist.all_to_all_single(recv, send[:sum(send_splits)].contiguous(), recv_splits, send_splits,
                                    group=self.group)
        return recv


class LocalExchange:
    """P ranks emulated in one process: each call gets a list of per-rank tensors."""

    def __init__(self, world: int):
        self.world = world

    def counts(self, send_counts_per_rank):
        import torch
        m = torch.stack([c.to("cpu", torch.int64) for c in send_counts_per_rank])   # [src][dst]
        return [m[:, r].to(send_counts_per_rank[r].device, send_counts_per_rank[r].dtype)
                for r in range(self.world)]

    def rows(self, sends, send_splits, recv_splits):
        import torch
        P = self.world
        offs = [[sum(send_splits[s][:d]) for d in range(P)] for s in range(P)]
        out = []
        for d in range(P):
            parts = [sends[s][offs[s][d]:offs[s][d] + send_splits[s][d]] for s in range(P)]
            out.append(torch.cat(parts, 0) if parts else sends[d][:0])
        return out


# ---- the protocol --------------------------------------------------------------------------------

def ep_layer(ops, exchange, x, hidden_out, **io_kw):
    """One expert-parallel layer for this rank's tokens x -> hidden_out (see module docstring).
    The shared expert is issued right after the dispatch: ops that own a second stream run it
    there, overlapping the exchanges; the combine waits for it."""
    import torch
    send_rows, send_meta, send_counts = ops.dispatch(x, **io_kw)
    ops.shared(x, **io_kw)
    recv_counts = exchange.counts(send_counts)
    P = send_counts.numel()
    both = [int(v) for v in torch.cat([send_counts.reshape(-1), recv_counts.reshape(-1)]).cpu().tolist()]  # one host trip
    s_split, r_split = both[:P], both[P:]
    recv_rows = exchange.rows(send_rows, s_split, r_split)
    recv_meta = exchange.rows(send_meta, s_split, r_split)
    ret_rows = ops.experts(recv_rows, recv_meta, sum(r_split))
    back = exchange.rows(ret_rows, r_split, s_split)
    ops.combine(x, hidden_out, back, **io_kw)
    return sum(s_split), sum(r_split)


def ep_layer_local(ops_per_rank, exchange: LocalExchange, xs, outs, io_kw_per_rank=None):
    """The same protocol with P ranks emulated in one process (sequential phases, one GPU)."""
    P = exchange.world
    kw = io_kw_per_rank or [{} for _ in range(P)]
    disp = [ops_per_rank[r].dispatch(xs[r], **kw[r]) for r in range(P)]
    recv_counts = exchange.counts([d[2] for d in disp])
    s_split = [[int(v) for v in d[2].cpu().tolist()] for d in disp]
    r_split = [[int(v) for v in c.cpu().tolist()] for c in recv_counts]
    recv_rows = exchange.rows([d[0] for d in disp], s_split, r_split)
    recv_meta = exchange.rows([d[1] for d in disp], s_split, r_split)
    for r in range(P):
        ops_per_rank[r].shared(xs[r], **kw[r])
    rets = [ops_per_rank[r].experts(recv_rows[r], recv_meta[r], sum(r_split[r])) for r in range(P)]
    back = exchange.rows(rets, r_split, s_split)
    for r in range(P):
        ops_per_rank[r].combine(xs[r], outs[r], back[r], **kw[r])
    return [sum(v) for v in r_split]


# ---- CUDA phases (C ABI) ---------------------------------------------------------------------------

class CudaEpOps:
    """This rank's four EP phases on its GPU through libgtmoe's C ABI."""

    def __init__(self, layer: Layer, rank: int, world: int, max_tokens: int, max_recv_rows: int,
                 device: str = "cuda"):
        import torch
        self.torch = torch
        self.layer = layer
        self.dims = default_dims()
        self.cfg = EpConfig(world, rank, max_tokens, max_recv_rows)
        n = lib().gtm_moe_ep_workspace_bytes(C.byref(self.dims), C.byref(self.cfg))
        if n == 0:
            raise GtmError(ERR_UNSUPPORTED, f"EP workspace size query failed ({world=}, {max_tokens=}, {max_recv_rows=})")
        self.workspace = torch.zeros(n + 256, dtype=torch.uint8, device=device)   # zeroed once, as required
        self.ws_ptr = C.c_void_p((self.workspace.data_ptr() + 255) // 256 * 256)
        self.ws_bytes = n
        self.device = device
        self.send_rows = torch.empty(max_tokens * TOP_K, HIDDEN, device=device)
        self.send_meta = torch.empty(max_tokens * TOP_K, META_WORDS, dtype=torch.int32, device=device)
        self.send_counts = torch.empty(world, dtype=torch.int32, device=device)
        self.ret_rows = torch.empty(max_recv_rows, HIDDEN, device=device)
        # the shared-expert phase runs on its own stream (it has its own workspace tiles)
        self.side = torch.cuda.Stream(device=device)
        self.ev_dispatch = torch.cuda.Event()
        self.ev_shared = torch.cuda.Event()

    def _io(self, x, hidden_out=None, topk_idx=None, topk_w=None, logits=None, h1=None, h2=None, logit_bias=None,
            route_logits=None):
        torch = self.torch
        xf = x if x.dtype == torch.float32 else None
        xb = x if x.dtype == torch.bfloat16 else None
        return TokensIO(x.shape[0], ptr(xf), ptr(xb), ptr(hidden_out), ptr(topk_idx), ptr(topk_w), ptr(logits),
                        ptr(h1), ptr(h2), ptr(logit_bias), ptr(route_logits))

    def dispatch(self, x, **kw):
        io = self._io(x, **kw)
        n = x.shape[0] * TOP_K
        check(lib().gtm_moe_ep_dispatch(C.byref(self.dims), C.byref(self.layer), C.byref(io), C.byref(self.cfg),
                                        ptr(self.send_rows), ptr(self.send_meta), ptr(self.send_counts),
                                        self.ws_ptr, self.ws_bytes, _stream()))
        self.ev_dispatch.record()
        return self.send_rows[:n], self.send_meta[:n], self.send_counts

    def shared(self, x, **kw):
        """On the side stream, after the dispatch (which wrote the dense views it reads)."""
        io = self._io(x, **kw)
        self.side.wait_event(self.ev_dispatch)
        check(lib().gtm_moe_ep_shared(C.byref(self.dims), C.byref(self.layer), C.byref(io), C.byref(self.cfg),
                                      self.ws_ptr, self.ws_bytes, _stream(self.side)))
        self.ev_shared.record(self.side)

    def experts(self, recv_rows, recv_meta, n_recv: int):
        if n_recv > self.cfg.max_recv_rows:
            raise GtmError(-5, f"received {n_recv} rows > max_recv_rows {self.cfg.max_recv_rows}")
        recv_rows = recv_rows.contiguous()
        recv_meta = recv_meta.contiguous()
        check(lib().gtm_moe_ep_experts(C.byref(self.dims), C.byref(self.layer), C.byref(self.cfg),
                                       ptr(recv_rows), ptr(recv_meta), n_recv, ptr(self.ret_rows),
                                       self.ws_ptr, self.ws_bytes, _stream()))
        return self.ret_rows[:n_recv]

    def combine(self, x, hidden_out, back_rows, **kw):
        io = self._io(x, hidden_out=hidden_out, **kw)
        back_rows = back_rows.contiguous()
        self.torch.cuda.current_stream().wait_event(self.ev_shared)
        check(lib().gtm_moe_ep_combine(C.byref(self.dims), C.byref(self.layer), C.byref(io), C.byref(self.cfg),
                                       ptr(back_rows), self.ws_ptr, self.ws_bytes, _stream()))

    def check(self):
        check(lib().gtm_moe_ep_check(self.ws_ptr, _stream()))


# ---- peer memory --------------------------------------------------------------------------------

class NcclBarrier:
    """Stream-ordered barrier of the peer protocol: a one-element all-reduce on the current
    stream (NCCL; gloo on CPU). Work queued after it on this stream runs once every rank has
    queued and finished the work before its own call."""

    def __init__(self, group=None, device="cuda"):
        import torch
        import torch.distributed as dist
        self.dist, self.group = dist, group
        self.flag = torch.zeros(1, dtype=torch.int32, device=device)

    def __call__(self):
        self.dist.all_reduce(self.flag, group=self.group)


def ep_layer_peer(ops, barrier, x, hidden_out, **io_kw):
    """One expert-parallel layer over peer memory (module docstring, second protocol)."""
    ops.dispatch(x, **io_kw)
    ops.shared(x, **io_kw)
    barrier()
    ops.experts()
    barrier()
    ops.combine(x, hidden_out, **io_kw)


def ep_layer_peer_local(ops_per_rank, xs, outs, io_kw_per_rank=None):
    """The peer protocol with P ranks emulated in one process on one GPU: the workspaces are
    plain device memory of this process and the phases run rank after rank on one stream, so
    stream order stands in for the barriers."""
    P = len(ops_per_rank)
    kw = io_kw_per_rank or [{} for _ in range(P)]
    for r in range(P):
        ops_per_rank[r].dispatch(xs[r], **kw[r])
        ops_per_rank[r].shared(xs[r], **kw[r])
    for r in range(P):
        ops_per_rank[r].experts()
    for r in range(P):
        ops_per_rank[r].combine(xs[r], outs[r], **kw[r])


class PeerEpOps:
    """This rank's peer-memory EP phases through libgtmoe's C ABI. The workspace is allocated
    for CUDA IPC (zeroed); `connect` exchanges the handles over a process group and maps the
    peers' workspaces, `connect_local` takes the workspaces of ranks emulated in this process."""

    def __init__(self, layer: Layer, rank: int, world: int, max_tokens: int, device: str = "cuda"):
        import torch
        self.torch = torch
        self.layer = layer
        self.rank, self.world = rank, world
        self.dims = default_dims()
        self.cfg = EpConfig(world, rank, max_tokens, 0)
        n = lib().gtm_moe_ep_peer_workspace_bytes(C.byref(self.dims), C.byref(self.cfg))
        if n == 0:
            raise GtmError(ERR_UNSUPPORTED, f"peer EP workspace size query failed ({world=}, {max_tokens=})")
        self.ws_bytes = n
        self.ws_ptr = C.c_void_p()
        self.handle = (C.c_uint8 * IPC_HANDLE_BYTES)()
        check(lib().gtm_ipc_alloc(n, C.byref(self.ws_ptr), self.handle))
        self.peers = EpPeers()
        self.peers.workspace_dev[rank] = self.ws_ptr.value
        self.opened = []
        self.device = device
        self.side = torch.cuda.Stream(device=device)
        self.ev_dispatch = torch.cuda.Event()
        self.ev_shared = torch.cuda.Event()

    def connect_local(self, ops_per_rank):
        for o in ops_per_rank:
            self.peers.workspace_dev[o.rank] = o.ws_ptr.value

    def connect(self, group=None):
        import torch.distributed as dist
        torch = self.torch
        dev = self.device if dist.get_backend(group) == "nccl" else "cpu"
        mine = torch.tensor(list(bytes(self.handle)), dtype=torch.uint8, device=dev)
        allh = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(allh, mine, group=group)
        for s in range(self.world):
            if s == self.rank:
                continue
            h = (C.c_uint8 * IPC_HANDLE_BYTES)(*allh[s].cpu().tolist())
            p = C.c_void_p()
            check(lib().gtm_ipc_open(h, C.byref(p)))
            self.opened.append(p)
            self.peers.workspace_dev[s] = p.value

    def close(self):
        """Unmaps the peers' workspaces and frees the own one (after a barrier: no peer may
        still read or write it)."""
        for p in self.opened:
            check(lib().gtm_ipc_close(p))
        self.opened = []
        if self.ws_ptr.value:
            check(lib().gtm_ipc_free(self.ws_ptr))
            self.ws_ptr = C.c_void_p()

    _io = CudaEpOps._io

    def dispatch(self, x, **kw):
        io = self._io(x, **kw)
        check(lib().gtm_moe_ep_peer_dispatch(C.byref(self.dims), C.byref(self.layer), C.byref(io),
                                             C.byref(self.cfg), C.byref(self.peers), self.ws_bytes, _stream()))
        self.ev_dispatch.record()

    def shared(self, x, **kw):
        io = self._io(x, **kw)
        self.side.wait_event(self.ev_dispatch)
        check(lib().gtm_moe_ep_peer_shared(C.byref(self.dims), C.byref(self.layer), C.byref(io),
                                           C.byref(self.cfg), self.ws_ptr, self.ws_bytes, _stream(self.side)))
        self.ev_shared.record(self.side)

    def experts(self):
        check(lib().gtm_moe_ep_peer_experts(C.byref(self.dims), C.byref(self.layer), C.byref(self.cfg),
                                            C.byref(self.peers), self.ws_bytes, _stream()))

    def combine(self, x, hidden_out, **kw):
        io = self._io(x, hidden_out=hidden_out, **kw)
        self.torch.cuda.current_stream().wait_event(self.ev_shared)
        check(lib().gtm_moe_ep_peer_combine(C.byref(self.dims), C.byref(self.layer), C.byref(io),
                                            C.byref(self.cfg), self.ws_ptr, self.ws_bytes, _stream()))

    def check(self):
        check(lib().gtm_moe_ep_check(self.ws_ptr, _stream()))


class EpShardModel:
    """One layer of random-init weights for rank `rank`: the resident tensors (router, shared
    expert, norms; replicated) and only this rank's experts, generated on the device."""

    def __init__(self, layer_index: int, rank: int, world: int, seed: int = 0, device: str = "cuda"):
        import torch
        _, stride = expert_layout()
        _, rtotal = resident_layout()
        e0, e1 = experts_of(rank, world)
        self.resident = torch.empty(rtotal, dtype=torch.uint8, device=device)
        self.experts = torch.empty((e1 - e0) * stride, dtype=torch.uint8, device=device)
        L = lib()
        check(L.gtm_synth_resident(seed, layer_index, HIDDEN, 2112, EXPERTS, ptr(self.resident), _stream()))
        check(L.gtm_synth_experts(seed, layer_index, HIDDEN, MOE_INTER, e0, e1 - e0, ptr(self.experts), _stream()))
        self.layer = Layer()
        check(L.gtm_synth_layer_desc(HIDDEN, MOE_INTER, 2112, EXPERTS, ptr(self.resident), ptr(self.experts),
                                     C.byref(self.layer)))

    def weight_bytes(self) -> int:
        return self.resident.numel() + self.experts.numel()

"""Launched by tests/test_ep_multigpu.py under torch.distributed.run: one process per GPU runs
the expert-parallel layer on its share of 4096 bf16 tokens with uniform routing logits, over
NCCL all-to-all (EP_MODE=nccl: gtmoe.ep.ep_layer + NcclExchange) or over peer memory
(EP_MODE=peer: gtmoe.ep.ep_layer_peer + PeerEpOps, workspaces mapped through CUDA IPC); rank 0
gathers the outputs and compares them with the single-GPU path over all tokens (bit-identical)
and the top-8 indices. The layer runs twice, so the second call meets the first one's data."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "turbo-winfare_b200")]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import gtmoe  # noqa: E402
from gtmoe import ep, workloads  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    D, K, T = gtmoe.HIDDEN, gtmoe.TOP_K, int(os.environ.get("EP_TOKENS", "4096"))
    Tp = T // world
    x32 = torch.empty(T * D, device="cuda")
    gtmoe.synth_x(0, 0, T, x32)
    x = x32.view(T, D).to(torch.bfloat16)
    rl = torch.from_numpy(workloads.uniform_route_logits(T)).cuda()
    shard = ep.EpShardModel(0, rank, world)
    mode = os.environ.get("EP_MODE", "nccl")
    out = torch.empty(Tp, D, device="cuda")
    idx = torch.empty(Tp, K, dtype=torch.int32, device="cuda")
    sl = slice(rank * Tp, (rank + 1) * Tp)
    if mode == "peer":
        ops = ep.PeerEpOps(shard.layer, rank, world, max_tokens=Tp)
        ops.connect()
        bar = ep.NcclBarrier()
        for _ in range(2):
            ep.ep_layer_peer(ops, bar, x[sl], out, topk_idx=idx, route_logits=rl[sl])
    else:
        ops = ep.CudaEpOps(shard.layer, rank, world, max_tokens=Tp, max_recv_rows=T * K)
        for _ in range(2):
            ep.ep_layer(ops, ep.NcclExchange(), x[sl], out, topk_idx=idx, route_logits=rl[sl])
    ops.check()
    outs = [torch.empty_like(out) for _ in range(world)]
    idxs = [torch.empty_like(idx) for _ in range(world)]
    dist.all_gather(outs, out)
    dist.all_gather(idxs, idx)
    ok = True
    if rank == 0:
        full = gtmoe.SynthModel(1, seed=0)
        blk = gtmoe.TokenBlock(T)
        ref = torch.empty(T, D, device="cuda")
        ridx = torch.empty(T, K, dtype=torch.int32, device="cuda")
        blk(full.layers[0], x, ref, topk_idx=ridx, route_logits=rl)
        blk.check()
        got = torch.cat(outs)
        ok = torch.equal(torch.cat(idxs), ridx) and torch.equal(got, ref)
        print(f"EP {mode} world={world}: top-8 equal and outputs bit-identical to one GPU: {ok}; "
              f"max diff {float((got - ref).abs().max()):.3e}", flush=True)
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.broadcast(flag, 0)
    if mode == "peer":
        torch.cuda.synchronize()
        dist.barrier()        # no rank still reads or writes a peer's workspace
        ops.close()
        dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if int(flag.item()) == 1 else 1)


if __name__ == "__main__":
    main()

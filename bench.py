"""Benchmark of the B200 MoE block (BASELINE metric: MoE-layer tokens/s and achieved HBM GB/s).

Default workload: batch-1 decode through a 30-layer stack of the config-0
MoE block (hidden 2816, 128 experts, top-8, expert intermediate 704, shared expert 2112, MLX
affine int4 group 64, int8 router), random-init weights resident in HBM (~13 GB), a weightless
RMSNorm between layers, a different synthetic token every step. One step = one token through
the 30 layers = 30 MoE-layer tokens = one gtm_moe_decode launch.

  value   device-resident inputs, CUDA events around K steps, max over ranks
  e2e     the same through the public API with host buffers: each step copies its token from
          pinned host memory to the device and reads the result back, inside the timed region
  roofline  algorithmic weight bytes per launch / mean launch time vs MEASURED_PEAKS hbm_gbs

Multi-GPU (--gpus N under torchrun): batch-1 decode does not shard (one token's all-to-all
would cost more than the layer), so each rank runs an independent replica ("weak" scaling).

Other workloads (--workload), parity configs measured on request, not the default line:
  batch64      BASELINE config 2: 64 tokens per step through one layer, router logits biased to
               Zipf(1.1) expert popularity (gtm_moe_tokens); N>1 runs replicas
  prefill4096  BASELINE config 3: 4096 bf16 tokens per step through one layer, uniform routing
               logits; with N GPUs the layer is expert-parallel (128/N experts and 4096/N tokens
               per rank, NCCL all-to-all dispatch and combine, gtmoe.ep)

--impl reference runs the reference's own CPU arithmetic (src/cpu_reference.cpp compiled from
its sources into oracle/_ref/libgtref.so, single-threaded as shipped) on every host core in
parallel processes, for the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "turbo-winfare_b200"))
sys.path.insert(0, ROOT)

LAYERS_DEFAULT = 30
METRIC = "MoE-layer tokens/s (batch-1 decode, 30-layer stack)"
UNIT = "layer-tokens/s"
# algorithmic bytes per token per MoE layer: 8 routed experts (3 int4 matrices + bf16
# scales/biases each) + shared expert + int8 router (+ bf16 per-row scales/biases)
EXPERT_BYTES = 3 * (704 * 2816 // 2 + 2 * 704 * 44 * 2)          # 3,345,408
SHARED_BYTES = 3 * (2112 * 2816 // 2 + 2 * 2112 * 44 * 2)        # 10,036,224
ROUTER_BYTES = 128 * 2816 + 2 * 128 * 44 * 2                     # 382,976
LAYER_BYTES = 8 * EXPERT_BYTES + SHARED_BYTES + ROUTER_BYTES      # 37,182,464
NORM_BYTES = 6 * 2816 * 2 + 128 * 2 + 2                           # norm weights, per-expert scale, scalar
LAYER_FLOPS = 2 * (8 * 3 * 704 * 2816 + 3 * 2112 * 2816 + 128 * 2816)  # 131,563,520


def peaks(kind: str = "hbm"):
    """(peak, source): HBM GB/s or dense bf16 TFLOP/s (burst) of this pool's B200s."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return (float(d["hbm_gbs"]) if kind == "hbm" else float(d["bf16_tflops"])), "measured"
    return (6650.0 if kind == "hbm" else 1590.0), "fallback"


class ClockSampler:
    """SM clocks and throttle reasons sampled during the timed region.

    A thread polls NVML every 5 ms between __enter__ and __exit__; `sample()` called right
    before the closing synchronize adds one reading taken while the queued steps still run, so a
    timed region of a few milliseconds has at least one sample under load. Falls back to
    `nvidia-smi -lms 200` when NVML cannot be opened. Only reads; changes no GPU setting."""

    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu: int):
        self.gpu, self.samples, self.proc, self.nv, self.h = gpu, [], None, None, None
        self.stop = threading.Event()
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            try:
                import torch
                p = torch.cuda.get_device_properties(gpu)
                bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
                self.h = nv.nvmlDeviceGetHandleByPciBusId_v2(bus)
            except Exception:
                self.h = nv.nvmlDeviceGetHandleByIndex(gpu)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
            g = lambda n, d: getattr(nv, n, d)
            self.bits = [g("nvmlClocksEventReasonHwSlowdown", g("nvmlClocksThrottleReasonHwSlowdown", 0x8)),
                         g("nvmlClocksEventReasonHwThermalSlowdown", g("nvmlClocksThrottleReasonHwThermalSlowdown", 0x40)),
                         g("nvmlClocksEventReasonSwThermalSlowdown", g("nvmlClocksThrottleReasonSwThermalSlowdown", 0x20)),
                         g("nvmlClocksEventReasonSwPowerCap", g("nvmlClocksThrottleReasonSwPowerCap", 0x4))]
            self._reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception:
            self.nv = None

    def sample(self):
        if self.nv is None:
            return
        try:
            mhz = float(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            r = int(self._reasons(self.h))
            self.samples.append((mhz, self.max_mhz, [n for n, b in zip(self.NAMES, self.bits) if r & b]))
        except Exception:
            pass

    def _poll(self):
        while not self.stop.wait(0.005):
            self.sample()

    def _read_smi(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                self.samples.append((float(parts[1]), float(parts[2]) if parts[2].replace(".", "").isdigit() else None,
                                     [n for i, n in enumerate(self.NAMES) if parts[5 + i] == "Active"]))

    def __enter__(self):
        if self.nv is not None:
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return self
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read_smi, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.stop.set()
        if self.nv is not None:
            self.t.join(timeout=1)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(s[0] for s in self.samples)
        mx = max((s[1] for s in self.samples if s[1] is not None), default=None)
        reasons = sorted({n for s in self.samples for n in s[2]})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(self.samples), "source": "nvml" if self.nv is not None else "nvidia-smi"}


def cpu_reference_worker(args):
    """Runs the reference's compiled MoE arithmetic for `seconds`; returns layer-tokens done."""
    seconds, worker, layers, impl = args
    import oracle
    ls = [oracle.SynthLayer(0, l) for l in range(layers)]
    x = oracle.synth_x(0, worker)
    # materialise the experts outside the timed loop
    for L in ls:
        x = L.block(x, impl=impl)["hidden"]
    x = oracle.synth_x(0, worker)
    done, t0 = 0, time.perf_counter()
    while True:
        for L in ls:
            x = L.block(x, impl=impl)["hidden"]
            x = oracle.rms_norm(x, None, impl=impl)
            done += 1
        if time.perf_counter() - t0 >= seconds:
            break
    return done, time.perf_counter() - t0


def cpu_baseline(seconds: float, processes: int, layers: int = 2):
    """Reference CPU arithmetic on `processes` host cores (spawned before any GPU use)."""
    import multiprocessing as mp
    import oracle
    # the reference's own helpers when their prebuilt library is present, else the restated port
    kind, impl = ("reference", "ref") if oracle.ref_available() else ("port", "oracle")
    ctx = mp.get_context("spawn")
    with ctx.Pool(processes) as pool:
        res = pool.map(cpu_reference_worker, [(seconds, w, layers, impl) for w in range(processes)])
    total = sum(r[0] for r in res)
    wall = max(r[1] for r in res)
    src = "oracle/_ref (src/cpu_reference.cpp compiled)" if kind == "reference" else "oracle port"
    return {"value": total / wall, "unit": UNIT, "cores": processes, "kind": kind,
            "sample": f"{total} layer-tokens of config-1 layers 0..{layers - 1} (block + between-layer norm), "
                      f"{processes} process(es) x ~{seconds:.0f} s, {src}"}


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cores = len(os.sched_getaffinity(0))
    per_step = max(2.0, 20.0 / max(1, args.steps + args.warmup))
    if args.workload != "decode30":
        # the token workloads: the reference runs its block one token at a time on the CPU
        cfg = args.workload
        cb = token_cpu_baseline(per_step * args.steps, cfg, cores)
        line = {"impl": "reference", "metric": TOKEN_METRIC[cfg], "value": cb["value"], "unit": "tokens/s",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": 1000.0 * TOKENS_PER_STEP[cfg] / cb["value"], "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": TOKEN_WORKLOAD[cfg] + " (CPU sample)", "tokens_per_step": TOKENS_PER_STEP[cfg]},
                "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0
    cb = cpu_baseline(per_step * args.steps, cores)
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * LAYERS_DEFAULT / cb["value"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config1: batch-1 decode, 30-layer MoE stack (CPU sample)", "layers": LAYERS_DEFAULT},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--layers", type=int, default=LAYERS_DEFAULT, help="stack depth (profiling only)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="decode30", choices=["decode30", "batch64", "prefill4096"])
    ap.add_argument("--ep", default="peer", choices=["peer", "nccl"],
                    help="prefill4096 on N>1 GPUs: expert exchange over peer memory or NCCL all-to-all")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3

    if args.impl == "reference":
        return run_reference_arm(args)
    if args.workload != "decode30":
        return bench_tokens(args)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    # CPU baseline first: worker processes are spawned before this process touches the GPU
    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(args.cpu_seconds, 1)

    import torch
    import gtmoe
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))

    L = args.layers
    model = gtmoe.SynthModel(L, seed=0)
    dec = gtmoe.Decoder(model.layers, L)
    n_tok = args.warmup + args.steps
    D = gtmoe.HIDDEN
    xs = torch.empty(n_tok * D, device="cuda")
    gtmoe.synth_x(0, rank * n_tok, n_tok, xs)
    out = torch.empty(D, device="cuda")
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-resident timing ----
    for i in range(args.warmup):
        dec(xs[i * D:(i + 1) * D], out)
    dec.check()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for i in range(args.steps):
            j = args.warmup + i
            dec(xs[j * D:(j + 1) * D], out)
        ev1.record(stream)
        clk.sample()
        torch.cuda.synchronize()
    dec.check()
    ms = ev0.elapsed_time(ev1)
    barrier()
    # ---- end to end through host buffers ----
    xh = torch.empty((n_tok, D), dtype=torch.float32, pin_memory=True)
    xh.copy_(xs.view(n_tok, D).cpu())
    oh = torch.empty((args.steps, D), dtype=torch.float32, pin_memory=True)
    xin = torch.empty(D, device="cuda")
    for i in range(args.warmup):
        xin.copy_(xh[i], non_blocking=True)
        dec(xin, out)
        oh[0].copy_(out, non_blocking=True)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        xin.copy_(xh[args.warmup + i], non_blocking=True)
        dec(xin, out)
        oh[i].copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    dec.check()
    ms_e2e = e0.elapsed_time(e1)

    if dist is not None:
        t = torch.tensor([ms, ms_e2e], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), float(t[1])

    layer_tokens = args.steps * L * world
    value = layer_tokens / (ms / 1000.0)
    e2e = layer_tokens / (ms_e2e / 1000.0)
    per_launch_ms = ms / args.steps
    bytes_per_launch = L * (LAYER_BYTES + NORM_BYTES)
    achieved = bytes_per_launch / (per_launch_ms / 1000.0) / 1e9
    peak, peak_kind = peaks()
    traffic = None
    tp = os.path.join(ROOT, "profiles", "decode_traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            tj = json.load(f)
        traffic = tj.get("bytes_per_layer", 0) * L if tj.get("bytes_per_layer") else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": per_launch_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"config1: batch-1 decode, {L}-layer MoE stack (hidden 2816, 128 experts top-8, "
                                   f"int4 experts 704, shared 2112, int8 router), weights HBM-resident",
                       "layers": L, "tokens_per_s": value / L, "weights_gb": model.weight_bytes() / 1e9,
                       "l2": "inputs larger than L2: 1.1 GB of distinct weights touched per step, new token per step",
                       "parallelism": "replicas" if world > 1 else "single"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": peak_kind, "traffic": traffic,
                         "algorithmic_bytes_per_launch": bytes_per_launch,
                         "tflops": L * LAYER_FLOPS / (per_launch_ms / 1000.0) / 1e12},
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": D * 4, "d2h_bytes_per_step": D * 4},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
            "cpu_baseline": cb,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ---- T > 1 workloads (configs 2 and 3) ------------------------------------------------------------
WEIGHT_BYTES_EXPERT = EXPERT_BYTES


TOKEN_METRIC = {"batch64": "MoE-layer tokens/s (batch 64 decode, Zipf routing)",
                "prefill4096": "MoE-layer tokens/s (prefill 4096 bf16 tokens)"}
TOKEN_WORKLOAD = {"batch64": "config2: 64 tokens through one MoE layer, Zipf(1.1) router bias",
                  "prefill4096": "config3: 4096 bf16 tokens through one MoE layer, uniform routing logits"}
TOKENS_PER_STEP = {"batch64": 64, "prefill4096": 4096}


def token_cpu_baseline(seconds: float, cfg: str, processes: int = 1):
    """The reference's CPU arithmetic on a bounded sample of the workload's tokens (rank 0),
    in `processes` spawned processes (one token at a time each, as the reference runs them)."""
    import multiprocessing as mp
    import oracle
    kind, impl = ("reference", "ref") if oracle.ref_available() else ("port", "oracle")
    ctx = mp.get_context("spawn")
    with ctx.Pool(processes) as pool:
        res = pool.map(token_cpu_worker, [(seconds, cfg, impl)] * processes)
    done = sum(r[0] for r in res)
    wall = max(r[1] for r in res)
    return {"value": done / wall, "unit": "tokens/s", "cores": processes, "kind": kind,
            "sample": f"{done} tokens of the {cfg} workload through layer 0 ({processes} process(es), ~{seconds:.0f} s)"}


def token_cpu_worker(a):
    seconds, cfg, impl = a
    import numpy as np
    import oracle
    from gtmoe import workloads
    L = oracle.SynthLayer(0, 0)
    bias = workloads.zipf_logit_bias() if cfg == "batch64" else None
    rl = workloads.uniform_route_logits(64) if cfg == "prefill4096" else None
    xs = [oracle.synth_x(0, t) for t in range(64)]
    if cfg == "prefill4096":
        xs = [workloads.bf16_round(x) for x in xs]
    for t in range(4):   # materialise experts outside the timed loop
        L.block(xs[t], logit_bias=bias, route_logits=None if rl is None else rl[t], impl=impl)
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        t = done % 64
        L.block(xs[t], logit_bias=bias, route_logits=None if rl is None else rl[t], impl=impl)
        done += 1
    return done, time.perf_counter() - t0


def bench_tokens(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg = args.workload
    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = token_cpu_baseline(args.cpu_seconds, cfg)

    import numpy as np
    import torch
    import gtmoe
    from gtmoe import ep, workloads
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    D, K = gtmoe.HIDDEN, gtmoe.TOP_K
    T_total = 64 if cfg == "batch64" else 4096
    expert_parallel = cfg == "prefill4096" and world > 1
    T = T_total // world if expert_parallel else T_total
    n_sets = 4   # distinct token batches cycled over the steps
    x32 = torch.empty(n_sets * T * D, device="cuda")
    gtmoe.synth_x(0, rank * n_sets * T, n_sets * T, x32)
    xs = x32.view(n_sets, T, D)
    kw = {}
    if cfg == "batch64":
        kw["logit_bias"] = torch.from_numpy(workloads.zipf_logit_bias()).cuda()
    else:
        xs = xs.to(torch.bfloat16)
        rl_all = torch.from_numpy(workloads.uniform_route_logits(n_sets * T_total)).cuda().view(n_sets, T_total, -1)
        rl = rl_all[:, rank * T:(rank + 1) * T] if expert_parallel else rl_all
    out = torch.empty(T, D, device="cuda")
    idx_hist = torch.empty(n_sets, T, K, dtype=torch.int32, device="cuda")

    # kernels of ours per step (the NCCL collectives not counted): views 1, routing 3 (count, scan,
    # scatter), gather 1, grouped GEMMs 2, combine 1; expert parallelism adds the dispatch (NCCL:
    # 2 kernels; peer memory: the token-count word) and the shared-expert pass (scan + 2 GEMMs)
    launches = 8
    if expert_parallel:
        shard = ep.EpShardModel(0, rank, world)
        weights_gb = shard.weight_bytes() / 1e9
        rl_c = [rl[j].contiguous() for j in range(n_sets)]
        if args.ep == "peer":
            ops = ep.PeerEpOps(shard.layer, rank, world, max_tokens=T)
            ops.connect()
            bar = ep.NcclBarrier()
            launches = 12

            def step(i, x=None, o=None):
                j = i % n_sets
                ep.ep_layer_peer(ops, bar, xs[j] if x is None else x, out if o is None else o,
                                 topk_idx=idx_hist[j], route_logits=rl_c[j], **kw)
        else:
            ops = ep.CudaEpOps(shard.layer, rank, world, max_tokens=T, max_recv_rows=T_total * K)
            xch = ep.NcclExchange()
            launches = 13

            def step(i, x=None, o=None):
                j = i % n_sets
                ep.ep_layer(ops, xch, xs[j] if x is None else x, out if o is None else o, topk_idx=idx_hist[j],
                            route_logits=rl_c[j], **kw)
        check = ops.check
    else:
        model = gtmoe.SynthModel(1, seed=0)
        blk = gtmoe.TokenBlock(T)
        weights_gb = model.weight_bytes() / 1e9

        def step(i, x=None, o=None):
            j = i % n_sets
            a = dict(kw)
            if cfg == "prefill4096":
                a["route_logits"] = rl[j]
            blk(model.layers[0], xs[j] if x is None else x, out if o is None else o, topk_idx=idx_hist[j], **a)
        check = blk.check
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(args.warmup):
        step(i)
    check()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
        clk.sample()
        torch.cuda.synchronize()
    check()
    ms = ev0.elapsed_time(ev1)
    barrier()
    # end to end, as a serving host runs it: every step's tokens go host -> device and its result
    # device -> host inside the timed region, on two copy streams with double buffers, so the copies
    # of steps i + 1 and i - 1 overlap the compute of step i
    xh = torch.empty((n_sets, T, D), dtype=xs.dtype, pin_memory=True)
    xh.copy_(xs.cpu())
    oh = [torch.empty((T, D), dtype=torch.float32, pin_memory=True) for _ in range(2)]
    xin = [torch.empty(T, D, dtype=xs.dtype, device="cuda") for _ in range(2)]
    outs = [torch.empty(T, D, device="cuda") for _ in range(2)]
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]   # the buffer's last step has computed
    ev_out = [torch.cuda.Event() for _ in range(2)]    # the buffer's last result is on the host

    def run_e2e(n):
        for i in range(n):
            b = i % 2
            with torch.cuda.stream(h2d):
                if i >= 2:
                    h2d.wait_event(ev_used[b])
                xin[b].copy_(xh[i % n_sets], non_blocking=True)
                ev_in[b].record(h2d)
            stream.wait_event(ev_in[b])
            if i >= 2:
                stream.wait_event(ev_out[b])
            step(i, xin[b], outs[b])
            ev_used[b].record(stream)
            with torch.cuda.stream(d2h):
                d2h.wait_event(ev_used[b])
                oh[b].copy_(outs[b], non_blocking=True)
                ev_out[b].record(d2h)
        stream.wait_stream(d2h)

    run_e2e(args.warmup)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run_e2e(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    check()
    ms_e2e = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms, ms_e2e], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), float(t[1])
    per_step_ms = ms / args.steps
    tokens_per_step = T_total if expert_parallel else T * world
    value = tokens_per_step * args.steps / (ms / 1000.0)
    e2e = tokens_per_step * args.steps / (ms_e2e / 1000.0)
    ids = idx_hist.cpu().numpy()
    distinct = float(np.mean([len(np.unique(ids[j])) for j in range(n_sets)]))
    act_bytes = T * D * (2 if cfg == "prefill4096" else 4) + T * D * 4
    if cfg == "batch64":
        alg = distinct * EXPERT_BYTES + SHARED_BYTES + ROUTER_BYTES + act_bytes
        achieved = alg / (per_step_ms / 1000.0) / 1e9
        peak, pk = peaks("hbm")
        roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "peak_source": pk, "traffic": None, "algorithmic_bytes_per_step": alg,
                "scope": "whole layer call (views, routing, two grouped GEMMs, combine)",
                "distinct_experts_per_step": distinct}
        metric = TOKEN_METRIC[cfg]
    else:
        flops = T_total * (LAYER_FLOPS - 2 * 128 * 2816)   # experts + shared (routing logits given)
        achieved = flops / (per_step_ms / 1000.0) / 1e12 / (world if expert_parallel else 1)
        peak, pk = peaks("tensor")
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_source": pk, "traffic": None, "flops_per_step": flops,
                "scope": "whole layer call, useful FLOPs per GPU (the fp16 high/low activation split doubles "
                         "the tensor-core work)"}
        metric = TOKEN_METRIC[cfg]
    if rank == 0:
        line = {
            "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": per_step_ms, "higher_is_better": True,
            "scaling": "strong" if expert_parallel else "weak", "vs_baseline": None,
            "dtype": "f32 (fp16 hi/lo tensor-core operands)", "data": "synthetic",
            "config": {"workload": TOKEN_WORKLOAD[cfg],
                       "tokens_per_step": tokens_per_step, "weights_gb_per_gpu": weights_gb,
                       "parallelism": (f"ep{world}" if expert_parallel else ("replicas" if world > 1 else "single")),
                       **({"ep_exchange": ("peer memory (CUDA IPC, NVLink loads/stores)" if args.ep == "peer"
                                           else "NCCL all-to-all")} if expert_parallel else {}),
                       "l2": "4 token sets cycled; weights of touched experts 0.3-0.45 GB > L2"},
            "roofline": roof,
            "e2e": {"value": e2e, "unit": "tokens/s", "copies": "two copy streams, double buffers: the copies of "
                    "steps i+1 and i-1 overlap step i", "h2d_bytes_per_step": T * D * xs.element_size(),
                    "d2h_bytes_per_step": T * D * 4},
            "gpu_launches": args.steps * launches,
            "clocks": clk.summary(),
            "cpu_baseline": cb,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        if expert_parallel and args.ep == "peer":
            torch.cuda.synchronize()
            ops.close()
            dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

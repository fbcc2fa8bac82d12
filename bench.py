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


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    def __init__(self, gpu: int):
        self.gpu, self.samples, self.proc = gpu, [], None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit())
        mx = max((float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[5 + i] == "Active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(self.samples)}


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
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3

    if args.impl == "reference":
        return run_reference_arm(args)

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


if __name__ == "__main__":
    sys.exit(main())

"""Benchmark of the B200 MoE block (BASELINE metric: MoE-layer tokens/s and achieved HBM GB/s or
tensor %, at 1/2/4/8 B200).

Default workload: prefill of 4096 bf16 tokens (x ~ N(0,1), a different token
set each step from 4 cycled sets) through one config-0 MoE layer (hidden 2816, 128 experts,
top-8 over uniform-random routing logits, expert intermediate 704, shared expert 2112, MLX affine
int4 group 64), random-init weights resident in HBM. One step = one layer call over the 4096
tokens:
  N = 1   gtm_moe_tokens (views, routing, tcgen05 grouped gate/up and down GEMMs, combine)
  N > 1   expert parallel over NVLink peer memory: 128/N experts and 4096/N tokens per rank
          (gtmoe.ep.ep_layer_peer; --ep nccl for the NCCL all-to-all variant)

  value     tokens/s of the whole job, device-resident inputs, CUDA events around K steps, max
            over ranks
  e2e       the same through the public API as a serving host runs it: each step's tokens go
            host -> device and its output device -> host inside the timed region (two copy
            streams, double buffers)
  roofline  the dominant kernels (the two grouped GEMMs, timed live with gtm_set_phase_events at
            N = 1): useful expert + shared-expert FLOPs / their time vs the measured bf16 peak;
            at N > 1 the whole per-GPU step
  parity    outside the timed region, one step's outputs against the CPU oracle: every token's
            top-8, and h1, h2 and the new residual of a sample (all ranks' tokens at N > 1)
  extra     at N = 1 the other single-GPU BASELINE configs measured in the same run: config 1
            (batch-1 decode through the 30-layer stack, HBM roofline) and config 2 (64 tokens,
            Zipf(1.1) routing, HBM roofline)

--workload decode30|batch64 makes config 1 or config 2 the main line (N > 1: replicas).
--workload decode_batch32 is BASELINE config 4: greedy decode of 32 sequences (1024-token
random-id prompts, 64 generated tokens) through a 30-layer Gemma-4-26B-A4B-shaped random-init
model (vocab 262144, sliding/full attention, MoE as config 0) with gtmoe.batch.BatchDecoder; at
N > 1 the sequences split over the ranks and the experts are sharded (expert parallel over peer
memory). Metric: generated tokens/s of the whole job; prefill tokens/s beside it.

--impl reference runs the reference's own CPU arithmetic (src/cpu_reference.cpp compiled from
its sources into oracle/_ref/libgtref.so, single-threaded as shipped, one token at a time as its
prefill runs) on every host core in parallel processes, for the same metric and config.
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
TOL = 2e-3
# algorithmic bytes per token per MoE layer: 8 routed experts (3 int4 matrices + bf16
# scales/biases each) + shared expert + int8 router (+ bf16 per-row scales/biases)
EXPERT_BYTES = 3 * (704 * 2816 // 2 + 2 * 704 * 44 * 2)          # 3,345,408
SHARED_BYTES = 3 * (2112 * 2816 // 2 + 2 * 2112 * 44 * 2)        # 10,036,224
ROUTER_BYTES = 128 * 2816 + 2 * 128 * 44 * 2                     # 382,976
LAYER_BYTES = 8 * EXPERT_BYTES + SHARED_BYTES + ROUTER_BYTES      # 37,182,464
NORM_BYTES = 6 * 2816 * 2 + 128 * 2 + 2                           # norm weights, per-expert scale, scalar
LAYER_FLOPS = 2 * (8 * 3 * 704 * 2816 + 3 * 2112 * 2816 + 128 * 2816)  # 131,563,520
EXPERT_SHARED_FLOPS = LAYER_FLOPS - 2 * 128 * 2816                # routing logits given (config 3)

WORKLOADS = ("prefill4096", "batch64", "decode30", "decode_batch32")
METRIC = {"prefill4096": "MoE-layer tokens/s (prefill 4096 bf16 tokens)",
          "batch64": "MoE-layer tokens/s (batch 64 decode, Zipf routing)",
          "decode30": "MoE-layer tokens/s (batch-1 decode, 30-layer stack)",
          "decode_batch32": "generated tokens/s (greedy decode, 32 sequences, 30-layer model)"}
UNIT = {"prefill4096": "tokens/s", "batch64": "tokens/s", "decode30": "layer-tokens/s", "decode_batch32": "tokens/s"}
WORKLOAD_TEXT = {
    "prefill4096": "config3: 4096 bf16 tokens through one MoE layer (hidden 2816, 128 experts top-8, int4 experts "
                   "704, shared 2112), uniform routing logits",
    "batch64": "config2: 64 tokens through one MoE layer, Zipf(1.1) router bias",
    "decode30": "config1: batch-1 decode, 30-layer MoE stack (hidden 2816, 128 experts top-8, int4 experts 704, "
                "shared 2112, int8 router), weights HBM-resident",
    "decode_batch32": "config4: 30-layer Gemma-4-26B-A4B-shaped model (vocab 262144, hidden 2816, MoE as config 0), "
                      "32 sequences, 1024-token random-id prompts, 64 greedy tokens"}
TOKENS_PER_STEP = {"prefill4096": 4096, "batch64": 64}


def bench_config(workload: str, world: int, ep_mode: str) -> dict:
    """The line's `config`: static descriptors only, so the reference arm prints the same one."""
    if workload == "decode_batch32":
        return {"workload": WORKLOAD_TEXT[workload], "sequences": 32, "prompt_tokens": 1024, "new_tokens": 64,
                "layers": LAYERS_DEFAULT, "parallelism": f"ep{world}" if world > 1 else "single"}
    if workload == "decode30":
        return {"workload": WORKLOAD_TEXT[workload], "layers": LAYERS_DEFAULT,
                "l2": "inputs larger than L2: 1.1 GB of distinct weights touched per step, new token per step",
                "parallelism": "replicas" if world > 1 else "single"}
    ep = workload == "prefill4096" and world > 1
    c = {"workload": WORKLOAD_TEXT[workload],
         "tokens_per_step": TOKENS_PER_STEP[workload] * (1 if ep else world),
         "parallelism": f"ep{world}" if ep else ("replicas" if world > 1 else "single"),
         "l2": "4 token sets cycled; weights of touched experts 0.3-0.45 GB > L2"}
    if ep:
        c["ep_exchange"] = ("peer memory (CUDA IPC, NVLink stores from the kernels, two NCCL barriers)"
                            if ep_mode == "peer" else "NCCL all-to-all")
    return c


def peaks(kind: str = "hbm"):
    """(peak, source): HBM GB/s or dense bf16 TFLOP/s (burst) of this pool's B200s."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return (float(d["hbm_gbs"]) if kind == "hbm" else float(d["bf16_tflops"])), "measured"
    return (6650.0 if kind == "hbm" else 1590.0), "fallback"


def profile_traffic(name: str):
    """DRAM bytes per step from an ncu capture summarised under profiles/ (or None)."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return json.load(f)


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


# ---- CPU legs: the reference's arithmetic (the checker, never the thing measured) -------------------

def cpu_reference_worker(args):
    """Runs the reference's compiled MoE arithmetic for `seconds`; returns layer-tokens done."""
    seconds, worker, layers, impl = args
    import oracle
    ls = [oracle.SynthLayer(0, l) for l in range(layers)]
    x = oracle.synth_x(0, worker)
    for L in ls:   # materialise the experts outside the timed loop
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


def decode_cpu_baseline(seconds: float, processes: int, layers: int = 2):
    """Reference CPU arithmetic of the decode stack on `processes` host cores (spawned before any
    GPU use)."""
    import multiprocessing as mp
    import oracle
    kind, impl = ("reference", "ref") if oracle.ref_available() else ("port", "oracle")
    with mp.get_context("spawn").Pool(processes) as pool:
        res = pool.map(cpu_reference_worker, [(seconds, w, layers, impl) for w in range(processes)])
    total = sum(r[0] for r in res)
    wall = max(r[1] for r in res)
    src = "oracle/_ref (src/cpu_reference.cpp compiled)" if kind == "reference" else "oracle port"
    return {"value": total / wall, "unit": UNIT["decode30"], "cores": processes, "kind": kind,
            "sample": f"{total} layer-tokens of config-1 layers 0..{layers - 1} (block + between-layer norm), "
                      f"{processes} process(es) x ~{seconds:.0f} s, {src}"}


def token_cpu_worker(a):
    seconds, cfg, impl = a
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


def token_cpu_baseline(seconds: float, cfg: str, processes: int = 1):
    """The reference's CPU arithmetic on a bounded sample of the workload's tokens, one token at a
    time as the reference runs its prefill, in `processes` spawned processes."""
    import multiprocessing as mp
    import oracle
    kind, impl = ("reference", "ref") if oracle.ref_available() else ("port", "oracle")
    with mp.get_context("spawn").Pool(processes) as pool:
        res = pool.map(token_cpu_worker, [(seconds, cfg, impl)] * processes)
    done = sum(r[0] for r in res)
    wall = max(r[1] for r in res)
    return {"value": done / wall, "unit": "tokens/s", "cores": processes, "kind": kind,
            "sample": f"{done} tokens of the {cfg} workload through layer 0, one at a time "
                      f"({processes} process(es) x ~{seconds:.0f} s)"}


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    cores = len(os.sched_getaffinity(0))
    per_step = max(2.0, 20.0 / max(1, args.steps + args.warmup))
    cfg = args.workload
    if cfg == "decode_batch32":
        print(json.dumps({"impl": "reference", "metric": METRIC[cfg], "unit": UNIT[cfg], "config": bench_config(cfg, world, args.ep),
                          "unavailable": "the reference decodes on its CPU at about 14 s per token of this model; "
                                         "35,000 tokens of config 4 do not fit a bounded run (its per-layer cost is "
                                         "the decode30 arm)"}), flush=True)
        return 0
    if cfg == "decode30":
        cb = decode_cpu_baseline(per_step * args.steps, cores)
        ms = 1000.0 * LAYERS_DEFAULT / cb["value"]
    else:
        cb = token_cpu_baseline(per_step * args.steps, cfg, cores)
        ms = 1000.0 * bench_config(cfg, world, args.ep)["tokens_per_step"] / cb["value"]
    line = {"impl": "reference", "metric": METRIC[cfg], "value": cb["value"], "unit": UNIT[cfg],
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong" if (cfg == "prefill4096" and world > 1) else "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": bench_config(cfg, world, args.ep),
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": UNIT[cfg], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---- parity (outside every timed region) ------------------------------------------------------------

def tokens_parity(x, idx, out, h1, h2, route_logits=None, logit_bias=None, pes=None, sample=6, token0=0):
    """Host arrays of one step's tokens: every token's top-8 against the oracle's selection and a
    sample's h1, h2 and new residual against the exact oracle (rel. to the output RMS)."""
    import numpy as np
    import oracle
    layer = oracle.SynthLayer(0, 0)
    T = x.shape[0]
    bad = 0
    for t in range(T):
        if route_logits is not None:
            want, _ = oracle.topk(route_logits[t], 8, pes)
        else:
            want = layer.route(x[t], logit_bias=logit_bias)
        bad += int(not np.array_equal(idx[t].view(np.uint32), want))
    errs = {"h1": 0.0, "h2": 0.0, "hidden": 0.0}
    picks = sorted({int(v) for v in np.linspace(0, T - 1, sample)}) if T else []
    for t in picks:
        r = layer.block(x[t], logit_bias=logit_bias, route_logits=None if route_logits is None else route_logits[t])
        bad += int(not np.array_equal(idx[t].view(np.uint32), r["idx"]))
        for k, got in (("h1", h1), ("h2", h2), ("hidden", out)):
            if got is None:
                continue
            ref = r[k].astype(np.float64)
            errs[k] = max(errs[k], float(np.abs(got[t] - ref).max() / np.sqrt(np.mean(ref ** 2))))
    return {"tokens": T, "topk_mismatch": bad, "sample": [token0 + p for p in picks], "max_rel_err": errs}


def merge_parity(parts, tol=TOL):
    tokens = sum(p["tokens"] for p in parts)
    bad = sum(p["topk_mismatch"] for p in parts)
    errs = {k: max(p["max_rel_err"][k] for p in parts) for k in ("h1", "h2", "hidden")}
    return {"ok": bad == 0 and max(errs.values()) <= tol, "tokens_topk_checked": tokens, "topk_mismatch": bad,
            "sample_tokens": sum(len(p["sample"]) for p in parts), "max_rel_err": errs, "tol": tol,
            "oracle": "oracle/moe_oracle.c (pinned to src/cpu_reference.cpp)"}


# ---- device measurements ----------------------------------------------------------------------------

def clocks_ok(c):
    return not any(r in c.get("reasons", []) for r in ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"))


def measure_decode(steps: int, warmup: int, layers: int, rank: int, local: int, dist, with_e2e=True):
    """Config 1: one token through `layers` MoE layers per step (one gtm_moe_decode launch)."""
    import torch
    import gtmoe
    model = gtmoe.SynthModel(layers, seed=0)
    dec = gtmoe.Decoder(model.layers, layers)
    n_tok = warmup + steps
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

    for i in range(warmup):
        dec(xs[i * D:(i + 1) * D], out)
    dec.check()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for i in range(steps):
            j = warmup + i
            dec(xs[j * D:(j + 1) * D], out)
        ev1.record(stream)
        clk.sample()
        torch.cuda.synchronize()
    dec.check()
    ms = ev0.elapsed_time(ev1)
    barrier()
    ms_e2e = None
    if with_e2e:
        xh = torch.empty((n_tok, D), dtype=torch.float32, pin_memory=True)
        xh.copy_(xs.view(n_tok, D).cpu())
        oh = torch.empty((steps, D), dtype=torch.float32, pin_memory=True)
        xin = torch.empty(D, device="cuda")
        for i in range(warmup):
            xin.copy_(xh[i], non_blocking=True)
            dec(xin, out)
            oh[0].copy_(out, non_blocking=True)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            xin.copy_(xh[warmup + i], non_blocking=True)
            dec(xin, out)
            oh[i].copy_(out, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        dec.check()
        ms_e2e = e0.elapsed_time(e1)
    world = 1
    if dist is not None:
        world = dist.get_world_size()
        t = torch.tensor([ms, ms_e2e or 0.0], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), (float(t[1]) if with_e2e else None)
    per_launch_ms = ms / steps
    bytes_per_launch = layers * (LAYER_BYTES + NORM_BYTES)
    achieved = bytes_per_launch / (per_launch_ms / 1000.0) / 1e9
    peak, peak_kind = peaks("hbm")
    tj = profile_traffic("decode_traffic.json")
    layer_tokens = steps * layers * world
    r = {"value": layer_tokens / (ms / 1000.0), "ms_per_step": per_launch_ms, "gpu_launches": steps,
         "weights_gb": model.weight_bytes() / 1e9,
         "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                      "peak_source": peak_kind,
                      "traffic": tj["bytes_per_layer"] * layers if tj and tj.get("bytes_per_layer") else None,
                      "algorithmic_bytes_per_launch": bytes_per_launch, "kernel": "dec::moe_decode_kernel",
                      "tflops": layers * LAYER_FLOPS / (per_launch_ms / 1000.0) / 1e12},
         "clocks": clk.summary()}
    if with_e2e:
        r["e2e"] = {"value": layer_tokens / (ms_e2e / 1000.0), "unit": UNIT["decode30"],
                    "h2d_bytes_per_step": D * 4, "d2h_bytes_per_step": D * 4}
    del dec, model, xs
    torch.cuda.empty_cache()
    return r


def measure_tokens(cfg: str, steps: int, warmup: int, rank: int, world: int, local: int, dist, ep_mode: str,
                   with_e2e=True, with_parity=True):
    """Configs 2 and 3: T tokens through one layer per step (gtm_moe_tokens, or expert parallel)."""
    import numpy as np
    import torch
    import gtmoe
    from gtmoe import ep, workloads
    D, K = gtmoe.HIDDEN, gtmoe.TOP_K
    T_total = TOKENS_PER_STEP[cfg]
    expert_parallel = cfg == "prefill4096" and world > 1
    T = T_total // world if expert_parallel else T_total
    n_sets = 4   # distinct token batches cycled over the steps
    if expert_parallel:
        # the ranks' slices of the single-GPU token sets
        full = torch.empty(n_sets * T_total * D, device="cuda")
        gtmoe.synth_x(0, 0, n_sets * T_total, full)
        xs = full.view(n_sets, T_total, D)[:, rank * T:(rank + 1) * T].contiguous()
        del full
    else:
        # replicas (N > 1 on batch64) take their own tokens
        x32 = torch.empty(n_sets * T * D, device="cuda")
        gtmoe.synth_x(0, rank * n_sets * T, n_sets * T, x32)
        xs = x32.view(n_sets, T, D)
    kw = {}
    rl_np = None
    if cfg == "batch64":
        kw["logit_bias"] = torch.from_numpy(workloads.zipf_logit_bias()).cuda()
    else:
        xs = xs.to(torch.bfloat16)
        rl_np = workloads.uniform_route_logits(n_sets * T_total).reshape(n_sets, T_total, -1)
        rl_all = torch.from_numpy(rl_np).cuda()
        rl = rl_all[:, rank * T:(rank + 1) * T] if expert_parallel else rl_all
        rl_c = [rl[j].contiguous() for j in range(n_sets)]
    out = torch.empty(T, D, device="cuda")
    idx_hist = torch.empty(n_sets, T, K, dtype=torch.int32, device="cuda")

    # kernels of ours per step (NCCL collectives not counted): views 1, routing 3 (count, scan,
    # scatter; one fused kernel when the entries fit one 1024-entry chunk), grouped GEMMs 2,
    # combine 1; peer expert parallelism adds the token-count word and the shared-expert pass
    # (scan + 2 GEMMs); the NCCL variant the dispatch pair
    launches = 7 if T * K > 1024 else 5
    phase_names = None
    if expert_parallel:
        shard = ep.EpShardModel(0, rank, world)
        weights_gb = shard.weight_bytes() / 1e9
        resident = shard.resident
        layer = shard.layer
        if ep_mode == "peer":
            ops = ep.PeerEpOps(shard.layer, rank, world, max_tokens=T)
            ops.connect()
            bar = ep.NcclBarrier()
            launches = 11
            phase_names = ("dispatch", "barrier_1", "experts", "barrier_2", "combine")

            def step(i, x=None, o=None, marks=None, **extra):
                j = i % n_sets
                a = dict(topk_idx=idx_hist[j], route_logits=rl_c[j], **kw, **extra)
                xx, oo = (xs[j] if x is None else x), (out if o is None else o)
                if marks is None:
                    ep.ep_layer_peer(ops, bar, xx, oo, **a)
                    return
                marks[0].record()
                ops.dispatch(xx, **a)
                marks[1].record()
                ops.shared(xx, **a)
                bar()
                marks[2].record()
                ops.experts()
                marks[3].record()
                bar()
                marks[4].record()
                ops.combine(xx, oo, **a)
                marks[5].record()
        else:
            ops = ep.CudaEpOps(shard.layer, rank, world, max_tokens=T, max_recv_rows=T_total * K)
            xch = ep.NcclExchange()
            launches = 12

            def step(i, x=None, o=None, marks=None, **extra):
                j = i % n_sets
                ep.ep_layer(ops, xch, xs[j] if x is None else x, out if o is None else o, topk_idx=idx_hist[j],
                            route_logits=rl_c[j], **kw, **extra)
        check = ops.check
    else:
        model = gtmoe.SynthModel(1, seed=0)
        blk = gtmoe.TokenBlock(T)
        weights_gb = model.weight_bytes() / 1e9
        resident = model.resident[0]
        layer = model.layers[0]
        phase_names = gtmoe.PHASE_NAMES

        def step(i, x=None, o=None, marks=None, **extra):
            j = i % n_sets
            a = dict(kw, **extra)
            if cfg == "prefill4096":
                a["route_logits"] = rl[j]
            if marks is not None:
                gtmoe.set_phase_events(marks)
            blk(layer, xs[j] if x is None else x, out if o is None else o, topk_idx=idx_hist[j], **a)
            if marks is not None:
                gtmoe.set_phase_events([])
        check = blk.check
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(warmup):
        step(i)
    check()
    barrier()
    # phase events for every timed step (recorded once first so their handles exist)
    marks = None
    if phase_names is not None:
        marks = [[torch.cuda.Event(enable_timing=True) for _ in range(len(phase_names) + 1)] for _ in range(steps)]
        for m in marks:
            for e in m:
                e.record(stream)
        torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for i in range(steps):
            step(i, marks=None if marks is None else marks[i])
        ev1.record(stream)
        clk.sample()
        torch.cuda.synchronize()
    check()
    ms = ev0.elapsed_time(ev1)
    phase_ms = None
    if marks is not None:
        phase_ms = [sum(m[p].elapsed_time(m[p + 1]) for m in marks) / steps for p in range(len(phase_names))]
    barrier()

    ms_e2e = None
    if with_e2e:
        # as a serving host runs it: every step's tokens go host -> device and its result device ->
        # host inside the timed region, on two copy streams with double buffers, so the copies of
        # steps i + 1 and i - 1 overlap the compute of step i
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

        run_e2e(warmup)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        run_e2e(steps)
        e1.record(stream)
        torch.cuda.synchronize()
        check()
        ms_e2e = e0.elapsed_time(e1)

    if dist is not None:
        vals = [ms, ms_e2e or 0.0] + (phase_ms or [])
        t = torch.tensor(vals, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), (float(t[1]) if with_e2e else None)
        if phase_ms:
            phase_ms = [float(v) for v in t[2:]]
    per_step_ms = ms / steps
    tokens_per_step = T_total if expert_parallel else T * world
    ids = idx_hist.cpu().numpy()
    distinct = float(np.mean([len(np.unique(ids[j])) for j in range(n_sets)]))
    r = {"value": tokens_per_step * steps / (ms / 1000.0), "ms_per_step": per_step_ms,
         "gpu_launches": steps * launches, "weights_gb_per_gpu": weights_gb}
    if phase_ms is not None:
        r["phase_ms"] = dict(zip(phase_names, phase_ms))
    if cfg == "batch64":
        act_bytes = T * D * 4 + T * D * 4
        alg = distinct * EXPERT_BYTES + SHARED_BYTES + ROUTER_BYTES + act_bytes
        achieved = alg / (per_step_ms / 1000.0) / 1e9
        peak, pk = peaks("hbm")
        r["roofline"] = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": pk, "traffic": None, "algorithmic_bytes_per_step": alg,
                         "scope": "whole layer call (views, routing, two grouped GEMMs, combine)",
                         "distinct_experts_per_step": distinct}
    else:
        flops = T_total * EXPERT_SHARED_FLOPS
        peak, pk = peaks("tensor")
        tr = profile_traffic("grouped_gemm_traffic.json")
        if not expert_parallel and phase_ms is not None:
            gemm_ms = r["phase_ms"]["gemm_gate_up"] + r["phase_ms"]["gemm_down"]
            achieved = flops / (gemm_ms / 1000.0) / 1e12
            r["roofline"] = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                             "frac": achieved / peak, "peak_source": pk,
                             "traffic": tr.get("bytes_per_step") if tr else None,
                             "flops_per_launch": flops, "kernel": "grouped_gemm<0> + grouped_gemm<1> (tcgen05)",
                             "kernel_ms": gemm_ms,
                             "whole_step_frac": flops / (per_step_ms / 1000.0) / 1e12 / peak,
                             "note": "useful FLOPs; the fp16 high/low activation split issues twice the tensor work"}
        else:
            achieved = flops / world / (per_step_ms / 1000.0) / 1e12
            r["roofline"] = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                             "frac": achieved / peak, "peak_source": pk, "traffic": None,
                             "flops_per_gpu_per_step": flops / world,
                             "scope": "whole per-GPU step (dispatch, barriers, experts, combine)"}
    r["clocks"] = clk.summary()
    if with_e2e:
        r["e2e"] = {"value": tokens_per_step * steps / (ms_e2e / 1000.0), "unit": "tokens/s",
                    "copies": "two copy streams, double buffers: the copies of steps i+1 and i-1 overlap step i",
                    "h2d_bytes_per_step": T * D * xs.element_size() * (1 if expert_parallel else world),
                    "d2h_bytes_per_step": T * D * 4 * (1 if expert_parallel else world)}

    if with_parity:
        # one step over token set 0 with every output, compared with the oracle on the host
        h1 = torch.empty(T, D, device="cuda")
        h2 = torch.empty(T, D, device="cuda")
        wts = torch.empty(T, K, device="cuda")
        step(0, None, out, h1=h1, h2=h2, topk_w=wts)
        torch.cuda.synchronize()
        check()
        o = resident.cpu().numpy()
        pes = o[layer.per_expert_scale:layer.per_expert_scale + 256].view(np.uint16)
        rl0 = None if rl_np is None else rl_np[0][rank * T:(rank + 1) * T]
        lb = kw["logit_bias"].cpu().numpy() if "logit_bias" in kw else None
        part = tokens_parity(xs[0].float().cpu().numpy(), idx_hist[0].cpu().numpy(), out.cpu().numpy(),
                             h1.cpu().numpy(), h2.cpu().numpy(), route_logits=rl0, logit_bias=lb, pes=pes,
                             sample=2 if expert_parallel else 6, token0=rank * T)
        if dist is not None:
            parts = [None] * world
            dist.all_gather_object(parts, part)
        else:
            parts = [part]
        r["parity"] = merge_parity(parts)

    if expert_parallel and ep_mode == "peer":
        torch.cuda.synchronize()
        barrier()
        ops.close()
        barrier()
    return r


def measure_batch_decode(rank: int, world: int, local: int, dist, seqs: int = 32, prompt_len: int = 1024,
                         new_tokens: int = 64, layers: int = LAYERS_DEFAULT):
    """Config 4: greedy decode of `seqs` sequences through the whole synthetic model; wall clock
    around the run (every generation step reads its tokens back, so the host waits on the device
    each step), split at the step that ends the prefill."""
    import numpy as np
    import torch
    import gtmoe
    from gtmoe import batch, ep
    S = seqs // world
    attn, embed, final = batch.synth_decoder(layers)
    if world == 1:
        model = gtmoe.SynthModel(layers, seed=0)
        moe = batch.LocalMoe(model.layers, S)
        ops = None
    else:
        shards = [ep.EpShardModel(l, rank, world) for l in range(layers)]
        ops = ep.PeerEpOps(shards[0].layer, rank, world, max_tokens=S)
        ops.connect()
        moe = batch.PeerEpMoe(ops, ep.NcclBarrier(), [sh.layer for sh in shards])
    bd = batch.BatchDecoder(attn, moe, embed, final, prompt_len + new_tokens + 1, S, dist=dist)
    prompts = np.random.default_rng(7).integers(0, embed["rows"], size=(seqs, prompt_len))
    mine = prompts[rank * S:(rank + 1) * S].tolist()
    stops = (1, 106, 50)
    bd.greedy([p[:3] for p in mine], 2, stops)   # warm-up
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    marks = {}

    def on_step(step):
        if step == prompt_len - 1:
            marks["prefill"] = time.perf_counter()
    with ClockSampler(local) as clk:
        t0 = time.perf_counter()
        out = bd.greedy(mine, new_tokens, stops, on_step=on_step)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        clk.sample()
    gen = sum(len(o) for o in out)
    vals = torch.tensor([t1 - t0, marks["prefill"] - t0, float(gen)], dtype=torch.float64, device="cuda")
    if dist is not None:
        mx = vals[:2].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        g = vals[2:].clone()
        dist.all_reduce(g)
        vals = torch.cat([mx, g])
    total_s, prefill_s, gen = float(vals[0]), float(vals[1]), int(vals[2])
    gen_s = total_s - prefill_s
    r = {"value": gen / gen_s, "ms_per_step": 1000.0 * gen_s / max(1, new_tokens - 1),
         "prefill_tokens_per_s": seqs * prompt_len / prefill_s, "prefill_s": prefill_s, "generate_s": gen_s,
         "generated_tokens": gen, "seq0_first_tokens": out[0][:8] if rank == 0 else None,
         "clocks": clk.summary(), "gpu_launches": None,
         "roofline": None}
    if ops is not None:
        torch.cuda.synchronize()
        dist.barrier()
        ops.close()
        dist.barrier()
    return r


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--layers", type=int, default=LAYERS_DEFAULT, help="decode stack depth (profiling only)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the other configs' lines at N = 1")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--workload", default="prefill4096", choices=list(WORKLOADS))
    ap.add_argument("--ep", default="peer", choices=["peer", "nccl"],
                    help="prefill4096 on N>1 GPUs: expert exchange over peer memory or NCCL all-to-all")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg = args.workload

    # CPU baseline first: worker processes are spawned before this process touches the GPU
    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and cfg != "decode_batch32":
        cb = decode_cpu_baseline(args.cpu_seconds, 1) if cfg == "decode30" else token_cpu_baseline(args.cpu_seconds,
                                                                                                   cfg)
    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))

    if cfg == "decode_batch32":
        m = measure_batch_decode(rank, world, local, dist)
        if rank == 0:
            line = {"metric": METRIC[cfg], "value": m["value"], "unit": UNIT[cfg], "n_gpus": world, "steps": 64,
                    "warmup": 1, "ms_per_step": m["ms_per_step"], "higher_is_better": True,
                    "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
                    "dtype": "f32 (fp16 hi/lo tensor-core operands in the MoE block)",
                    "data": "synthetic (random-init weights, random-id prompts)",
                    "config": bench_config(cfg, world, args.ep),
                    **{k: m[k] for k in ("prefill_tokens_per_s", "prefill_s", "generate_s", "generated_tokens",
                                         "seq0_first_tokens", "clocks")}}
            print(json.dumps(line), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return 0
    if cfg == "decode30":
        m = measure_decode(args.steps, args.warmup, args.layers, rank, local, dist)
    else:
        m = measure_tokens(cfg, args.steps, args.warmup, rank, world, local, dist, args.ep,
                           with_parity=not args.no_parity)
    extra = {}
    if world == 1 and not args.no_extra:
        # the other single-GPU configs, measured after the main line (not part of its timed region)
        others = [w for w in ("decode30", "batch64") if w != cfg]
        for w in others:
            if w == "decode30":
                d = measure_decode(min(args.steps, 50), args.warmup, LAYERS_DEFAULT, rank, local, None, with_e2e=False)
            else:
                d = measure_tokens(w, min(args.steps, 100), args.warmup, rank, world, local, None, args.ep,
                                   with_e2e=False, with_parity=False)
            extra[w] = {"metric": METRIC[w], "unit": UNIT[w], "config": bench_config(w, 1, args.ep),
                        **{k: d[k] for k in ("value", "ms_per_step", "roofline", "clocks", "phase_ms") if k in d}}
    if rank == 0:
        ep = cfg == "prefill4096" and world > 1
        line = {
            "metric": METRIC[cfg], "value": m["value"], "unit": UNIT[cfg], "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": m["ms_per_step"], "higher_is_better": True,
            "scaling": "strong" if ep else "weak", "vs_baseline": None,
            "dtype": "f32" if cfg == "decode30" else "f32 (fp16 hi/lo tensor-core operands)", "data": "synthetic",
            "config": bench_config(cfg, world, args.ep),
            "roofline": m["roofline"],
            "e2e": m.get("e2e"),
            "gpu_launches": m["gpu_launches"],
            "clocks": m["clocks"],
            "cpu_baseline": cb,
        }
        for k in ("parity", "phase_ms", "weights_gb", "weights_gb_per_gpu"):
            if k in m:
                line[k] = m[k]
        if extra:
            line["extra"] = extra
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

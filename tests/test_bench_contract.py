"""The reference arm of bench.py on the host (no GPU): `bench.py --impl reference` times the
reference's compiled CPU arithmetic (oracle/_ref when built, else the oracle port) and prints one
JSON line with the same metric, unit and config as the GPU arm. Under torchrun only rank 0 runs
and prints; the other ranks exit 0 without work. The multi-sequence decode (config 4) prints an
`unavailable` line instead, with its reason."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_bench(*args, env=None, timeout=300):
    e = dict(os.environ, **(env or {}))
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=e,
                       capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    return [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]


def test_reference_arm_batched_decode_is_unavailable_with_reason():
    lines = run_bench("--impl", "reference", "--workload", "decode_batch32", env={"RANK": "0", "WORLD_SIZE": "1"})
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference" and d["unavailable"]
    assert d["config"]["sequences"] == 32


def test_reference_arm_other_ranks_print_nothing():
    assert run_bench("--impl", "reference", env={"RANK": "1", "WORLD_SIZE": "2"}) == []


def test_reference_arm_line_batch64():
    """A bounded run (10 steps of 2 s): one line with the GPU arm's metric and config, a CPU
    baseline describing the run, and an e2e block with no host-device copies."""
    lines = run_bench("--impl", "reference", "--workload", "batch64", "--steps", "10", "--warmup", "0",
                      env={"RANK": "0", "WORLD_SIZE": "1"})
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["tokens_per_step"] == 64 and d["config"]["parallelism"] == "single"
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("reference", "port") and cb["cores"] >= 1
    assert "batch64" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}

"""Expert parallelism on 2..8 GPUs of one box (skipped with fewer than 2 GPUs), over NCCL
all-to-all and over peer memory: tests/ep_torchrun_main.py under torch.distributed.run, one
process per GPU."""
import os
import socket
import subprocess
import sys

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2+ GPUs")
@pytest.mark.parametrize("mode", ["nccl", "peer"])
def test_ep_all_gpus_bit_identical_to_single_gpu(mode):
    n = min(torch.cuda.device_count(), 8)
    while 128 % n:
        n -= 1
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(ROOT, "tests", "ep_torchrun_main.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE=os.environ.get("NCCL_NVLS_ENABLE", "1"), EP_MODE=mode)
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "bit-identical to one GPU: True" in r.stdout

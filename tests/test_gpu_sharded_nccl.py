"""Row-sharded pair block over a real NCCL process group (one process per
GPU, launched with torchrun on 127.0.0.1), checked against the CPU oracle at
the strict (1e-4) and fast (1e-2) tolerances. Skips with fewer than two
visible GPUs; single-GPU runs cover the phase kernels through
``test_gpu_sharded.py``."""
import json
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

WORKER = Path(__file__).resolve().parent / "sharded_nccl_worker.py"


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_block_nccl(cuda_device, tmp_path):
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    out = tmp_path / "verdict.json"
    cmd = ["timeout", "-k", "60", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr=127.0.0.1",
           f"--master-port={_free_port()}", str(WORKER), str(out)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr[-4000:]
    verdict = json.loads(out.read_text())
    assert verdict["world"] == world
    assert verdict["cases"], verdict
    for name, case in verdict["cases"].items():
        assert case["ok"], (name, case)

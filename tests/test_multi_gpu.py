"""The sharded paths on two GPUs: tests/multi_gpu_worker.py run as two ranks
(one process per GPU, NCCL over NVLink) by torch.distributed.run.  Skipped
when fewer than two GPUs are visible."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _gpus() -> int:
    import torch
    return torch.cuda.device_count()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_paths_match_the_whole_on_two_gpus():
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "tests" / "multi_gpu_worker.py")]
    env = dict(os.environ, CUDA_DEVICE_MAX_CONNECTIONS="8")
    run = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    lines = [l for l in run.stdout.splitlines() if l.startswith("{")]
    assert lines, f"no report (exit {run.returncode}):\n{run.stdout[-2000:]}\n{run.stderr[-4000:]}"
    report = json.loads(lines[-1])
    assert report["failures"] == [], report["failures"]
    assert run.returncode == 0, run.stderr[-4000:]

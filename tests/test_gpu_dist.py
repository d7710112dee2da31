"""Row-sharded multi-GPU path on 2 GPUs: per-rank partials, the CUDA
device's NCCL all-gather and the rank-order combine, checked against the same
computation done whole on one GPU (and max/argmax against the CPU oracle).
Runs tests/_dist_worker.py as two processes under torch.distributed.run;
skipped when the machine has fewer than two GPUs."""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def gpu_count() -> int:
    try:
        out = subprocess.run(["nvidia-smi", "-L"], capture_output=True, text=True, timeout=30).stdout
        return sum(1 for line in out.splitlines() if line.startswith("GPU "))
    except Exception:
        return 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(gpu_count() < 2, reason="needs two GPUs")
def test_two_rank_sharded_reductions_match_one_gpu():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=str(ROOT))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", str(ROOT / "tests" / "_dist_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    lines = [line for line in res.stdout.splitlines() if line.startswith("{")]
    assert lines, res.stdout[-3000:] + res.stderr[-3000:]
    report = json.loads(lines[-1])
    failed = [k for k, v in report["checks"].items() if not v]
    assert not failed, report

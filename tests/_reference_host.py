"""Shared driver for the reference built with its `cuda` device
(oracle/_ref/cuda_host, oracle/Makefile `host`).

The module is the reference's own pybind11 `vectorcore` with the patch in
vectorcore_b200/csrc/host/reference_cuda_device.patch applied; it and the
device-slot build cannot be imported into one process (pybind11 registers
the same C++ types), so every run here is a child process."""
import os
import re
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
HOST_DIR = ROOT / "oracle" / "_ref" / "cuda_host"
SUITES = HOST_DIR / "tree" / "tests" / "python"
CHECKS = Path(__file__).resolve().parent / "reference_host" / "cuda_device_checks.py"


def built() -> bool:
    return any(HOST_DIR.glob("vectorcore*.so")) and SUITES.is_dir()


def run_pytest(*targets, extra=(), timeout=1200):
    """pytest in a child process with the cuda-device build on its path."""
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(HOST_DIR), str(Path(__file__).resolve().parent),
                                         env.get("PYTHONPATH", "")])
    cmd = [sys.executable, "-m", "pytest", "-q", "-rA", "-p", "no:cacheprovider", *map(str, targets), *extra]
    res = subprocess.run(cmd, env=env, cwd=str(ROOT), capture_output=True, text=True, timeout=timeout)
    return res.returncode, res.stdout + res.stderr


def passed_ids(output):
    return re.findall(r"^PASSED (\S+)", output, flags=re.M)


def cuda_cases(ids):
    """Test ids whose parameters (the part after the last '::') name cuda."""
    return [i for i in ids if "cuda" in i.rsplit("::", 1)[-1]]


def counts(output):
    tail = output.strip().splitlines()[-1] if output.strip() else ""
    got = {k: int(v) for v, k in re.findall(r"(\d+) (passed|failed|skipped|error|errors)", tail)}
    return got

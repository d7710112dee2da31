"""bench.py's host-side plumbing on CPU: the block-wise generators give every
shard layout the same global tensor (strong scaling compares like with
like), and the reference arm -- the reference's own CPU path -- prints one
well-formed JSON line (run here on a shrunk sample)."""
import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from vectorcore_b200.dist import RowShard  # noqa: E402


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_block_rows_are_the_same_global_tensor_for_every_shard_layout(world):
    rows, cols = 2500, 48  # rows not a multiple of the 1024-row generator block
    whole = bench.uniform_rows(2, 0.1, 2.0, 0, rows, cols)
    parts = [bench.uniform_rows(2, 0.1, 2.0, s.start, s.stop, cols)
             for s in (RowShard(rows, world, r) for r in range(world))]
    assert np.array_equal(np.concatenate(parts), whole)
    assert whole.dtype == np.float32 and whole.min() >= 0.1 and whole.max() <= 2.0
    normal = bench.normal_rows(4, 1.0, 1000, 1100, cols)
    assert np.array_equal(normal, bench.normal_rows(4, 1.0, 0, rows, cols)[1000:1100])


@pytest.mark.skipif(not any((ROOT / "oracle" / "_ref").glob("vectorcore*.so")),
                    reason="the reference's CPU build is absent (make -C oracle ref)")
def test_reference_arm_prints_one_json_line():
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--rows", "128",
                          "--steps", "1", "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [line for line in res.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1, res.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["value"] > 0
    assert d["higher_is_better"] is True and d["metric"].startswith("effective HBM GB/s (config 2")
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


class _Done:
    def __init__(self, returncode, stdout, stderr=""):
        self.returncode, self.stdout, self.stderr = returncode, stdout, stderr


def test_per_configuration_child_command_and_its_json_line(monkeypatch):
    """The default run times each extra configuration in a child process
    (`bench.py --config-only cfgN`) and takes the child's last JSON line; a
    child that fails is reported with its configuration's name."""
    import argparse

    seen = {}

    def fake_run(cmd, **kw):
        seen["cmd"], seen["env"] = cmd, kw.get("env", {})
        return _Done(0, 'log line\n{"value": 1.5, "per_op": {}}\n')

    monkeypatch.setenv("RANK", "0")
    monkeypatch.setattr(bench.subprocess, "run", fake_run)
    got = bench.config_in_child("cfg4", argparse.Namespace(steps=20))
    assert got == {"value": 1.5, "per_op": {}}
    assert seen["cmd"][1:] == [str(ROOT / "bench.py"), "--config-only", "cfg4", "--steps", "20"]
    assert "RANK" not in seen["env"]  # the child is a one-GPU process of its own

    monkeypatch.setattr(bench.subprocess, "run", lambda cmd, **kw: _Done(3, "", "CUDA error"))
    with pytest.raises(RuntimeError, match="cfg4.*exit 3"):
        bench.config_in_child("cfg4", argparse.Namespace(steps=5))

"""The reference built with its `cuda` device, on a machine without a GPU.

oracle/Makefile `host` applies vectorcore_b200/csrc/host/
reference_cuda_device.patch to a copy of the reference and links it to the
CUDA library. Without a GPU the `cuda` device reports itself unavailable
(creating a cuda tensor raises the reference's RuntimeError, as an absent
Metal does) and everything else is the reference unchanged: its own Python
suites pass exactly as on the stock build (cpu only; Metal-only tests
skipped)."""
import pytest

import _reference_host as H
from conftest import has_nvidia_device

pytestmark = pytest.mark.skipif(not H.built(), reason="cuda-device build of the reference absent (make -C oracle host)")


@pytest.mark.skipif(has_nvidia_device(), reason="checks the behaviour without a GPU")
def test_reference_suites_pass_unchanged_without_a_gpu():
    rc, out = H.run_pytest(H.SUITES)
    assert rc == 0, out[-4000:]
    assert not H.cuda_cases(H.passed_ids(out)), "cuda cases ran without a GPU"
    assert H.counts(out).get("passed", 0) >= 127, out[-2000:]


@pytest.mark.skipif(has_nvidia_device(), reason="checks the behaviour without a GPU")
def test_cuda_device_reports_unavailable():
    rc, out = H.run_pytest(H.CHECKS)  # every check skips: no CUDA device
    assert rc == 0, out[-3000:]
    code = ("import vectorcore as vc\n"
            "assert not vc.cuda_available()\n"
            "try:\n    vc.Tensor([1.0], device='cuda')\nexcept RuntimeError as e:\n"
            "    assert 'CUDA is unavailable' in str(e), e\nelse:\n    raise SystemExit('no error')\n"
            "vc.synchronize()\nprint('ok')\n")
    import os
    import subprocess
    import sys

    env = dict(os.environ, PYTHONPATH=str(H.HOST_DIR))
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert res.returncode == 0 and "ok" in res.stdout, res.stdout + res.stderr

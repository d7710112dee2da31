"""The reference's OWN Python suites on its new `cuda` device.

oracle/_ref/cuda_host is the reference with the CUDA device added next to
CPU and Metal (vectorcore_b200/csrc/host/reference_cuda_device.patch,
oracle/Makefile `host`): DeviceType::CUDA, "cuda" in parse_device,
cuda_available(), and a cuda branch at every dispatch site calling
CudaBackend over the C ABI, with the fused kernels behind sum_to_shape,
broadcast_to, the mul/div/relu/sigmoid gradients, max, log_softmax/softmax
and cross_entropy. With `cuda` in their DEVICES lists, the reference's
tests/python suites (test_classifier_ops.py, test_performance_paths.py,
test_autograd_correctness.py, test_vectorcore.py) run every device-
parametrised case on the B200 against their own numpy / PyTorch / finite-
difference references. tests/reference_host/cuda_device_checks.py adds the
CUDA versions of the reference's Metal-only checks and compares the fused
paths with the CPU device of the same module."""
import pytest

import _reference_host as H

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not H.built(), reason="cuda-device build of the reference absent")]


def test_reference_suites_on_the_cuda_device():
    rc, out = H.run_pytest(H.SUITES)
    assert rc == 0, out[-6000:]
    cuda_cases = H.cuda_cases(H.passed_ids(out))
    # every device-parametrised case of the three suites ran on cuda too
    assert len(cuda_cases) >= 40, (len(cuda_cases), out[-3000:])
    print(f"{len(cuda_cases)} cuda cases of the reference's suites passed; {H.counts(out)}")


def test_cuda_device_checks():
    rc, out = H.run_pytest(H.CHECKS)
    assert rc == 0, out[-6000:]
    c = H.counts(out)
    assert c.get("passed", 0) >= 20 and not c.get("skipped"), c

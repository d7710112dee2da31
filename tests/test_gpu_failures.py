"""Failure detection on the device, without faulting it.

The reference surfaces asynchronous device errors at the next sync and stays
usable (src/metal/metal_backend.mm:428-443, completion handlers :545-549).
The CUDA device does the same through its device error word:

* a bounded wait that runs out -- a kernel waits on an mbarrier that nothing
  completes, with the bounded wait every pipelined kernel uses cut to a few
  hundred polls (vc_cuda_selftest_wait_timeout) -- gives up, the next
  blocking call fails with VC_ERR_TIMEOUT (DeviceTimeout, a RuntimeError),
  and the device keeps working;
* an allocation failure injected on the host (VC_CUDA_FAKE_OOM, checked on a
  pool miss before cudaMalloc) comes back as VC_ERR_OOM (DeviceOutOfMemory)
  and the pool keeps working once it is lifted.

No test here traps, faults or hangs the GPU: every wait is bounded and the
failures are made on the host or by a flag that nothing sets."""
import os
import time

import numpy as np
import pytest

from vectorcore_b200 import _abi
from vectorcore_b200 import backend as B

pytestmark = pytest.mark.gpu


def _still_usable(be):
    x = np.arange(1000, dtype=np.float32)
    got = be.download(be.binary_scalar(be.upload(x), x.size, 2.0, B.MUL))
    np.testing.assert_array_equal(got, x * 2)


def test_bounded_wait_gives_up_and_the_device_stays_usable(backend):
    backend.synchronize()
    t0 = time.monotonic()
    _abi.call("vc_cuda_selftest_wait_timeout", 500)  # <= 500 polls of <= 2 us
    with pytest.raises(_abi.DeviceTimeout, match="bounded device-side wait timed out"):
        backend.synchronize()
    assert time.monotonic() - t0 < 10.0
    backend.synchronize()  # the error was reported once and cleared
    _still_usable(backend)


def test_timeout_is_reported_by_a_download_too(backend):
    x = backend.upload(np.ones(8, np.float32))
    _abi.call("vc_cuda_selftest_wait_timeout", 200)
    with pytest.raises(RuntimeError, match="timed out"):
        backend.download(x)
    np.testing.assert_array_equal(backend.download(x), np.ones(8, np.float32))


def test_selftest_rejects_bad_poll_counts(backend):
    with pytest.raises(IndexError):
        _abi.call("vc_cuda_selftest_wait_timeout", 0)
    with pytest.raises(IndexError):
        _abi.call("vc_cuda_selftest_wait_timeout", (1 << 21) + 1)


def test_injected_allocation_failure_and_recovery(backend):
    backend.synchronize()
    _abi.call("vc_cuda_pool_trim")  # nothing cached: the next allocation is a pool miss
    misses = _abi.pool_stats()["misses"]
    os.environ["VC_CUDA_FAKE_OOM"] = "1"
    try:
        with pytest.raises(_abi.DeviceOutOfMemory, match="VC_CUDA_FAKE_OOM"):
            backend.allocate(3_000_001)
        with pytest.raises(RuntimeError):  # DeviceOutOfMemory derives from RuntimeError
            backend.upload(np.zeros(5_000_003, np.float32))
    finally:
        del os.environ["VC_CUDA_FAKE_OOM"]
    assert _abi.pool_stats()["misses"] > misses
    s = backend.allocate(3_000_001)
    assert s.ptr
    _still_usable(backend)

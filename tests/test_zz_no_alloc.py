"""The allocation-free sum (vc_cuda_reduce_sum_noalloc) against the reference's
sum (the CPU oracle) and the regular entry point (vc_cuda_reduce_all).

Some callers of this library cannot allocate device memory at arbitrary
points: a host that reserved the device's memory up front under a hard
budget, or a loop that must not stall on cudaMalloc / cudaFree. For them the
allocation-free entry point keeps its scratch in an array compiled into the
library instead of taking it from the device pool. These tests call it
through the C ABI twice in a row, on different data, and check each result
against the oracle and against the regular entry point within the sum
tolerance the other tests use (_util.assert_sum_close); that the device
pool's counters do not move across the calls (it allocates nothing); the
edge cases (an empty input, an input that is not 16-byte aligned, exactly
the maximum count, one past it); and a call from a second host thread. The
file name makes pytest collect it last; it passes on its own in a fresh
process too (it initialises the device itself)."""
import ctypes
import threading

import numpy as np
import pytest

from _util import assert_sum_close

pytestmark = pytest.mark.gpu

MAX_COUNT = 1 << 28


def _noalloc(abi, ptr, n, out_ptr):
    abi.call("vc_cuda_reduce_sum_noalloc", ctypes.c_void_p(ptr), ctypes.c_size_t(n), ctypes.c_void_p(out_ptr))


def _pool_counters(abi):
    cached, in_use, hits, misses = (ctypes.c_size_t() for _ in range(4))
    abi.call("vc_cuda_pool_stats", ctypes.byref(cached), ctypes.byref(in_use), ctypes.byref(hits),
             ctypes.byref(misses))
    return cached.value, in_use.value, hits.value, misses.value


@pytest.fixture(scope="module")
def lib():
    from vectorcore_b200 import _abi
    from vectorcore_b200.backend import CudaBackend

    _abi.check(_abi.lib.vc_cuda_init(0))  # the entry point needs the device's stream to exist
    return _abi, CudaBackend.instance()


def test_noalloc_sum_matches_the_oracle_and_the_pool_sum_on_two_calls_in_a_row(lib, port):
    abi, be = lib
    rng = np.random.default_rng(2024)
    cases = []
    for n in (3_000_001, (1 << 20) + 7):
        x = rng.normal(size=n).astype(np.float32)
        dx = be.upload(x)
        ref = be.download(be.reduce_sum(dx, n))[0]
        cases.append((n, x, dx, ref, be.allocate(1)))
    be.synchronize()
    before = _pool_counters(abi)
    for n, x, dx, ref, out in cases:  # two calls in a row, nothing allocated in between
        _noalloc(abi, dx.ptr, n, out.ptr)
    be.synchronize()
    after = _pool_counters(abi)
    assert after == before, f"pool counters moved across the calls: {before} -> {after}"
    for n, x, dx, ref, out in cases:
        got = be.download(out)[0]
        assert_sum_close(got, port.sum(x), n, 1.0, what=f"allocation-free sum of {n} vs the oracle")
        assert_sum_close(got, ref, n, 1.0, what=f"allocation-free sum of {n} vs vc_cuda_reduce_all")


def test_noalloc_sum_empty_and_unaligned_inputs(lib, port):
    abi, be = lib
    x = np.random.default_rng(7).uniform(-1, 1, 70_001).astype(np.float32)
    dx = be.upload(x)
    out = be.upload(np.full(1, 123.0, np.float32))
    _noalloc(abi, dx.ptr, 0, out.ptr)  # empty input: +0, like cpu::sum of nothing
    assert be.download(out)[0] == 0.0
    # one float past a 256-byte aligned block: the kernel's scalar path
    _noalloc(abi, dx.ptr + 4, x.size - 1, out.ptr)
    assert_sum_close(be.download(out)[0], port.sum(x[1:]), x.size - 1, 1.0, what="unaligned input")


def test_noalloc_sum_at_its_maximum_count_and_beyond(lib):
    abi, be = lib
    ones = be.fill(MAX_COUNT, 1.0)  # 1 GiB of 1.0: the exact sum is 2^28
    out = be.allocate(1)
    _noalloc(abi, ones.ptr, MAX_COUNT, out.ptr)
    assert be.download(out)[0] == float(MAX_COUNT)
    # rejected on the host before anything is launched
    with pytest.raises(OverflowError, match="maximum"):
        _noalloc(abi, ones.ptr, MAX_COUNT + 1, out.ptr)
    _noalloc(abi, ones.ptr, 4, out.ptr)
    assert be.download(out)[0] == 4.0


def test_noalloc_sum_from_a_second_host_thread(lib, port):
    # A host thread that never called into the library: the call binds it to
    # the library's GPU before it launches.
    abi, be = lib
    x = np.random.default_rng(11).normal(size=1_000_003).astype(np.float32)
    dx = be.upload(x)
    out = be.allocate(1)
    be.synchronize()
    errors = []

    def worker():
        try:
            _noalloc(abi, dx.ptr, x.size, out.ptr)
        except Exception as exc:  # reported on the main thread
            errors.append(exc)

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert not errors, errors
    assert_sum_close(be.download(out)[0], port.sum(x), x.size, 1.0, what="sum from a second thread")

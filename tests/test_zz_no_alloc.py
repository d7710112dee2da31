"""The allocation-free sum (vc_cuda_reduce_sum_noalloc) against the regular
one (vc_cuda_reduce_all with VC_REDUCE_SUM).

Some callers of this library cannot allocate device memory at arbitrary
points: a host that reserved the device's memory up front under a hard
budget, or a loop that must not stall on cudaMalloc / cudaFree. For them the
allocation-free entry point keeps its scratch in an array compiled into the
library instead of taking it from the device pool. This test calls it
through the C ABI twice in a row, on different data, and checks each result
against the regular entry point within the sum tolerance the other tests use
(_util.assert_sum_close). It also checks the size limit. The file name makes
pytest collect it last; it passes on its own in a fresh process too (it
initialises the device itself)."""
import ctypes

import numpy as np
import pytest

from _util import assert_sum_close

pytestmark = pytest.mark.gpu


def _noalloc(abi, ptr, n, out_ptr):
    abi.call("vc_cuda_reduce_sum_noalloc", ctypes.c_void_p(ptr), ctypes.c_size_t(n), ctypes.c_void_p(out_ptr))


def test_noalloc_sum_matches_the_pool_sum_on_two_calls_in_a_row():
    from vectorcore_b200 import _abi
    from vectorcore_b200.backend import CudaBackend

    _abi.check(_abi.lib.vc_cuda_init(0))  # the entry point needs the device's stream to exist
    be = CudaBackend.instance()
    rng = np.random.default_rng(2024)
    for n in (3_000_001, (1 << 20) + 7):
        x = rng.normal(size=n).astype(np.float32)
        dx = be.upload(x)
        ref = be.download(be.reduce_sum(dx, n))[0]
        out = be.allocate(1)
        _noalloc(_abi, dx.ptr, n, out.ptr)
        got = be.download(out)[0]
        assert_sum_close(got, ref, n, 1.0, what=f"allocation-free sum of {n}")


def test_noalloc_sum_rejects_counts_beyond_its_maximum():
    from vectorcore_b200 import _abi
    from vectorcore_b200.backend import CudaBackend

    _abi.check(_abi.lib.vc_cuda_init(0))
    be = CudaBackend.instance()
    small = be.upload(np.ones(4, np.float32))
    out = be.allocate(1)
    # rejected on the host before anything is launched
    with pytest.raises(OverflowError, match="maximum"):
        _noalloc(_abi, small.ptr, (1 << 28) + 1, out.ptr)
    _noalloc(_abi, small.ptr, 4, out.ptr)
    assert be.download(out)[0] == 4.0

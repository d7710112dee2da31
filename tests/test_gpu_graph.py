"""GPU: CUDA graph capture and replay of the library stream (vc_cuda_graph_*),
with the graph-owned pool blocks that keep replays from writing into memory
the pool has handed to someone else."""
import ctypes

import numpy as np
import pytest

from _util import assert_bitexact, assert_sum_close
from vectorcore_b200 import _abi
from vectorcore_b200 import backend as B

pytestmark = pytest.mark.gpu


def test_replays_match_eager_and_follow_new_inputs(backend):
    rows, cols = 300, 1028
    rng = np.random.default_rng(1)
    x_np = rng.uniform(-1, 1, (rows, cols)).astype(np.float32)
    b_np = rng.normal(size=cols).astype(np.float32)
    x, b = backend.upload(x_np), backend.upload(b_np)
    one = backend.upload(np.ones(1, np.float32))
    eager_loss = backend.download(backend.bias_relu_sum(x, b, rows, cols))[0]
    eager_dx, eager_db = backend.bias_relu_sum_backward(x, b, one, rows, cols)

    def step():
        loss = backend.bias_relu_sum(x, b, rows, cols)
        dx, db = backend.bias_relu_sum_backward(x, b, one, rows, cols)
        return loss, dx, db

    graph, (loss, dx, db) = backend.capture(step)
    try:
        assert graph.nodes >= 2
        for _ in range(3):
            graph.launch()
            backend.synchronize()
            assert backend.download(loss)[0] == eager_loss
            assert_bitexact(backend.download(dx), backend.download(eager_dx), "dx")
            assert_bitexact(backend.download(db), backend.download(eager_db), "db")
        # replays read the current contents of the captured inputs
        x2_np = -x_np
        _abi.call("vc_cuda_upload", ctypes.c_void_p(x.ptr), x2_np.ctypes.data_as(ctypes.c_void_p),
                  ctypes.c_size_t(x2_np.nbytes))
        graph.launch()
        backend.synchronize()
        ref = np.maximum(x2_np + b_np, 0).astype(np.float64).sum()
        assert_sum_close(backend.download(loss)[0], ref, x2_np.size, 1.0)
    finally:
        graph.close()


def test_captured_blocks_stay_reserved_until_the_graph_is_destroyed(backend):
    n = 1 << 16
    src = backend.upload(np.arange(n, dtype=np.float32))

    def step():
        return backend.unary(src, n, B.NEG)

    graph, out = backend.capture(step)
    try:
        out_ptr = out.ptr
        del out  # the captured output's block goes back -- to the graph, not the pool
        fresh = [backend.upload(np.full(n, 7.0, np.float32)) for _ in range(4)]
        assert all(f.ptr != out_ptr for f in fresh)
        for _ in range(2):
            graph.launch()
        backend.synchronize()
        for f in fresh:
            assert np.all(backend.download(f) == 7.0)  # no replay wrote into them
    finally:
        graph.close()
    # after destroy the block is back in the pool and reusable
    again = [backend.allocate(n) for _ in range(8)]
    assert any(a.ptr == out_ptr for a in again)


def test_a_capture_that_synchronises_fails_cleanly(backend):
    x = backend.upload(np.ones(1024, np.float32))

    def step():
        y = backend.unary(x, 1024, B.NEG)
        backend.synchronize()  # not capturable
        return y

    with pytest.raises(RuntimeError):
        backend.capture(step)
    # no capture is left open and the device still works
    y = backend.unary(x, 1024, B.NEG)
    assert np.all(backend.download(y) == -1.0)
    graph, z = backend.capture(lambda: backend.unary(x, 1024, B.EXP))
    graph.launch()
    backend.synchronize()
    assert np.allclose(backend.download(z), np.e)
    graph.close()

"""GPU: asynchronous host <-> device transfers (vc_cuda_upload_async,
vc_cuda_download_async, vc_cuda_transfer_wait / _sync).

These entry points have no counterpart in the reference (its upload and
download are synchronous); the tests pin their ordering contract: a copy runs
after the work enqueued before it, later work waits only after
transfer_wait, and a freed device buffer is not reused under a transfer."""
import numpy as np
import pytest

from vectorcore_b200 import backend as B

pytestmark = pytest.mark.gpu


def test_round_trip_through_compute(backend):
    n = 1 << 22
    src = B.PinnedBuffer(n)
    src.array[:] = np.random.default_rng(1).uniform(-2, 2, n).astype(np.float32)
    dst = B.PinnedBuffer(n)
    dev = backend.allocate(n)
    t_up = backend.upload_async(dev, src)
    backend.transfer_wait(t_up)
    out = backend.unary(dev, n, B.NEG)
    t_down = backend.download_async(dst, out)
    backend.transfer_sync(t_down)
    assert np.array_equal(dst.array, -src.array)


def test_upload_overlaps_but_orders_after_earlier_work(backend):
    """An upload into a buffer that enqueued work still reads starts after
    that work: the earlier op sees the old contents."""
    n = 1 << 22
    old = np.full(n, 3.0, np.float32)
    dev = backend.upload(old)
    before = backend.unary(dev, n, B.NEG)  # enqueued before the upload
    src = B.PinnedBuffer(n)
    src.array[:] = 7.0
    t = backend.upload_async(dev, src)
    backend.transfer_wait(t)
    after = backend.unary(dev, n, B.NEG)
    assert np.all(backend.download(before) == -3.0)
    assert np.all(backend.download(after) == -7.0)


def test_freed_buffer_not_reused_under_a_download(backend):
    n = 1 << 24
    values = np.random.default_rng(2).uniform(-1, 1, n).astype(np.float32)
    dev = backend.upload(values)
    dst = B.PinnedBuffer(n)
    t = backend.download_async(dst, dev)
    del dev  # back to the pool while the copy may still run
    other = backend.fill(n, 5.0)  # same size class: may reuse the freed block
    backend.transfer_sync(t)
    assert np.array_equal(dst.array, values)
    assert np.all(backend.download(other) == 5.0)


def test_synchronize_waits_for_transfers(backend):
    n = 1 << 22
    src = B.PinnedBuffer(n)
    src.array[:] = 1.5
    dev = backend.allocate(n)
    backend.upload_async(dev, src)
    backend.synchronize()
    dst = B.PinnedBuffer(n)
    backend.download_async(dst, dev)
    backend.synchronize()
    assert np.all(dst.array == 1.5)


def test_many_tickets_retire(backend):
    src = B.PinnedBuffer(256)
    src.array[:] = np.arange(256, dtype=np.float32)
    dev = backend.allocate(256)
    first = backend.upload_async(dev, src)
    last = first
    for _ in range(1100):  # more than the ticket ring holds
        last = backend.upload_async(dev, src)
    backend.transfer_wait(first)  # retired: already complete
    backend.transfer_sync(first)
    backend.transfer_sync(last)
    assert np.array_equal(backend.download(dev), src.array)


def test_pageable_memory_and_bad_tickets_are_rejected(backend):
    import ctypes

    from vectorcore_b200 import _abi

    dev = backend.allocate(16)
    host = np.zeros(16, np.float32)  # pageable
    t = ctypes.c_uint64(0)
    with pytest.raises(ValueError, match="page-locked"):
        _abi.call("vc_cuda_upload_async", ctypes.c_void_p(dev.ptr), host.ctypes.data_as(ctypes.c_void_p),
                  ctypes.c_size_t(host.nbytes), ctypes.byref(t))
    with pytest.raises(ValueError, match="ticket"):
        backend.transfer_wait(0)
    with pytest.raises(ValueError, match="ticket"):
        backend.transfer_sync(1 << 60)


def test_not_allowed_during_capture(backend):
    dev = backend.allocate(16)
    src = B.PinnedBuffer(16)

    def body():
        backend.upload_async(dev, src)

    with pytest.raises(ValueError, match="graph"):
        backend.capture(body)
    backend.synchronize()


@pytest.mark.parametrize("elements", [(8 << 20) // 4, (100 << 20) // 4 + 3, (64 << 20) // 4])
def test_pageable_copies_through_staging(backend, elements):
    """Pageable uploads / downloads of 8 MiB and more go through the
    page-locked staging pieces (32 MiB): sizes on and off the piece grid."""
    values = np.random.default_rng(elements % 97).uniform(-1, 1, elements).astype(np.float32)
    dev = backend.upload(values)  # pageable numpy source
    neg = backend.unary(dev, elements, B.NEG)
    back = backend.download(neg)  # pageable numpy destination
    assert np.array_equal(back, -values)
    # the source may be reused as soon as upload returns
    values[:] = 0.0
    assert np.array_equal(backend.download(dev), -back)


def test_tensor_to_round_trip_large(backend):
    import pytensor as vc

    x = np.random.default_rng(5).normal(size=(3000, 7001)).astype(np.float32)
    t = vc.Tensor(x, requires_grad=True)
    c = t.to("cuda")
    assert c.device == "cuda"
    h = (c * 2.0).to("cpu")
    assert h.device == "cpu"
    assert np.array_equal(h.numpy(), x * 2.0)
    (c * 2.0).sum().backward()  # the gradient flows back through to()
    assert t.grad.device == "cpu"
    assert np.all(t.grad.numpy() == 2.0)

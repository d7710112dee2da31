"""GPU parity: full and per-axis reductions and their backward passes through
the C ABI, against the CPU oracle and the reference's golden vectors.

max / argmax and every backward pass (broadcast, scatter) are bit-exact.
Sums and means are double-accumulated on both sides and rounded once; they
must stay within the SUM_RTOL class (and in practice agree bit for bit --
the tests record how many do)."""
import numpy as np
import pytest

import _cases as C
import oracle
from _util import assert_bitexact, assert_sum_close, sha256
from vectorcore_b200 import backend as B

pytestmark = pytest.mark.gpu


def dev(be, a):
    return be.upload(np.ascontiguousarray(a, np.float32))


def split(shape, axis):
    ax = axis % len(shape)
    return (int(np.prod(shape[:ax], dtype=np.int64)), int(shape[ax]),
            int(np.prod(shape[ax + 1:], dtype=np.int64)))


@pytest.mark.parametrize("n", [1, 3, 127, 1024, 65535, 65536, 65537, 3_000_001, (1 << 24) + 7, 1 << 26])
def test_reduce_all(backend, port, n):
    # past 2^24 elements the full reductions take >= 1024 segments of 16384
    # and finish with 1024 threads per output
    x = np.random.default_rng(n).normal(size=n).astype(np.float32)
    dx = dev(backend, x)
    got = backend.download(backend.reduce_sum(dx, n))[0]
    assert_sum_close(got, port.sum(x), n, 1.0, what="sum")
    mean = backend.download(backend.reduce_all(dx, n, B.REDUCE_MEAN))[0]
    assert_sum_close(mean, port.reduce_op("mean", x, None)[0], n, 1.0 / n, what="mean")
    v, i = backend.reduce_all(dx, n, B.REDUCE_MAX, want_index=True)
    ref_i = port.argmax_i64(x, 1, n, 1)
    assert_bitexact(backend.download(v), port.reduce_op("max", x, None)[0].reshape(1))
    assert backend.download(i)[0] == ref_i[0]
    af = backend.reduce_all(dx, n, B.REDUCE_ARGMAX)
    assert backend.download(af)[0] == np.float32(ref_i[0])


def test_sum_is_deterministic(backend):
    x = np.random.default_rng(4).normal(size=3_000_001).astype(np.float32)
    dx = dev(backend, x)
    values = {backend.download(backend.reduce_sum(dx, x.size))[0].tobytes() for _ in range(5)}
    assert len(values) == 1


SHAPES = [(3, 4, 5), (64, 500, 33), (64, 512), (1, 70000), (70000, 1), (5, 1, 7), (2, 131072), (4, 3, 65537)]


@pytest.mark.parametrize("shape", SHAPES)
def test_reduce_axis(backend, port, shape):
    x = np.random.default_rng(len(shape) + shape[0]).normal(size=shape).astype(np.float32)
    dx = dev(backend, x)
    for axis in range(len(shape)):
        outer, length, inner = split(shape, axis)
        s = backend.download(backend.reduce_axis(dx, outer, length, inner, B.REDUCE_SUM))
        assert_sum_close(s, port.reduce_axis(oracle.SUM, x, outer, length, inner), length, 1.0)
        m = backend.download(backend.reduce_axis(dx, outer, length, inner, B.REDUCE_MEAN))
        assert_sum_close(m, port.reduce_op("mean", x, axis)[0].reshape(-1), length, 1.0 / length)
        v, i = backend.reduce_axis(dx, outer, length, inner, B.REDUCE_MAX, want_index=True)
        assert_bitexact(backend.download(v), port.reduce_axis(oracle.MAX, x, outer, length, inner))
        assert np.array_equal(backend.download(i), port.argmax_i64(x, outer, length, inner))
        af = backend.reduce_axis(dx, outer, length, inner, B.REDUCE_ARGMAX)
        assert_bitexact(backend.download(af), port.reduce_axis(oracle.ARGMAX, x, outer, length, inner))


def test_max_argmax_scan_semantics(backend, port):
    # ties (first wins), signed zeros, NaN at index 0 (wins), NaN elsewhere (ignored), all NaN
    rows = np.array([
        [1.0, 3.0, 3.0, 2.0],
        [2.0, 2.0, 0.0, 2.0],
        [-0.0, 0.0, -1.0, -0.0],
        [0.0, -0.0, -1.0, 0.0],
        [np.nan, 5.0, 7.0, 1.0],
        [1.0, np.nan, 7.0, np.nan],
        [np.nan, np.nan, np.nan, np.nan],
        [-np.inf, -np.inf, -np.inf, -np.inf],
    ], np.float32)
    d = dev(backend, rows)
    for (outer, length, inner) in ((8, 4, 1), (1, 8, 4)):
        v, i = backend.reduce_axis(d, outer, length, inner, B.REDUCE_MAX, want_index=True)
        assert_bitexact(backend.download(v), port.reduce_axis(oracle.MAX, rows, outer, length, inner))
        assert np.array_equal(backend.download(i), port.argmax_i64(rows, outer, length, inner))
    # the same semantics across split segments of a long row
    long = np.full(200_001, -1.0, np.float32)
    long[[5, 70_000, 150_000]] = 9.0
    long[100_000] = np.nan
    dl = dev(backend, long)
    v, i = backend.reduce_all(dl, long.size, B.REDUCE_MAX, want_index=True)
    assert backend.download(v)[0] == 9.0 and backend.download(i)[0] == 5
    long[0] = np.nan
    v, i = backend.reduce_all(dev(backend, long), long.size, B.REDUCE_MAX, want_index=True)
    assert np.isnan(backend.download(v)[0]) and backend.download(i)[0] == 0


def test_empty_axis(backend):
    x = backend.upload(np.zeros(4, np.float32))
    s = backend.reduce_axis(x, 2, 0, 1, B.REDUCE_SUM)
    assert backend.download(s).tolist() == [0.0, 0.0]
    with pytest.raises(ValueError):
        backend.reduce_axis(x, 2, 0, 1, B.REDUCE_MAX)
    with pytest.raises(ValueError):
        backend.reduce_axis(x, 2, 0, 1, B.REDUCE_MEAN)


@pytest.mark.parametrize("shape", [(3, 4, 5), (64, 512), (7, 33)])
def test_axis_backward_passes(backend, port, shape):
    rng = np.random.default_rng(9)
    x = rng.normal(size=shape).astype(np.float32)
    dx_ = dev(backend, x)
    for axis in range(len(shape)):
        outer, length, inner = split(shape, axis)
        g = rng.uniform(-1, 1, size=outer * inner).astype(np.float32)
        dg = dev(backend, g)
        for kind, op in (("sum", B.REDUCE_SUM), ("mean", B.REDUCE_MEAN), ("max", B.REDUCE_MAX)):
            idx = None
            if kind == "max":
                _, idx = backend.reduce_axis(dx_, outer, length, inner, B.REDUCE_MAX, want_index=True)
            got = backend.download(backend.reduce_axis_backward(op, dg, idx, outer, length, inner))
            ref = port.reduce_op(kind, x, axis, g.reshape(np.delete(shape, axis)))[1]
            assert_bitexact(got.reshape(shape), ref, f"{kind} axis {axis}")


def test_scatter_axis_float_indices(backend, port):
    x = np.random.default_rng(2).normal(size=(6, 9, 4)).astype(np.float32)
    idx = port.reduce_axis(oracle.ARGMAX, x, 6, 9, 4)
    vals = np.random.default_rng(3).normal(size=24).astype(np.float32)
    got = backend.download(backend.scatter_axis(dev(backend, vals), dev(backend, idx), 6, 9, 4))
    assert_bitexact(got, port.scatter_axis(vals, idx, 6, 9, 4))


def test_golden_cfg3(backend, golden):
    x = C.cfg3(C.SMALL["cfg3"]["x"])
    r, c = x.shape
    d = dev(backend, x)
    s1 = backend.download(backend.reduce_axis(d, r, c, 1, B.REDUCE_SUM))
    assert_sum_close(s1, golden["cfg3/sum1/out"].reshape(-1), c, 1.0)
    m1 = backend.download(backend.reduce_axis(d, r, c, 1, B.REDUCE_MEAN))
    assert_sum_close(m1, golden["cfg3/mean1/out"].reshape(-1), c, 1.0 / c)
    mx1, i1 = backend.reduce_axis(d, r, c, 1, B.REDUCE_MAX, want_index=True)
    assert_bitexact(backend.download(mx1), golden["cfg3/max1/out"].reshape(-1))
    assert_bitexact(backend.download(backend.reduce_axis(d, r, c, 1, B.REDUCE_ARGMAX)),
                    golden["cfg3/argmax1/out"].reshape(-1))
    s0 = backend.download(backend.reduce_axis(d, 1, r, c, B.REDUCE_SUM))
    assert_sum_close(s0, golden["cfg3/sum0/out"], r, 1.0)
    mx0 = backend.download(backend.reduce_axis(d, 1, r, c, B.REDUCE_MAX))
    assert_bitexact(mx0, golden["cfg3/max0/out"])
    g = golden["cfg3/max1/g"].reshape(-1)
    dxm = backend.download(backend.reduce_axis_backward(B.REDUCE_MAX, dev(backend, g), i1, r, c, 1))
    assert_bitexact(dxm.reshape(x.shape), golden["cfg3/max1/dx"])
    total = backend.download(backend.reduce_sum(d, x.size))[0]
    assert_sum_close(total, golden["cfg3/sum_all/out"], x.size, 1.0)
    one = dev(backend, np.ones((), np.float32))
    dxs = backend.download(backend.broadcast_to(one, (), x.shape))
    assert sha256(dxs) == str(golden["cfg3/sum_all/dx/sha256"])


def test_golden_cfg1_full_forward_backward(backend, golden):
    """relu(x + b).sum() and its backward at the full configuration-1 shape."""
    x, b = C.cfg1()
    dx_, db_ = dev(backend, x), dev(backend, b)
    h = backend.binary(dx_, x.shape, None, db_, b.shape, None, x.shape, B.ADD)
    y = backend.unary(h, x.size, B.RELU)
    loss = backend.download(backend.reduce_sum(y, x.size))[0]
    assert sha256(backend.download(y)) == str(golden["cfg1_full/y/sha256"])
    assert_sum_close(loss, golden["cfg1_full/loss"], x.size, 1.0)
    one = dev(backend, np.ones((), np.float32))
    g = backend.broadcast_to(one, (), x.shape)
    gh = backend.unary_backward(B.RELU, h, None, g, x.size)
    gx, gb = backend.binary_backward(B.ADD, dx_, x.shape, db_, b.shape, gh, x.shape)
    assert sha256(backend.download(gx)) == str(golden["cfg1_full/dx/sha256"])
    assert_sum_close(backend.download(gb), golden["cfg1_full/db"], x.shape[0], 1.0)

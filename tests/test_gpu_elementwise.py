"""GPU parity: broadcast elementwise ops, unary ops and their backward rules,
called through the C ABI (CudaBackend) and compared with the CPU oracle on the
same seeded inputs, and with the reference's golden vectors.

Tolerances: bit-exact for add/sub/mul/div/neg/relu (and every backward rule
given the same saved tensors); <= 2 ulp for exp/log/sigmoid; sums of broadcast
gradients within the SUM_RTOL class (_util.py)."""
import numpy as np
import pytest

import _cases as C
from _util import assert_bitexact, assert_sum_close, assert_ulp, sha256
from vectorcore_b200 import backend as B

pytestmark = pytest.mark.gpu

OPS = {"add": B.ADD, "sub": B.SUB, "mul": B.MUL, "div": B.DIV}


def dev(be, a):
    return be.upload(np.ascontiguousarray(a, np.float32))


def host(be, s, shape):
    return be.download(s).reshape(shape)


@pytest.mark.parametrize("a_shape,b_shape", C.BROADCAST_CASES)
def test_binary_broadcast_bitexact(backend, port, a_shape, b_shape):
    rng = np.random.default_rng(len(a_shape) * 13 + len(b_shape))
    a = rng.uniform(0.5, 2, size=a_shape).astype(np.float32)
    b = rng.uniform(0.5, 2, size=b_shape).astype(np.float32)
    out_shape = np.broadcast_shapes(a_shape, b_shape)
    da, db = dev(backend, a), dev(backend, b)
    for name, op in OPS.items():
        got = host(backend, backend.binary(da, a_shape, None, db, b_shape, None, out_shape, op), out_shape)
        assert_bitexact(got, port.binary(op, a, b), f"{name} {a_shape} {b_shape}")


@pytest.mark.parametrize("n", [4095, 4096, 4097, 8191, 8196, (1 << 20) + 5, (3 << 20) + 2])
def test_chunked_streams_across_chunk_ends(backend, port, n):
    """The flat kernels give each CTA 4096 elements (1024 float4) and the
    last CTA the n % 4 tail: sizes on both sides of chunk ends, forward and
    backward, bit for bit (exp, log and sigmoid within 2 ulp)."""
    rng = np.random.default_rng(n)
    a = rng.uniform(0.1, 2, size=n).astype(np.float32)
    b = rng.uniform(0.1, 2, size=n).astype(np.float32)
    g = rng.uniform(-1, 1, size=n).astype(np.float32)
    da_, db_, dg = dev(backend, a), dev(backend, b), dev(backend, g)
    shape = (n,)
    for name, op in OPS.items():
        assert_bitexact(host(backend, backend.binary(da_, shape, None, db_, shape, None, shape, op), shape),
                        port.binary(op, a, b), f"{name} n={n}")
        ga, gb = backend.binary_backward(op, da_, shape, db_, shape, dg, shape)
        ra, rb = port.binary_backward(op, a, b, g)
        assert_bitexact(host(backend, ga, shape), ra, f"{name} da n={n}")
        assert_bitexact(host(backend, gb, shape), rb, f"{name} db n={n}")
    assert_bitexact(host(backend, backend.binary_scalar(da_, n, 0.5, B.MUL), shape),
                    port.binary(B.MUL, a, np.array(0.5, np.float32)))
    for op in (B.NEG, B.RELU, B.RELU_GRAD):
        assert_bitexact(host(backend, backend.unary(dg, n, op), shape), port.unary(op, g), f"unary {op} n={n}")
    for op, x, dx in ((B.SIGMOID, g, dg), (B.EXP, g, dg), (B.LOG, a, da_)):
        assert_ulp(host(backend, backend.unary(dx, n, op), shape), port.unary(op, x), what=f"unary {op} n={n}")
    assert_bitexact(host(backend, backend.unary_backward(B.RELU, dg, None, db_, n), shape),
                    port.unary_backward(B.RELU, g, b), f"relu backward n={n}")
    one = dev(backend, np.full(1, 0.25, np.float32))
    got = host(backend, backend.broadcast_to(one, (1,), shape), shape)
    assert (got == np.float32(0.25)).all()


@pytest.mark.parametrize("lo,hi", [(-1.0, 1.0), (-20.0, 20.0), (-90.0, 90.0), (-110.0, 110.0)])
def test_exp_log_sigmoid_wide_sweep(backend, port, lo, hi):
    """2^22 inputs per range (log on |x| spread over 1e-38..1e38): the
    table-driven float exp stays within 1 ulp of the reference's glibc
    result, sigmoid and log within 2 -- including the inputs exp routes to
    its double-precision fallback (|x| > 86, infinities, NaN)."""
    rng = np.random.default_rng(int(hi))
    x = rng.uniform(lo, hi, size=1 << 22).astype(np.float32)
    x[:6] = [np.inf, -np.inf, np.nan, 0.0, -0.0, 86.0]
    dx = dev(backend, x)
    n = x.size
    assert_ulp(host(backend, backend.unary(dx, n, B.EXP), x.shape), port.unary(B.EXP, x), max_ulp=1, what="exp")
    assert_ulp(host(backend, backend.unary(dx, n, B.SIGMOID), x.shape), port.unary(B.SIGMOID, x), what="sigmoid")
    lx = np.exp(rng.uniform(np.log(1e-38), np.log(1e38), size=1 << 22)).astype(np.float32)
    lx[:5] = [np.inf, 0.0, 1e-40, 1.0, np.float32(0.75)]
    assert_ulp(host(backend, backend.unary(dev(backend, lx), n, B.LOG), lx.shape), port.unary(B.LOG, lx),
               what="log")


@pytest.mark.parametrize("shape", [(1,), (3,), (127,), (1023,), (4097,), (65537,), (2, 3, 5, 7), ()])
def test_binary_odd_sizes_and_rank0(backend, port, shape):
    rng = np.random.default_rng(sum(shape) + 1)
    a = rng.uniform(0.1, 2, size=shape).astype(np.float32)
    b = rng.uniform(0.1, 2, size=shape).astype(np.float32)
    da, db = dev(backend, a), dev(backend, b)
    for op in OPS.values():
        got = host(backend, backend.binary(da, shape, None, db, shape, None, shape, op), shape)
        assert_bitexact(got, port.binary(op, a, b))


def test_binary_strided_operand(backend):
    # a transposed view of a contiguous buffer: shape [300, 1000], strides [1, 300]
    rng = np.random.default_rng(1)
    base = rng.normal(size=(1000, 300)).astype(np.float32)
    b = rng.normal(size=(300, 1000)).astype(np.float32)
    dbase, db = dev(backend, base), dev(backend, b)
    got = host(backend, backend.binary(dbase, (300, 1000), (1, 300), db, (300, 1000), None, (300, 1000), B.MUL),
               (300, 1000))
    assert_bitexact(got, base.T * b)


def test_binary_zero_size(backend):
    s = backend.upload(np.zeros(4, np.float32))
    out = backend.binary(s, (0, 4), None, s, (4,), None, (0, 4), B.ADD)
    assert out.size == 0
    backend.synchronize()


def test_binary_rejects_bad_broadcast(backend):
    s = backend.upload(np.zeros(6, np.float32))
    with pytest.raises(ValueError):
        backend.binary(s, (2, 3), None, s, (3, 2), None, (2, 3), B.ADD)


def test_scalar_operand_paths(backend, port):
    a = C.uniform(2, (257, 33), 0.1, 2.0)
    da = dev(backend, a)
    for op in OPS.values():
        for first in (False, True):
            got = host(backend, backend.binary_scalar(da, a.size, 0.5, op, first), a.shape)
            s = np.array(0.5, np.float32)
            ref = port.binary(op, s, a) if first else port.binary(op, a, s)
            assert_bitexact(got, ref)
            # one-element device tensor as the scalar (MetalBackend::binary shape [])
            ds = dev(backend, s)
            got2 = (backend.binary(ds, (), None, da, a.shape, None, a.shape, op) if first
                    else backend.binary(da, a.shape, None, ds, (), None, a.shape, op))
            assert_bitexact(host(backend, got2, a.shape), ref)


SPECIAL = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan, 1e-40, -1e-40, 1e-30, 88.72, 88.73,
                    -87.3, -103.9, -104.0, 20.0, -20.0, 1e30, -1e30, 3.4e38], np.float32)


@pytest.mark.parametrize("op,name", [(B.NEG, "neg"), (B.RELU, "relu"), (B.RELU_GRAD, "relu_grad"),
                                     (B.EXP, "exp"), (B.LOG, "log"), (B.SIGMOID, "sigmoid")])
def test_unary(backend, port, op, name):
    x = C.uniform(3, (700, 301), -5, 5)
    if op == B.LOG:
        x = np.abs(x) + np.float32(0.01)
    for xx in (x, SPECIAL, np.abs(SPECIAL)):
        got = host(backend, backend.unary(dev(backend, xx), xx.size, op), xx.shape)
        ref = port.unary(op, xx)
        if op in (B.EXP, B.LOG, B.SIGMOID):
            assert_ulp(got, ref, 2, name)
        else:
            assert_bitexact(got, ref, name)


@pytest.mark.parametrize("op", [B.NEG, B.RELU, B.EXP, B.LOG, B.SIGMOID])
def test_unary_backward_bitexact_given_saved(backend, port, op):
    x = C.uniform(4, (513, 129), -4, 4)
    if op == B.LOG:
        x = np.abs(x) + np.float32(0.05)
    g = C.uniform(5, x.shape, -1, 1)
    y = port.unary(op, x)  # the same saved output on both sides
    got = host(backend, backend.unary_backward(op, dev(backend, x), dev(backend, y), dev(backend, g), x.size),
               x.shape)
    assert_bitexact(got, port.unary_backward_saved(op, x, y, g))


@pytest.mark.parametrize("a_shape,b_shape", C.BROADCAST_CASES + [((64, 1, 16, 32), (1, 8, 1, 32))])
def test_binary_backward(backend, port, a_shape, b_shape):
    rng = np.random.default_rng(len(a_shape) * 7 + len(b_shape))
    a = rng.uniform(0.5, 2, size=a_shape).astype(np.float32)
    b = rng.uniform(0.5, 2, size=b_shape).astype(np.float32)
    out_shape = np.broadcast_shapes(a_shape, b_shape)
    g = rng.uniform(-1, 1, size=out_shape).astype(np.float32)
    da_, db_, dg = dev(backend, a), dev(backend, b), dev(backend, g)
    for name, op in OPS.items():
        ga, gb = backend.binary_backward(op, da_, a_shape, db_, b_shape, dg, out_shape)
        ra, rb = port.binary_backward(op, a, b, g)
        for got_s, ref, shape, other in ((ga, ra, a_shape, a), (gb, rb, b_shape, b)):
            got = host(backend, got_s, shape)
            n = int(np.prod(out_shape)) // max(1, int(np.prod(shape)))
            if n <= 1:
                assert_bitexact(got, ref, f"{name} grad {shape}")
            else:
                assert_sum_close(got, ref, n, 1.0, what=f"{name} grad {shape} of {out_shape}")


# Two-sided broadcasts: both gradients reduce, from one pass over g. Cases
# cover V (the dims only b spans) = 128, a non-power-of-two V, a partial
# 32-float chunk of the inner run, two a-only and two b-only dims
# interleaved, an outer dim both operands span, and enough a-only positions
# for many U segments. The TMA-fed kernel takes one V dim of 16, 32, 64 or
# 128 rows with the inner run a multiple of 64 (V = 128, 64, 32 and 16 below,
# with one a-only dim or two, one U segment or up to 256); the register
# kernel the rest (V = 128 with a 96-float run keeps its full-tile path).
FUSED_CASES = [((8, 1, 64, 256), (1, 128, 1, 256)), ((16, 1, 40, 64), (1, 3, 1, 64)),
               ((4, 1, 50, 96), (1, 100, 1, 96)), ((7, 1, 33, 36), (1, 9, 1, 36)),
               ((1, 6, 1, 10, 16), (4, 1, 5, 1, 16)), ((5, 3, 1, 128), (5, 1, 2, 128)),
               ((64, 1, 512, 64), (1, 16, 1, 64)), ((4, 1, 20, 96), (1, 128, 1, 96)),
               ((3, 1, 70, 128), (1, 64, 1, 128)), ((300, 1, 192), (1, 32, 192)),
               ((2, 1, 5, 64), (1, 32, 1, 64))]


@pytest.mark.parametrize("a_shape,b_shape", FUSED_CASES)
def test_binary_backward_two_sided_broadcast(backend, port, a_shape, b_shape):
    rng = np.random.default_rng(int(np.prod(a_shape)) % 997)
    a = rng.uniform(0.5, 2, size=a_shape).astype(np.float32)
    b = rng.uniform(0.5, 2, size=b_shape).astype(np.float32)
    out_shape = np.broadcast_shapes(a_shape, b_shape)
    g = rng.uniform(-1, 1, size=out_shape).astype(np.float32)
    da_, db_, dg = dev(backend, a), dev(backend, b), dev(backend, g)
    for name, op in OPS.items():
        ga, gb = backend.binary_backward(op, da_, a_shape, db_, b_shape, dg, out_shape)
        ra, rb = port.binary_backward(op, a, b, g)
        for got_s, ref, shape in ((ga, ra, a_shape), (gb, rb, b_shape)):
            n = int(np.prod(out_shape)) // int(np.prod(shape))
            assert_sum_close(host(backend, got_s, shape), ref, n, 1.0, what=f"{name} grad {shape} of {out_shape}")
    backend.synchronize()  # no bounded wait gave up


@pytest.mark.parametrize("a_shape,b_shape", [((16, 1, 40, 64), (1, 24, 1, 64)), ((16, 1, 40, 64), (1, 32, 1, 64)),
                                             ((2, 1, 5, 64), (1, 32, 1, 64))])
def test_binary_backward_partial_two_sided(backend, port, a_shape, b_shape):
    """The shard-partial entry point returns the unrounded double sums of the
    same fused pass (register kernel; TMA-fed kernel with several U segments
    and with one)."""
    import ctypes

    from vectorcore_b200 import _abi

    rng = np.random.default_rng(3)
    a = rng.uniform(0.5, 2, size=a_shape).astype(np.float32)
    b = rng.uniform(0.5, 2, size=b_shape).astype(np.float32)
    out_shape = np.broadcast_shapes(a_shape, b_shape)
    g = rng.uniform(-1, 1, size=out_shape).astype(np.float32)
    da_, db_, dg = dev(backend, a), dev(backend, b), dev(backend, g)
    pa = backend.allocate(2 * a.size)  # room for a.size doubles
    pb = backend.allocate(2 * b.size)
    shp = lambda s: (ctypes.c_size_t * len(s))(*s)
    _abi.call("vc_cuda_binary_backward_partial", B.MUL, ctypes.c_void_p(da_.ptr), shp(a_shape), len(a_shape),
              ctypes.c_void_p(db_.ptr), shp(b_shape), len(b_shape), ctypes.c_void_p(dg.ptr), shp(out_shape),
              len(out_shape), ctypes.c_void_p(pa.ptr), ctypes.c_void_p(pb.ptr))
    got_a = backend.download(pa).view(np.float64).reshape(a_shape)
    got_b = backend.download(pb).view(np.float64).reshape(b_shape)
    ra, rb = port.binary_backward(B.MUL, a, b, g)
    n_b = int(np.prod(out_shape)) // b.size
    assert_sum_close(got_a.astype(np.float32), ra, b_shape[1], 1.0, what="da partial")
    assert_sum_close(got_b.astype(np.float32), rb, n_b, 1.0, what="db partial")


def test_binary_backward_scalar_upstream(backend, port):
    # sum() backward hands a 0-d gradient; the kernel reads it broadcast.
    a, b = C.cfg5(C.SMALL["cfg5"]["a"], C.SMALL["cfg5"]["b"])
    out_shape = np.broadcast_shapes(a.shape, b.shape)
    one = dev(backend, np.ones((), np.float32))
    ga, gb = backend.binary_backward(B.MUL, dev(backend, a), a.shape, dev(backend, b), b.shape, one, ())
    ra, rb = port.binary_backward(B.MUL, a, b, np.ones(out_shape, np.float32))
    assert_sum_close(host(backend, ga, a.shape), ra, 16, 1.0)
    assert_sum_close(host(backend, gb, b.shape), rb, 32, 1.0)


# A 0-d upstream makes each gradient constant along the dims only the other
# operand spans: the reduction runs on the compact shape and is replicated --
# by the reduction itself when the copies are few and lead the kept dims
# (single-launch sliced sums, sliced finishes), by a broadcast when they are
# many, and by a broadcast from a scratch block when they interleave.
@pytest.mark.parametrize("a_shape,b_shape", [((2, 1, 300, 40), (1, 7, 1, 40)), ((64, 1, 512, 64), (1, 16, 1, 64)),
                                             ((4, 6), (4, 1)), ((3, 1, 5), (1, 4, 1)), ((1, 9, 1, 33), (6, 1, 70, 33)),
                                             ((5, 2000), (2000,))])
def test_binary_backward_scalar_upstream_layouts(backend, port, a_shape, b_shape):
    rng = np.random.default_rng(int(np.prod(a_shape)) % 1009)
    a = rng.uniform(0.5, 2, size=a_shape).astype(np.float32)
    b = rng.uniform(0.5, 2, size=b_shape).astype(np.float32)
    out_shape = np.broadcast_shapes(a_shape, b_shape)
    u = np.float32(-0.37)
    du = dev(backend, np.full((), u, np.float32))
    da_, db_ = dev(backend, a), dev(backend, b)
    for name, op in OPS.items():
        for _ in range(2):  # the replicas of a reused output block are rewritten, not accumulated
            ga, gb = backend.binary_backward(op, da_, a_shape, db_, b_shape, du, ())
        ra, rb = port.binary_backward(op, a, b, np.full(out_shape, u, np.float32))
        for got_s, ref, shape in ((ga, ra, a_shape), (gb, rb, b_shape)):
            n = int(np.prod(out_shape)) // int(np.prod(shape))
            assert_sum_close(host(backend, got_s, shape), ref, n, 1.0, what=f"{name} grad {shape} of {out_shape}")


@pytest.mark.parametrize("big,small", C.SUM_TO_SHAPE_CASES)
def test_sum_to_shape(backend, port, big, small):
    g = np.random.default_rng(6).normal(size=big).astype(np.float32)
    got = host(backend, backend.sum_to_shape(dev(backend, g), big, small), small)
    ref = port.sum_to_shape(g, small)
    n = int(np.prod(big)) // max(1, int(np.prod(small)))
    assert_sum_close(got, ref, n, 1.0, what=f"{big}->{small}")


def test_broadcast_to_turns_negative_zero_positive(backend):
    v = np.array([-0.0, 1.0, np.nan], np.float32)
    got = host(backend, backend.broadcast_to(dev(backend, v), (3,), (2, 3)), (2, 3))
    assert_bitexact(got, np.broadcast_to(v + np.float32(0.0), (2, 3)))
    assert got.view(np.uint32)[0, 0] == 0  # +0.0


def test_axpy(backend):
    t = C.uniform(1, (1001,), -1, 1)
    s = C.uniform(2, (1001,), -1, 1)
    dt = dev(backend, t)
    backend.axpy_inplace(dt, dev(backend, s), t.size, -0.25)
    assert_bitexact(host(backend, dt, t.shape), t - np.float32(0.25) * s)


# ---- golden vectors of the reference ------------------------------------------------

def test_golden_elementwise(backend, golden):
    a, b = golden["kat/ew/a"], golden["kat/ew/b"]
    for name, op in OPS.items():
        got = host(backend, backend.binary(dev(backend, a), a.shape, None, dev(backend, b), b.shape, None, a.shape, op),
                   a.shape)
        assert_bitexact(got, golden[f"kat/ew/{name}"])
    a2, b2, g2 = C.cfg2(C.SMALL["cfg2"]["a"])
    for name, op in OPS.items():
        out = host(backend, backend.binary(dev(backend, a2), a2.shape, None, dev(backend, b2), b2.shape, None,
                                           a2.shape, op), a2.shape)
        assert_bitexact(out, golden[f"cfg2/{name}/out"], name)
        ga, gb = backend.binary_backward(op, dev(backend, a2), a2.shape, dev(backend, b2), b2.shape,
                                         dev(backend, g2), a2.shape)
        assert_bitexact(host(backend, ga, a2.shape), golden[f"cfg2/{name}/da"], name)
        assert_bitexact(host(backend, gb, a2.shape), golden[f"cfg2/{name}/db"], name)
    for name, op in (("neg", B.NEG), ("relu", B.RELU), ("exp", B.EXP), ("log", B.LOG), ("sigmoid", B.SIGMOID)):
        x = golden[f"cfg2/{name}/x"]
        got = host(backend, backend.unary(dev(backend, x), x.size, op), x.shape)
        if op in (B.EXP, B.LOG, B.SIGMOID):
            assert_ulp(got, golden[f"cfg2/{name}/out"], 2, name)
        else:
            assert_bitexact(got, golden[f"cfg2/{name}/out"], name)


def test_golden_cfg5_forward_hash(backend, golden):
    a, b = C.cfg5(C.SMALL["cfg5"]["a"], C.SMALL["cfg5"]["b"])
    out_shape = np.broadcast_shapes(a.shape, b.shape)
    got = host(backend, backend.binary(dev(backend, a), a.shape, None, dev(backend, b), b.shape, None, out_shape,
                                       B.MUL), out_shape)
    assert sha256(got) == str(golden["cfg5/out/sha256"])

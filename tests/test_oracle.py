"""Pin the CPU oracle: the C restatement (oracle/vc_oracle.c) must reproduce
the reference's own outputs -- the golden vectors made by the reference's
Python module (tests/golden/make_golden.py) and, where the reference's CPU
path was compiled here (oracle/_ref), the reference itself on random inputs.
CPU only."""
import numpy as np
import pytest

import _cases as C
import oracle
from _util import assert_bitexact, sha256

ADD, SUB, MUL, DIV = oracle.ADD, oracle.SUB, oracle.MUL, oracle.DIV
BIN = {"add": ADD, "sub": SUB, "mul": MUL, "div": DIV}


# ---- known answers of the reference's own test suites ---------------------------

def test_kat_elementwise(port, golden):
    a, b = golden["kat/ew/a"], golden["kat/ew/b"]
    for name, op in BIN.items():
        assert_bitexact(port.binary(op, a, b), golden[f"kat/ew/{name}"], name)
    assert_bitexact(port.unary(oracle.NEG, a), golden["kat/ew/neg"])
    m = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    assert_bitexact(port.binary(ADD, m, np.array([10, 20, 30], np.float32)), golden["kat/bcast/row"])


def test_kat_bias_grad(port, golden):
    # tests/cpp/test_vectorcore.cpp:125-131: bias.grad == {2, 2, 2}
    x = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    b = np.array([0.1, 0.2, 0.3], np.float32)
    g = port.reduce_op("sum", port.binary(ADD, x, b), None, np.float32(1.0))[1]
    dx, db = port.binary_backward(ADD, x, b, g)
    assert_bitexact(dx, golden["kat/bias_grad/dx"])
    assert_bitexact(db, golden["kat/bias_grad/db"])
    assert db.tolist() == [2.0, 2.0, 2.0]


def test_kat_axis_reductions(port, golden):
    x = golden["kat/axis/x"]
    assert_bitexact(port.reduce_op("sum", x, 0)[0], golden["kat/axis/sum0"])
    assert_bitexact(port.reduce_op("sum", x, -1)[0], golden["kat/axis/sum_m1_keep"].reshape(-1))
    assert_bitexact(port.reduce_op("mean", x, 1)[0], golden["kat/axis/mean1"])
    assert_bitexact(port.reduce_op("max", x, 1)[0], golden["kat/axis/max1"])
    assert_bitexact(port.reduce_axis(oracle.ARGMAX, x, 2, 3, 1), golden["kat/axis/argmax1"])
    assert_bitexact(port.reduce_op("max", x, None)[0], golden["kat/axis/max_all"])


def test_kat_cross_entropy(port, golden):
    loss, dx = port.cross_entropy(np.zeros((2, 2), np.float32), [0, 1])
    assert_bitexact(loss, golden["kat/ce/loss"])
    assert_bitexact(dx, golden["kat/ce/grad"])
    assert dx.tolist() == [[-0.25, 0.25], [0.25, -0.25]]


def test_kat_ties_and_kinks(port, golden):
    t = np.array([[1, 3, 3], [2, 2, 0]], np.float32)
    assert_bitexact(port.reduce_axis(oracle.ARGMAX, t, 2, 3, 1), golden["kat/ties/argmax1"])
    _, dx = port.reduce_op("max", np.array([[1, 3, 3]], np.float32), 1, np.ones(1, np.float32))
    assert_bitexact(dx, golden["kat/ties/max_grad"])
    k = np.array([0.0, -0.0, 1.0], np.float32)
    assert_bitexact(port.unary_backward(oracle.RELU, k, np.ones(3, np.float32)), golden["kat/relu_kink/grad"])


def test_kat_huge_logits(port, golden):
    huge = np.array([[1000, 1001, 1002], [-1000, 0, 1000]], np.float32)
    assert_bitexact(port.softmax(huge, -1), golden["kat/huge/softmax"])
    _, dx = port.cross_entropy(huge, [2, 0])
    assert_bitexact(dx, golden["kat/huge/ce_grad"])


# ---- seeded benchmark configurations at golden scale -----------------------------

def test_golden_cfg1(port, golden):
    for tag, shape in (("cfg1_small", C.SMALL["cfg1"]["x"]), ("cfg1_full", C.CFG1["x"])):
        x, b = C.cfg1(shape)
        y = port.unary(oracle.RELU, port.binary(ADD, x, b))
        loss, g = port.reduce_op("sum", y, None, np.float32(1.0))
        dy = port.unary_backward(oracle.RELU, port.binary(ADD, x, b), g)
        dx, db = port.binary_backward(ADD, x, b, dy)
        assert_bitexact(loss, golden[f"{tag}/loss"], tag)
        assert_bitexact(db, golden[f"{tag}/db"], tag)
        assert sha256(dx) == str(golden[f"{tag}/dx/sha256"])
        assert sha256(y) == str(golden[f"{tag}/y/sha256"])


def test_golden_cfg2(port, golden):
    a, b, g = C.cfg2(C.SMALL["cfg2"]["a"])
    for name, op in BIN.items():
        assert_bitexact(port.binary(op, a, b), golden[f"cfg2/{name}/out"], name)
        da, db = port.binary_backward(op, a, b, g)
        assert_bitexact(da, golden[f"cfg2/{name}/da"], name)
        assert_bitexact(db, golden[f"cfg2/{name}/db"], name)
    un = {"neg": oracle.NEG, "exp": oracle.EXP, "log": oracle.LOG, "relu": oracle.RELU,
          "sigmoid": oracle.SIGMOID}
    for name, op in un.items():
        x = golden[f"cfg2/{name}/x"]
        assert_bitexact(port.unary(op, x), golden[f"cfg2/{name}/out"], name)
        assert_bitexact(port.unary_backward(op, x, g), golden[f"cfg2/{name}/dx"], name)
    x = golden["cfg2/scalar_mul/x"]
    assert_bitexact(port.binary(MUL, x, np.float32(0.5)), golden["cfg2/scalar_mul/out"])
    assert_bitexact(port.binary_backward(MUL, x, np.array(0.5, np.float32), g, need_b=False)[0],
                    golden["cfg2/scalar_mul/dx"])


def test_golden_cfg3(port, golden):
    x = C.cfg3(C.SMALL["cfg3"]["x"])
    for name, axis in (("sum1", 1), ("mean1", 1), ("max1", 1), ("sum0", 0), ("max0", 0)):
        g = golden[f"cfg3/{name}/g"]
        out, dx = port.reduce_op(name[:-1], x, axis, g)
        assert_bitexact(out, golden[f"cfg3/{name}/out"].reshape(out.shape), name)
        assert_bitexact(dx, golden[f"cfg3/{name}/dx"], name)
    assert_bitexact(port.reduce_axis(oracle.ARGMAX, x, x.shape[0], x.shape[1], 1),
                    golden["cfg3/argmax1/out"].reshape(-1))
    for name in ("sum", "mean"):
        out, dx = port.reduce_op(name, x, None, np.float32(1.0))
        assert_bitexact(out, golden[f"cfg3/{name}_all/out"], name)
        assert sha256(dx) == str(golden[f"cfg3/{name}_all/dx/sha256"])


def test_golden_cfg4(port, golden):
    lg, tg = C.cfg4(C.SMALL["cfg4"]["logits"])
    assert np.array_equal(tg, golden["cfg4/targets"])
    g = C.uniform(10, lg.shape, -1.0, 1.0)
    assert_bitexact(port.softmax(lg), golden["cfg4/softmax/out"])
    assert_bitexact(port.log_softmax(lg), golden["cfg4/log_softmax/out"])
    assert_bitexact(port.softmax_backward(lg, g), golden["cfg4/softmax/dx"])
    assert_bitexact(port.log_softmax_backward(lg, g), golden["cfg4/log_softmax/dx"])
    loss, dx = port.cross_entropy(lg, tg)
    assert_bitexact(loss, golden["cfg4/ce/loss"])
    assert_bitexact(dx, golden["cfg4/ce/dx"])


def test_golden_cfg5(port, golden):
    a, b = C.cfg5(C.SMALL["cfg5"]["a"], C.SMALL["cfg5"]["b"])
    out = port.binary(MUL, a, b)
    assert sha256(out) == str(golden["cfg5/out/sha256"])
    s, g = port.reduce_op("sum", out, None, np.float32(1.0))
    assert_bitexact(s, golden["cfg5/sum"])
    da, db = port.binary_backward(MUL, a, b, g)
    assert_bitexact(da, golden["cfg5/sum_bwd/da"])
    assert_bitexact(db, golden["cfg5/sum_bwd/db"])
    gd = C.uniform(11, out.shape, -1.0, 1.0)
    da, db = port.binary_backward(MUL, a, b, gd)
    assert_bitexact(da, golden["cfg5/dense_bwd/da"])
    assert_bitexact(db, golden["cfg5/dense_bwd/db"])


# ---- restatement vs the reference's own compiled CPU path ------------------------

needs_ref = pytest.mark.skipif(not oracle.reference_available(),
                               reason="reference CPU path not built here (oracle/_ref)")


@needs_ref
@pytest.mark.parametrize("a_shape,b_shape", C.BROADCAST_CASES)
def test_port_matches_reference_binary(port, a_shape, b_shape):
    ref = oracle.reference()
    rng = np.random.default_rng(len(a_shape) * 13 + len(b_shape))
    a = rng.uniform(0.5, 2, size=a_shape).astype(np.float32)
    b = rng.uniform(0.5, 2, size=b_shape).astype(np.float32)
    g = rng.normal(size=np.broadcast_shapes(a_shape, b_shape)).astype(np.float32)
    for op in range(4):
        assert_bitexact(port.binary(op, a, b), ref.binary(op, a, b))
        pa, pb = port.binary_backward(op, a, b, g)
        ra, rb = ref.binary_backward(op, a, b, g)
        assert_bitexact(pa, ra)
        assert_bitexact(pb, rb)


@needs_ref
def test_port_matches_reference_unary_and_sum(port):
    ref = oracle.reference()
    rng = np.random.default_rng(3)
    x = rng.uniform(-5, 5, size=(700, 300)).astype(np.float32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -1e-40, 88.7, -88.7, 1e30], np.float32)
    for op in range(6):
        for xx in (x, special):
            xx = np.abs(xx) + np.float32(0.1) if op == oracle.LOG and xx is x else xx
            assert_bitexact(port.unary(op, xx), ref.unary(op, xx), f"unary {op}")
    g = rng.normal(size=x.shape).astype(np.float32)
    for op in (oracle.NEG, oracle.RELU, oracle.SIGMOID, oracle.EXP, oracle.LOG):
        xx = np.abs(x) + np.float32(0.1) if op == oracle.LOG else x
        assert_bitexact(port.unary_backward(op, xx, g), ref.unary_backward(op, xx, g))
    v = rng.normal(size=3_000_001).astype(np.float32)
    assert_bitexact(port.sum(v), ref.sum(v))


@needs_ref
def test_port_matches_reference_reductions(port):
    ref = oracle.reference()
    rng = np.random.default_rng(5)
    t = rng.normal(size=(64, 50, 33)).astype(np.float32)
    t[3, 0, 4] = np.nan
    t[5, 7, 2] = np.nan
    for axis in range(3):
        for kind in ("sum", "mean", "max"):
            gg = rng.normal(size=np.delete(t.shape, axis)).astype(np.float32)
            po, pdx = port.reduce_op(kind, t, axis, gg)
            ro, rdx = ref.reduce_op(kind, t, axis, gg)
            assert_bitexact(po, ro, f"{kind} axis {axis}")
            assert_bitexact(pdx, rdx, f"{kind} axis {axis} backward")
    for kind in ("sum", "mean", "max"):
        po, pdx = port.reduce_op(kind, t, None, np.float32(0.7))
        ro, rdx = ref.reduce_op(kind, t, None, np.float32(0.7))
        assert_bitexact(po, ro)
        assert_bitexact(pdx, rdx)


@needs_ref
@pytest.mark.parametrize("big,small", C.SUM_TO_SHAPE_CASES)
def test_port_matches_reference_sum_to_shape(port, big, small):
    ref = oracle.reference()
    g = np.random.default_rng(6).normal(size=big).astype(np.float32)
    assert_bitexact(port.sum_to_shape(g, small), ref.sum_to_shape(g, small))


@needs_ref
@pytest.mark.parametrize("axis", [0, 1, -1])
def test_port_matches_reference_softmax_family(port, axis):
    ref = oracle.reference()
    rng = np.random.default_rng(4)
    s = (rng.normal(size=(37, 45)) * 3).astype(np.float32)
    g = rng.normal(size=s.shape).astype(np.float32)
    assert_bitexact(port.log_softmax(s, axis), ref.log_softmax(s, axis))
    assert_bitexact(port.softmax(s, axis), ref.softmax(s, axis))
    assert_bitexact(port.log_softmax_backward(s, g, axis), ref.log_softmax_backward(s, g, axis))
    assert_bitexact(port.softmax_backward(s, g, axis), ref.softmax_backward(s, g, axis))


@needs_ref
def test_port_matches_reference_cross_entropy(port):
    ref = oracle.reference()
    rng = np.random.default_rng(9)
    lg = rng.normal(0, 2, (64, 1000)).astype(np.float32)
    tg = rng.integers(0, 1000, 64)
    for u in (1.0, 0.37, -2.5):
        pl, pd = port.cross_entropy(lg, tg, u)
        rl, rd = ref.cross_entropy(lg, tg, u)
        assert_bitexact(pl, rl)
        assert_bitexact(pd, rd)


def test_port_rejects_what_the_reference_rejects(port):
    with pytest.raises(oracle.OracleError):
        port.reduce_axis(oracle.MAX, np.zeros((2, 0), np.float32), 2, 0, 1)
    with pytest.raises(oracle.OracleError):
        port.cross_entropy(np.zeros((1, 2), np.float32), [2])
    with pytest.raises(oracle.OracleError):
        port.sum_to_shape(np.zeros((3, 4), np.float32), (2, 4))

"""GPU parity: fused softmax, log_softmax and softmax cross-entropy, forward
and backward, through the C ABI against the CPU oracle (which replays the
reference's composed ops and autograd chain) and the golden vectors.

Tolerance: relative 1e-5 (SUM_RTOL class; _util.assert_rel) -- the fused
kernels perform the reference's float operations in the same order, so the
remaining differences come from expf/logf ulps and the order of double
additions. Row lengths cover every cluster size (1, 2, 4, 8 CTAs per row),
unaligned rows (plain loads instead of TMA bulk copies) and the column
kernel (other axes, rows longer than a cluster holds)."""
import numpy as np
import pytest

import _cases as C
from _util import assert_rel
from vectorcore_b200 import backend as B

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def dev(be, a):
    return be.upload(np.ascontiguousarray(a))


def split(shape, axis):
    ax = axis % len(shape)
    return (int(np.prod(shape[:ax], dtype=np.int64)), int(shape[ax]),
            int(np.prod(shape[ax + 1:], dtype=np.int64)))


CASES = [((6, 5), -1), ((6, 5), 0), ((3, 7, 9), 1), ((37, 45), 0), ((64, 1000), -1), ((16, 8191), -1),
         ((8, 9000), -1), ((4, 20000), -1), ((4, 32000), -1), ((2, 70000), -1), ((2, 196608), -1),
         ((2, 200003), -1), ((3, 33), -1), ((1, 1), -1),
         # thousands of rows: many clusters per SM, every cluster size
         ((3000, 1000), -1), ((700, 9000), -1), ((1200, 32000), -1), ((300, 70000), -1), ((2500, 33), -1),
         # the forward's shared-memory ring (rows of 8192..40960 floats, in
         # 2048-float chunks): both ends, a ragged last chunk, rows > SMs
         ((150, 8192), -1), ((160, 40960), -1), ((149, 10004), -1)]


@pytest.mark.parametrize("shape,axis", CASES)
def test_softmax_family(backend, port, shape, axis):
    rng = np.random.default_rng(int(np.prod(shape)) % 1000)
    x = (rng.normal(size=shape) * 2).astype(np.float32)
    g = rng.uniform(-1, 1, size=shape).astype(np.float32)
    outer, length, inner = split(shape, axis)
    dx, dg = dev(backend, x), dev(backend, g)
    for log in (True, False):
        y, m, s = backend.softmax(dx, outer, length, inner, log=log)
        ref = port.log_softmax(x, axis) if log else port.softmax(x, axis)
        assert_rel(backend.download(y).reshape(shape), ref, RTOL, f"{'log_' if log else ''}softmax {shape}")
        gx = backend.softmax_backward(dx, m, s, dg, outer, length, inner, log=log)
        refb = port.log_softmax_backward(x, g, axis) if log else port.softmax_backward(x, g, axis)
        assert_rel(backend.download(gx).reshape(shape), refb, RTOL, f"backward {shape}", scale=np.abs(g).max())
    _, pm, ps = port.log_softmax(x, axis, stats=True)
    assert np.array_equal(backend.download(m), pm)  # the row max is exact
    # the row sums' exp terms come from an ex2-based exp (a few float ulps a
    # term): the sum stays within 2e-6 of the reference's double sum of expf
    np.testing.assert_allclose(backend.download(s), ps, rtol=2e-6, atol=0)


@pytest.mark.parametrize("length", [1024, 32000])
def test_softmax_edge_rows_among_many(backend, port, length):
    """Rows with the scan's special cases (a zero maximum whose first zero is
    -0.0, NaN at index 0, NaN elsewhere, -inf, +-1000) scattered among
    thousands of ordinary rows, in CTAs other than the first of a cluster."""
    rows = 3000 if length == 1024 else 400
    rng = np.random.default_rng(length)
    x = rng.normal(0, 2, size=(rows, length)).astype(np.float32)
    x[5] = 0.0
    x[5, : length // 3] = -5.0
    x[5, length // 3] = -0.0            # the first zero is negative
    x[6] = -0.0
    x[6, length - 1] = 0.0
    x[7, 0] = np.nan                    # NaN at index 0 wins the max
    x[rows // 2, length - 3] = np.nan   # NaN elsewhere: skipped by the max, poisons the sum
    x[rows - 1, ::7] = -np.inf
    x[rows - 2, 1] = 1000.0
    x[rows - 2, length - 2] = -1000.0
    x[rows - 3] = 0.0                   # all +0.0
    g = rng.uniform(-1, 1, size=x.shape).astype(np.float32)
    dx, dg = dev(backend, x), dev(backend, g)
    with np.errstate(invalid="ignore"):
        for log in (True, False):
            y, m, s = backend.softmax(dx, rows, length, 1, log=log)
            ref = port.log_softmax(x, -1) if log else port.softmax(x, -1)
            assert_rel(backend.download(y).reshape(x.shape), ref, RTOL, f"{'log_' if log else ''}softmax edges")
            gx = backend.softmax_backward(dx, m, s, dg, rows, length, 1, log=log)
            refb = port.log_softmax_backward(x, g, -1) if log else port.softmax_backward(x, g, -1)
            assert_rel(backend.download(gx).reshape(x.shape), refb, RTOL, "backward edges", scale=1.0)
    _, pm, _ = port.log_softmax(x, -1, stats=True)
    got_m = backend.download(m)
    same = (got_m.view(np.uint32) == pm.view(np.uint32)) | (np.isnan(got_m) & np.isnan(pm))
    assert same.all(), np.flatnonzero(~same)[:10]
    assert got_m.view(np.uint32)[5] == np.float32(-0.0).view(np.uint32)


def test_softmax_rows_sum_to_one_and_huge_logits(backend, golden):
    huge = np.array([[1000, 1001, 1002], [-1000, 0, 1000]], np.float32)
    y, _, _ = backend.softmax(dev(backend, huge), 2, 3, 1)
    got = backend.download(y).reshape(2, 3)
    assert np.all(np.isfinite(got))
    assert_rel(got, golden["kat/huge/softmax"], RTOL)


def test_cross_entropy(backend, port):
    for shape in ((6, 4), (64, 1000), (33, 32000), (5, 9001)):
        lg = np.random.default_rng(shape[1]).normal(0, 2, size=shape).astype(np.float32)
        tg = np.random.default_rng(shape[0]).integers(0, shape[1], shape[0]).astype(np.int64)
        dlg, dtg = dev(backend, lg), dev(backend, tg)
        loss, m, s, part = backend.cross_entropy(dlg, dtg, *shape)
        ref_loss, ref_dx = port.cross_entropy(lg, tg, 1.0)
        assert_rel(backend.download(loss), np.array([ref_loss]), RTOL, f"loss {shape}")
        for u in (1.0, 0.37):
            up = dev(backend, np.array([u], np.float32))
            dx = backend.cross_entropy_backward(dlg, dtg, m, s, up, *shape)
            _, rdx = port.cross_entropy(lg, tg, u)
            assert_rel(backend.download(dx).reshape(shape), rdx, RTOL, f"dlogits {shape} u={u}")


@pytest.mark.parametrize("length", [4, 12, 132, 1024, 32000])
def test_cross_entropy_edge_rows_among_many(backend, port, length):
    """The cross-entropy row statistics under the scan's special cases (a
    zero maximum whose first zero is -0.0, NaN at index 0, NaN elsewhere,
    -inf, +-1000), for rows shorter than a warp's first pass (4, 12 values)
    and longer; the loss of the rows without NaN."""
    rows = 3000 if length <= 1024 else 400
    rng = np.random.default_rng(length + 1)
    x = rng.normal(0, 2, size=(rows, length)).astype(np.float32)
    x[5] = 0.0
    x[5, : length // 3] = -5.0
    x[5, length // 3] = -0.0
    x[6] = -0.0
    x[6, length - 1] = 0.0
    x[rows - 1, ::3] = -np.inf
    x[rows - 2, 1] = 1000.0
    x[rows - 2, length - 2] = -1000.0
    x[rows - 3] = 0.0
    tg = rng.integers(0, length, rows).astype(np.int64)
    tg[rows - 1] = 1  # a finite logit: the loss stays finite
    dtg = dev(backend, tg)
    loss, _, _, _ = backend.cross_entropy(dev(backend, x), dtg, rows, length)
    ref_loss, _ = port.cross_entropy(x, tg, 1.0)
    assert_rel(backend.download(loss), np.array([ref_loss]), RTOL, f"loss {length}")
    x[7, 0] = np.nan
    x[rows // 2, length - 1] = np.nan
    with np.errstate(invalid="ignore"):
        _, m, s, _ = backend.cross_entropy(dev(backend, x), dtg, rows, length)
        _, pm, ps = port.log_softmax(x, -1, stats=True)
    got_m, got_s = backend.download(m), backend.download(s)
    same = (got_m.view(np.uint32) == pm.view(np.uint32)) | (np.isnan(got_m) & np.isnan(pm))
    assert same.all(), np.flatnonzero(~same)[:10]
    assert got_m.view(np.uint32)[5] == np.float32(-0.0).view(np.uint32)
    assert np.array_equal(np.isnan(got_s), np.isnan(ps)), np.flatnonzero(np.isnan(got_s) != np.isnan(ps))[:10]
    ok = ~np.isnan(ps)
    np.testing.assert_allclose(got_s[ok], ps[ok], rtol=2e-6, atol=0)


def test_cross_entropy_known_answers(backend, golden):
    lg = np.zeros((2, 2), np.float32)
    loss, m, s, _ = backend.cross_entropy(dev(backend, lg), dev(backend, np.array([0, 1], np.int64)), 2, 2)
    assert abs(backend.download(loss)[0] - np.log(2.0)) < 1e-6
    up = dev(backend, np.ones(1, np.float32))
    dx = backend.cross_entropy_backward(dev(backend, lg), dev(backend, np.array([0, 1], np.int64)), m, s, up, 2, 2)
    assert backend.download(dx).reshape(2, 2).tolist() == golden["kat/ce/grad"].tolist()
    huge = np.array([[1000, 1001, 1002], [-1000, 0, 1000]], np.float32)
    dh, th = dev(backend, huge), dev(backend, np.array([2, 0], np.int64))
    _, m, s, _ = backend.cross_entropy(dh, th, 2, 3)
    dx = backend.download(backend.cross_entropy_backward(dh, th, m, s, up, 2, 3)).reshape(2, 3)
    assert np.all(np.isfinite(dx))
    assert_rel(dx, golden["kat/huge/ce_grad"], RTOL)


def test_golden_cfg4(backend, golden):
    lg, tg = C.cfg4(C.SMALL["cfg4"]["logits"])
    g = C.uniform(10, lg.shape, -1.0, 1.0)
    r, c = lg.shape
    dlg, dg = dev(backend, lg), dev(backend, g)
    for name, log in (("softmax", False), ("log_softmax", True)):
        y, m, s = backend.softmax(dlg, r, c, 1, log=log)
        assert_rel(backend.download(y).reshape(lg.shape), golden[f"cfg4/{name}/out"], RTOL, name)
        gx = backend.softmax_backward(dlg, m, s, dg, r, c, 1, log=log)
        assert_rel(backend.download(gx).reshape(lg.shape), golden[f"cfg4/{name}/dx"], RTOL, name, scale=1.0)
    dtg = dev(backend, tg)
    loss, m, s, _ = backend.cross_entropy(dlg, dtg, r, c)
    assert_rel(backend.download(loss), golden["cfg4/ce/loss"].reshape(1), RTOL)
    dx = backend.cross_entropy_backward(dlg, dtg, m, s, dev(backend, np.ones(1, np.float32)), r, c)
    assert_rel(backend.download(dx).reshape(lg.shape), golden["cfg4/ce/dx"], RTOL)


def test_cross_entropy_bad_target_fails_at_sync(backend):
    lg = dev(backend, np.zeros((2, 3), np.float32))
    tg = dev(backend, np.array([0, 3], np.int64))
    backend.cross_entropy(lg, tg, 2, 3)
    with pytest.raises((IndexError, RuntimeError)):
        backend.synchronize()
    backend.synchronize()  # the error was consumed; the device stays usable
    ok = backend.cross_entropy(lg, dev(backend, np.array([0, 2], np.int64)), 2, 3)[0]
    assert abs(backend.download(ok)[0] - np.log(3.0)) < 1e-6

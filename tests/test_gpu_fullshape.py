"""GPU parity at the FULL shapes of benchmark configurations 2-5, through the C
ABI, against the CPU oracle (the reference's CPU path restated) and numpy's
IEEE float32 arithmetic.

These are the shapes bench.py times, so the kernels and the dispatch choices
they exercise (chunked streams at 2^28 elements, the 8192-row column split of
axis-0 reductions, 65536 vocabulary rows, the 2^32-element strided broadcast
and its one-pass backward) are the ones the measured numbers come from.

The oracle runs on the host in row (or leading-index) slices on a thread
pool: rows are independent for every row-wise op, elementwise ops are
independent per element, and a column reduction is cut into column blocks.
Host memory stays bounded by the slices in flight; the device holds the full
tensors. Tolerance classes (written in tests/_util.py): bit-exact for add,
sub, mul, div, neg, relu, max, argmax and every backward rule given the same
saved tensors; <= 2 ulp for exp, log, sigmoid; relative 1e-5 (scaled by
sqrt(n) * rms for sums) for sums, means, softmax family and cross-entropy.

Inputs: configurations 2, 3 and 5's operands come from numpy default_rng with
the benchmark table's seeds; configuration 4's logits and targets and the
dense upstream gradients of 4 and 5 are drawn on the device with torch's
seeded generator (the same distributions), which keeps 8-17 GB arrays off the
host -- the oracle downloads the slices it checks."""
from __future__ import annotations

import ctypes
import os
from collections import deque
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import _cases as C
import oracle
from _util import assert_bitexact, assert_rel, assert_sum_close, assert_ulp
from vectorcore_b200 import _abi
from vectorcore_b200 import backend as B

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

WORKERS = max(2, min(16, os.cpu_count() or 4))
RTOL = 1e-5


# ---- helpers -----------------------------------------------------------------
def dl(storage, start, count, dtype=np.float32):
    """Download `count` elements of `storage` starting at element `start`."""
    dtype = np.dtype(dtype)
    out = np.empty(count, dtype)
    _abi.call("vc_cuda_download", ctypes.c_void_p(out.ctypes.data),
              ctypes.c_void_p(storage.ptr + start * dtype.itemsize), ctypes.c_size_t(out.nbytes))
    return out


def pipelined(jobs, work, in_flight=None):
    """Run work(*args) on the pool for every args the generator `jobs` yields.
    The generator runs on this thread (it does the downloads, which are
    serialised by the library anyway); at most `in_flight` jobs are queued so
    host memory stays bounded. Returns the results in job order."""
    in_flight = in_flight or WORKERS + 2
    results, pending = [], deque()
    with ThreadPoolExecutor(WORKERS) as pool:
        for args in jobs:
            pending.append(pool.submit(work, *args))
            while len(pending) >= in_flight:
                results.append(pending.popleft().result())
        while pending:
            results.append(pending.popleft().result())
    return results


def chunks(total, step):
    for lo in range(0, total, step):
        yield lo, min(total, lo + step)


def compare_flat(got, expected_fn, kind, what, step=1 << 24):
    """got: a host array of n elements; expected_fn(lo, hi) -> expected slice."""
    got = got.reshape(-1)

    def work(lo, hi):
        exp = expected_fn(lo, hi)
        if kind == "exact":
            assert_bitexact(got[lo:hi], exp, f"{what} [{lo}:{hi})")
            return 0
        return assert_ulp(got[lo:hi], exp, what=f"{what} [{lo}:{hi})")

    return max(pipelined(((lo, hi) for lo, hi in chunks(got.size, step)), work))


def from_torch(be, t):
    """Copy a torch CUDA tensor into a pool buffer of the library (set-up)."""
    import torch

    torch.cuda.synchronize()
    s = be.allocate(t.numel(), np.float32 if t.dtype.is_floating_point else np.int64)
    _abi.call("vc_cuda_copy", ctypes.c_void_p(s.ptr), ctypes.c_void_p(t.data_ptr()),
              ctypes.c_size_t(t.numel() * t.element_size()))
    be.synchronize()
    return s


@pytest.fixture
def trimmed(backend):
    """Give the pool's cached blocks back to the driver after a full-shape
    test (the next configuration's tensors have other sizes)."""
    yield backend
    backend.synchronize()
    _abi.call("vc_cuda_pool_trim")
    try:
        import torch

        torch.cuda.empty_cache()
    except Exception:
        pass


# ---- configuration 2: same-shape sweep on [16384, 16384] ------------------------------
def test_cfg2_full_shape(trimmed, port):
    be = trimmed
    shape = C.CFG2["a"]
    n = shape[0] * shape[1]
    a, b, g = (v.reshape(-1) for v in C.cfg2(shape))
    s = a - np.float32(1.0)  # signed input for neg / relu / sigmoid (bench.py's a - 1)
    da_, db_, dg_ = be.upload(a), be.upload(b), be.upload(g)
    ds = be.binary_scalar(da_, n, 1.0, B.SUB)
    compare_flat(be.download(ds), lambda lo, hi: s[lo:hi], "exact", "a - 1")

    def fwd(op):
        return be.download(be.binary(da_, shape, None, db_, shape, None, shape, op))

    compare_flat(fwd(B.ADD), lambda lo, hi: a[lo:hi] + b[lo:hi], "exact", "add")
    compare_flat(fwd(B.SUB), lambda lo, hi: a[lo:hi] - b[lo:hi], "exact", "sub")
    compare_flat(fwd(B.MUL), lambda lo, hi: a[lo:hi] * b[lo:hi], "exact", "mul")
    compare_flat(fwd(B.DIV), lambda lo, hi: a[lo:hi] / b[lo:hi], "exact", "div")
    compare_flat(be.download(be.unary(ds, n, B.NEG)), lambda lo, hi: -s[lo:hi], "exact", "neg")
    compare_flat(be.download(be.unary(ds, n, B.RELU)), lambda lo, hi: port.unary(oracle.RELU, s[lo:hi]),
                 "exact", "relu")
    compare_flat(be.download(be.binary_scalar(da_, n, 0.5, B.MUL)), lambda lo, hi: a[lo:hi] * np.float32(0.5),
                 "exact", "a * 0.5")
    y_exp_d = be.unary(da_, n, B.EXP)
    y_exp = be.download(y_exp_d)
    compare_flat(y_exp, lambda lo, hi: port.unary(oracle.EXP, a[lo:hi]), "ulp", "exp")
    compare_flat(be.download(be.unary(da_, n, B.LOG)), lambda lo, hi: port.unary(oracle.LOG, a[lo:hi]),
                 "ulp", "log")
    y_sig_d = be.unary(ds, n, B.SIGMOID)
    y_sig = be.download(y_sig_d)
    compare_flat(y_sig, lambda lo, hi: port.unary(oracle.SIGMOID, s[lo:hi]), "ulp", "sigmoid")

    # backward with the dense upstream g (same-shape operands: sum_to_shape is the identity)
    def bwd(op):
        ga, gb = be.binary_backward(op, da_, shape, db_, shape, dg_, shape)
        return be.download(ga), be.download(gb)

    ga, gb = bwd(B.ADD)
    compare_flat(ga, lambda lo, hi: g[lo:hi], "exact", "add da")
    compare_flat(gb, lambda lo, hi: g[lo:hi], "exact", "add db")
    ga, gb = bwd(B.SUB)
    compare_flat(ga, lambda lo, hi: g[lo:hi], "exact", "sub da")
    compare_flat(gb, lambda lo, hi: -g[lo:hi], "exact", "sub db")
    ga, gb = bwd(B.MUL)
    compare_flat(ga, lambda lo, hi: g[lo:hi] * b[lo:hi], "exact", "mul da")
    compare_flat(gb, lambda lo, hi: g[lo:hi] * a[lo:hi], "exact", "mul db")
    ga, gb = bwd(B.DIV)
    compare_flat(ga, lambda lo, hi: g[lo:hi] / b[lo:hi], "exact", "div da")
    compare_flat(gb, lambda lo, hi: -(g[lo:hi] * a[lo:hi]) / (b[lo:hi] * b[lo:hi]), "exact", "div db")
    del ga, gb
    compare_flat(be.download(be.unary_backward(B.NEG, None, None, dg_, n)), lambda lo, hi: -g[lo:hi],
                 "exact", "neg bwd")
    compare_flat(be.download(be.unary_backward(B.EXP, None, y_exp_d, dg_, n)),
                 lambda lo, hi: g[lo:hi] * y_exp[lo:hi], "exact", "exp bwd")
    compare_flat(be.download(be.unary_backward(B.LOG, da_, None, dg_, n)), lambda lo, hi: g[lo:hi] / a[lo:hi],
                 "exact", "log bwd")
    compare_flat(be.download(be.unary_backward(B.RELU, ds, None, dg_, n)),
                 lambda lo, hi: port.unary_backward_saved(oracle.RELU, s[lo:hi], s[lo:hi], g[lo:hi]),
                 "exact", "relu bwd")
    compare_flat(be.download(be.unary_backward(B.SIGMOID, None, y_sig_d, dg_, n)),
                 lambda lo, hi: (g[lo:hi] * y_sig[lo:hi]) * (np.float32(1.0) - y_sig[lo:hi]), "exact", "sigmoid bwd")
    compare_flat(be.download(be.binary_scalar(dg_, n, 0.5, B.MUL)), lambda lo, hi: g[lo:hi] * np.float32(0.5),
                 "exact", "a * 0.5 bwd")


# ---- configuration 3: reductions of [8192, 32768] -----------------------------------------
def test_cfg3_full_shape(trimmed, port):
    be = trimmed
    rows, cols = C.CFG3["x"]
    n = rows * cols
    x = C.cfg3()
    g1 = C.uniform(10, (rows,), -1.0, 1.0)  # upstream of the axis-1 reductions
    g0 = C.uniform(12, (cols,), -1.0, 1.0)  # upstream of the axis-0 reductions
    dx = be.upload(x)
    dg1, dg0 = be.upload(g1), be.upload(g0)

    # axis 1 (outer = rows, length = cols, inner = 1): rows are independent
    s1 = be.download(be.reduce_axis(dx, rows, cols, 1, B.REDUCE_SUM))
    m1 = be.download(be.reduce_axis(dx, rows, cols, 1, B.REDUCE_MEAN))
    v1d, i1d = be.reduce_axis(dx, rows, cols, 1, B.REDUCE_MAX, want_index=True)
    v1, i1 = be.download(v1d), be.download(i1d)
    a1 = be.download(be.reduce_axis(dx, rows, cols, 1, B.REDUCE_ARGMAX))

    def rows_work(lo, hi):
        xc = x[lo:hi]
        r = hi - lo
        assert_sum_close(s1[lo:hi], port.reduce_axis(oracle.SUM, xc, r, cols, 1), cols, 1.0, what="sum axis 1")
        assert_sum_close(m1[lo:hi], port.reduce_op("mean", xc, 1)[0], cols, 1.0 / cols, what="mean axis 1")
        assert_bitexact(v1[lo:hi], port.reduce_axis(oracle.MAX, xc, r, cols, 1), "max axis 1")
        assert np.array_equal(i1[lo:hi], port.argmax_i64(xc, r, cols, 1)), "argmax (int64) axis 1"
        assert_bitexact(a1[lo:hi], port.reduce_axis(oracle.ARGMAX, xc, r, cols, 1), "argmax (float) axis 1")

    pipelined(chunks(rows, 256), rows_work)

    # axis 0 (outer = 1, length = rows, inner = cols): the column split kernels
    s0 = be.download(be.reduce_axis(dx, 1, rows, cols, B.REDUCE_SUM))
    m0 = be.download(be.reduce_axis(dx, 1, rows, cols, B.REDUCE_MEAN))
    v0d, i0d = be.reduce_axis(dx, 1, rows, cols, B.REDUCE_MAX, want_index=True)
    v0, i0 = be.download(v0d), be.download(i0d)

    def cols_work(lo, hi):
        xc = np.ascontiguousarray(x[:, lo:hi])
        w = hi - lo
        assert_sum_close(s0[lo:hi], port.reduce_axis(oracle.SUM, xc, 1, rows, w), rows, 1.0, what="sum axis 0")
        assert_sum_close(m0[lo:hi], port.reduce_op("mean", xc, 0)[0], rows, 1.0 / rows, what="mean axis 0")
        assert_bitexact(v0[lo:hi], port.reduce_axis(oracle.MAX, xc, 1, rows, w), "max axis 0")
        assert np.array_equal(i0[lo:hi], port.argmax_i64(xc, 1, rows, w)), "argmax axis 0"

    pipelined(chunks(cols, 1024), cols_work)

    # full reductions
    assert_sum_close(be.download(be.reduce_sum(dx, n))[0], port.sum(x), n, 1.0, what="full sum")
    assert_sum_close(be.download(be.reduce_all(dx, n, B.REDUCE_MEAN))[0], port.reduce_op("mean", x, None)[0],
                     n, 1.0 / n, what="full mean")
    vf, jf = be.reduce_all(dx, n, B.REDUCE_MAX, want_index=True)
    flat = x.reshape(-1)
    assert_bitexact(be.download(vf), port.reduce_axis(oracle.MAX, flat, 1, n, 1), "full max")
    assert be.download(jf)[0] == port.argmax_i64(flat, 1, n, 1)[0]

    # backward passes: broadcast of g (+0) for sum, g / length (+0) for mean,
    # the scatter of g at the argmax for max
    def rows_bwd(name, got_d, fn):
        got = be.download(got_d).reshape(rows, cols)
        pipelined(chunks(rows, 512), lambda lo, hi: assert_bitexact(got[lo:hi], fn(lo, hi), f"{name} [{lo}:{hi})"))

    zero = np.float32(0.0)
    rows_bwd("sum axis 1 bwd", be.reduce_axis_backward(B.REDUCE_SUM, dg1, None, rows, cols, 1),
             lambda lo, hi: np.repeat((g1[lo:hi] + zero)[:, None], cols, axis=1))
    rows_bwd("mean axis 1 bwd", be.reduce_axis_backward(B.REDUCE_MEAN, dg1, None, rows, cols, 1),
             lambda lo, hi: np.repeat((g1[lo:hi] / np.float32(cols) + zero)[:, None], cols, axis=1))

    def scatter1(lo, hi):
        out = np.zeros((hi - lo, cols), np.float32)
        out[np.arange(hi - lo), i1[lo:hi]] = g1[lo:hi]
        return out

    rows_bwd("max axis 1 bwd", be.reduce_axis_backward(B.REDUCE_MAX, dg1, i1d, rows, cols, 1), scatter1)
    rows_bwd("sum axis 0 bwd", be.reduce_axis_backward(B.REDUCE_SUM, dg0, None, 1, rows, cols),
             lambda lo, hi: np.repeat((g0 + zero)[None, :], hi - lo, axis=0))

    def scatter0(lo, hi):
        out = np.zeros((hi - lo, cols), np.float32)
        hit = (i0 >= lo) & (i0 < hi)
        out[i0[hit] - lo, np.flatnonzero(hit)] = g0[hit]
        return out

    rows_bwd("max axis 0 bwd", be.reduce_axis_backward(B.REDUCE_MAX, dg0, i0d, 1, rows, cols), scatter0)
    one = be.upload(np.ones(1, np.float32))
    rows_bwd("full sum bwd", be.broadcast_to(one, (), (rows, cols)),
             lambda lo, hi: np.ones((hi - lo, cols), np.float32))
    inv = be.upload(np.array([np.float32(1.0) / np.float32(n)], np.float32))
    rows_bwd("full mean bwd", be.broadcast_to(inv, (), (rows, cols)),
             lambda lo, hi: np.full((hi - lo, cols), np.float32(1.0) / np.float32(n), np.float32))


# ---- configuration 4: softmax family and cross-entropy on [65536, 32000] -----------------
def test_cfg4_full_shape(trimmed, port):
    import torch

    be = trimmed
    rows, cols = C.CFG4["logits"]
    gen = torch.Generator(device="cuda").manual_seed(5)
    lg = from_torch(be, torch.randn(rows, cols, device="cuda", generator=gen) * 2)
    tg = from_torch(be, torch.randint(0, cols, (rows,), device="cuda", generator=gen, dtype=torch.int64))
    gg = from_torch(be, torch.rand(rows, cols, device="cuda", generator=gen) * 2 - 1)
    torch.cuda.empty_cache()

    y_sm, m_sm, s_sm = be.softmax(lg, rows, cols, 1, log=False)
    y_lsm, m_lsm, s_lsm = be.softmax(lg, rows, cols, 1, log=True)
    loss, m_ce, s_ce, _ = be.cross_entropy(lg, tg, rows, cols)
    one = be.upload(np.ones(1, np.float32))
    dlg = be.cross_entropy_backward(lg, tg, m_ce, s_ce, one, rows, cols)
    dx_sm = be.softmax_backward(lg, m_sm, s_sm, gg, rows, cols, 1, log=False)
    dx_lsm = be.softmax_backward(lg, m_lsm, s_lsm, gg, rows, cols, 1, log=True)
    stats = {k: be.download(v) for k, v in (("m_sm", m_sm), ("s_sm", s_sm), ("m_lsm", m_lsm), ("s_lsm", s_lsm),
                                             ("m_ce", m_ce), ("s_ce", s_ce))}
    targets = be.download(tg)
    got_loss = be.download(loss)[0]

    step = 256  # a power of two dividing the batch: the chunk's CE upstream b/B is exact

    def jobs():
        for lo, hi in chunks(rows, step):
            e0, cnt = lo * cols, (hi - lo) * cols
            yield (lo, hi, dl(lg, e0, cnt), dl(gg, e0, cnt), dl(y_sm, e0, cnt), dl(y_lsm, e0, cnt),
                   dl(dlg, e0, cnt), dl(dx_sm, e0, cnt), dl(dx_lsm, e0, cnt))

    def work(lo, hi, x, g, ysm, ylsm, dce, dsm, dlsm):
        r = hi - lo
        x, g = x.reshape(r, cols), g.reshape(r, cols)
        ref_lsm, pm, ps = port.log_softmax(x, -1, stats=True)
        assert_rel(ylsm.reshape(r, cols), ref_lsm, RTOL, f"log_softmax rows [{lo}:{hi})")
        assert_rel(ysm.reshape(r, cols), port.softmax(x, -1), RTOL, f"softmax rows [{lo}:{hi})")
        for k in ("m_sm", "m_lsm", "m_ce"):
            assert_bitexact(stats[k][lo:hi], pm, f"{k} rows [{lo}:{hi})")  # the row max is exact
        for k in ("s_sm", "s_lsm", "s_ce"):
            np.testing.assert_allclose(stats[k][lo:hi], ps, rtol=2e-6, atol=0, err_msg=f"{k} [{lo}:{hi})")
        # the chunk's mean loss with upstream r / rows: d(loss)/d(sum) is then
        # -(1 / rows) exactly, as for the whole batch
        chunk_loss, ref_dce = port.cross_entropy(x, targets[lo:hi], upstream=r / rows)
        assert_rel(dce.reshape(r, cols), ref_dce, RTOL, f"dlogits rows [{lo}:{hi})")
        assert_rel(dsm.reshape(r, cols), port.softmax_backward(x, g, -1), RTOL, f"softmax bwd [{lo}:{hi})",
                   scale=1.0)
        assert_rel(dlsm.reshape(r, cols), port.log_softmax_backward(x, g, -1), RTOL, f"log_softmax bwd [{lo}:{hi})",
                   scale=1.0)
        return -float(chunk_loss) * r  # the chunk's float sum of log-probabilities at the targets

    sums = pipelined(jobs(), work, in_flight=WORKERS)
    ref_loss = -sum(sums) / rows  # chunk sums recombined in row order
    assert abs(got_loss - ref_loss) <= RTOL * abs(ref_loss), (got_loss, ref_loss)


# ---- configuration 5: strided broadcast multiply to [64, 128, 512, 1024] -----------------
def test_cfg5_full_shape(trimmed):
    import torch

    be = trimmed
    a_shape, b_shape = C.CFG5["a"], C.CFG5["b"]
    P, Q, R, L = a_shape[0], b_shape[1], a_shape[2], a_shape[3]
    o_shape = (P, Q, R, L)
    n = P * Q * R * L
    assert n == 1 << 32  # past 2^31 and 2^32 - 1: 64-bit offsets everywhere
    a, b = C.cfg5()
    da_, db_ = be.upload(a), be.upload(b)
    b0 = b[0]  # [Q, 1, L]
    per = Q * R * L  # elements of one leading index

    out = be.binary(da_, a_shape, None, db_, b_shape, None, o_shape, B.MUL)
    total = be.download(be.reduce_sum(out, n))[0]

    def fwd_jobs():
        for i in range(P):
            yield i, dl(out, i * per, per)

    def fwd_work(i, got):
        exp = a[i] * b0  # [1,R,L] * [Q,1,L] -> [Q,R,L], IEEE float32 products
        assert_bitexact(got.reshape(Q, R, L), exp, f"a * b at leading index {i}")
        e = exp.reshape(-1)
        return float(np.sum(e, dtype=np.float64)), float(np.dot(e, e))

    res = pipelined(fwd_jobs(), fwd_work, in_flight=8)
    ref_total = sum(r[0] for r in res)
    rms = float(np.sqrt(sum(r[1] for r in res) / n))
    assert_sum_close(total, ref_total, n, rms, what="out.sum() over 2^32 elements")
    del out

    # backward, dense upstream g over the output shape: da = sum over axis 1 of
    # g * b, db = sum over axes 0 and 2 of g * a (the reference rounds db after
    # each axis; the fused kernel once: both within the sum class)
    gen = torch.Generator(device="cuda").manual_seed(11)
    gd = from_torch(be, torch.rand(*o_shape, device="cuda", generator=gen) * 2 - 1)
    torch.cuda.empty_cache()
    ga, gb = be.binary_backward(B.MUL, da_, a_shape, db_, b_shape, gd, o_shape)
    got_da = be.download(ga).reshape(P, R, L)
    got_db = be.download(gb).reshape(Q, L)

    def bwd_jobs():
        for i in range(P):
            yield i, dl(gd, i * per, per).reshape(Q, R, L)

    def bwd_work(i, g):
        gb_ = g * b0  # the reference's g * b, rounded to float
        da_i = np.sum(gb_, axis=0, dtype=np.float64)  # [R, L]
        v = gb_.reshape(-1)
        assert_sum_close(got_da[i], da_i.astype(np.float32), Q, float(np.sqrt(np.dot(v, v) / v.size)),
                         what=f"da at leading index {i}")
        del gb_, v
        ga_ = g * a[i]  # [Q,R,L]
        v = ga_.reshape(-1)
        return np.sum(ga_, axis=1, dtype=np.float64), float(np.dot(v, v) / v.size)  # [Q, L]

    parts = pipelined(bwd_jobs(), bwd_work, in_flight=8)
    db_ref = np.zeros((Q, L), np.float64)
    for p, _ in parts:  # combined in leading-index order
        db_ref += p
    rms_db = float(np.sqrt(np.mean([q for _, q in parts])))
    assert_sum_close(got_db, db_ref, P * R, rms_db, what="db (axes 0 and 2)")
    del gd

    # backward of out.sum(): the upstream is the 0-d 1.0 broadcast (compact path)
    one = be.upload(np.ones(1, np.float32))
    ga, gb = be.binary_backward(B.MUL, da_, a_shape, db_, b_shape, one, ())
    da_ref = np.sum(b0.reshape(Q, L), axis=0, dtype=np.float64)  # [L], the same for every (i, r)
    got_da = be.download(ga).reshape(P * R, L)
    rms_b = float(np.sqrt(np.mean(b0.astype(np.float64) ** 2)))
    for lo, hi in chunks(P * R, 4096):
        assert_sum_close(got_da[lo:hi], np.broadcast_to(da_ref, (hi - lo, L)), Q, rms_b, what="da of out.sum()")
    db_ref = np.sum(a.reshape(P * R, L), axis=0, dtype=np.float64)  # [L], the same for every q
    rms_a = float(np.sqrt(np.mean(a.astype(np.float64) ** 2)))
    assert_sum_close(be.download(gb).reshape(Q, L), np.broadcast_to(db_ref, (Q, L)), P * R, rms_a,
                     what="db of out.sum()")

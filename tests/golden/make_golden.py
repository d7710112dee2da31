"""Generate tests/golden/golden.npz by running the REFERENCE itself.

Usage (in a container that has the reference checkout):
    make -C oracle ref            # builds oracle/_ref/vectorcore*.so from the
                                  # reference's unmodified sources
    python tests/golden/make_golden.py

Every value in the fixture is produced by the reference's own public Python
API (``import vectorcore``, python/bindings.cpp) on the CPU device:

* ``kat/...``   the known-answer cases of the reference's own test suites
  (tests/cpp/test_vectorcore.cpp and tests/python/*.py), recomputed;
* ``cfgN/...``  seeded inputs of the five benchmark configurations at small
  shapes (tests/_cases.py: SMALL), and config 1 at its full shape.

Large bit-exact outputs are stored as a SHA-256 of their float32 bytes
(``.../sha256``) instead of the array. The fixture travels to the GPU box;
the reference does not.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle" / "_ref"))
sys.path.insert(0, str(ROOT / "tests"))

import vectorcore as vc  # noqa: E402  (the reference's module)
import _cases as C  # noqa: E402

OUT = Path(__file__).resolve().parent / "golden.npz"
G: dict[str, np.ndarray] = {}


def put(key, value):
    G[key] = np.asarray(value)


def sha(arr):
    return hashlib.sha256(np.ascontiguousarray(arr, np.float32).tobytes()).hexdigest()


def T(values, rg=False):
    return vc.Tensor(np.asarray(values, np.float32), requires_grad=rg)


def kat():
    a = T([[1, 2], [3, 4]])
    b = T([[4, 3], [2, 1]])
    put("kat/ew/a", a.numpy()); put("kat/ew/b", b.numpy())
    put("kat/ew/add", (a + b).numpy()); put("kat/ew/sub", (a - b).numpy())
    put("kat/ew/mul", (a * b).numpy()); put("kat/ew/div", (a / b).numpy())
    put("kat/ew/neg", (-a).numpy())
    m = T([[1, 2, 3], [4, 5, 6]])
    put("kat/bcast/row", (m + T([10, 20, 30])).numpy())
    x = T([[1, 2, 3], [4, 5, 6]], True)
    bias = T([0.1, 0.2, 0.3], True)
    (x + bias).sum().backward()
    put("kat/bias_grad/dx", x.grad.numpy()); put("kat/bias_grad/db", bias.grad.numpy())
    x = T([[1, 5, 3], [4, 2, 6]])
    put("kat/axis/x", x.numpy())
    put("kat/axis/sum0", x.sum(0).numpy()); put("kat/axis/sum_m1_keep", x.sum(-1, True).numpy())
    put("kat/axis/mean1", x.mean(1).numpy()); put("kat/axis/max1", x.max(1).numpy())
    put("kat/axis/argmax1", x.argmax(1).numpy()); put("kat/axis/max_all", x.max().numpy())
    lg = T(np.zeros((2, 2)), True)
    loss = vc.cross_entropy(lg, [0, 1])
    loss.backward()
    put("kat/ce/loss", loss.numpy()); put("kat/ce/grad", lg.grad.numpy())
    put("kat/ties/argmax1", T([[1, 3, 3], [2, 2, 0]]).argmax(1).numpy())
    t = T([[1, 3, 3]], True)
    t.max(1).sum().backward()
    put("kat/ties/max_grad", t.grad.numpy())
    huge = np.array([[1000, 1001, 1002], [-1000, 0, 1000]], np.float32)
    t = T(huge, True)
    put("kat/huge/softmax", t.softmax(-1).numpy())
    vc.cross_entropy(t, [2, 0]).backward()
    put("kat/huge/ce_grad", t.grad.numpy())
    k = T([0.0, -0.0, 1.0], True)
    k.relu().sum().backward()
    put("kat/relu_kink/grad", k.grad.numpy())
    gx = T([[-1, 2, 3], [-4, 5, 6]], True)
    gb = T([0.5, 1.0, -2.0], True)
    (gx + gb).relu().sum().backward()
    put("kat/bias_relu/dx", gx.grad.numpy()); put("kat/bias_relu/db", gb.grad.numpy())


def cfg1(tag, shape, full_arrays):
    x_np, b_np = C.cfg1(shape)
    x, b = vc.Tensor(x_np, requires_grad=True), vc.Tensor(b_np, requires_grad=True)
    y = (x + b).relu()
    loss = y.sum()
    loss.backward()
    put(f"{tag}/loss", loss.numpy()); put(f"{tag}/db", b.grad.numpy())
    if full_arrays:
        put(f"{tag}/y", y.numpy()); put(f"{tag}/dx", x.grad.numpy())
    put(f"{tag}/y/sha256", sha(y.numpy())); put(f"{tag}/dx/sha256", sha(x.grad.numpy()))


def cfg2():
    a_np, b_np, g_np = C.cfg2(C.SMALL["cfg2"]["a"])
    binary = {"add": lambda p, q: p + q, "sub": lambda p, q: p - q,
              "mul": lambda p, q: p * q, "div": lambda p, q: p / q}
    for name, fn in binary.items():
        a, b = vc.Tensor(a_np, requires_grad=True), vc.Tensor(b_np, requires_grad=True)
        y = fn(a, b)
        y.backward(vc.Tensor(g_np))
        put(f"cfg2/{name}/out", y.numpy()); put(f"cfg2/{name}/da", a.grad.numpy())
        put(f"cfg2/{name}/db", b.grad.numpy())
    unary = {"neg": lambda p: -p, "exp": lambda p: p.exp(), "log": lambda p: p.log(),
             "relu": lambda p: p.relu(), "sigmoid": lambda p: p.sigmoid(),
             "scalar_mul": lambda p: p * 0.5}
    # relu/sigmoid/neg see signed inputs (a - 1 spans [-0.9, 1]).
    for name, fn in unary.items():
        src = a_np if name in ("exp", "log", "scalar_mul") else (a_np - np.float32(1.0))
        a = vc.Tensor(src, requires_grad=True)
        y = fn(a)
        y.backward(vc.Tensor(g_np))
        put(f"cfg2/{name}/x", src); put(f"cfg2/{name}/out", y.numpy())
        put(f"cfg2/{name}/dx", a.grad.numpy())


def cfg3():
    x_np = C.cfg3(C.SMALL["cfg3"]["x"])
    rng = np.random.default_rng(12)
    for name, axis, keep in [("sum1", 1, True), ("mean1", 1, True), ("max1", 1, True),
                             ("sum0", 0, False), ("max0", 0, False)]:
        x = vc.Tensor(x_np, requires_grad=True)
        fn = {"sum": x.sum, "mean": x.mean, "max": x.max}[name[:-1]]
        y = fn(axis, keep)
        g = rng.uniform(-1, 1, size=y.shape).astype(np.float32)
        y.backward(vc.Tensor(g))
        put(f"cfg3/{name}/out", y.numpy()); put(f"cfg3/{name}/g", g)
        put(f"cfg3/{name}/dx", x.grad.numpy())
    put("cfg3/argmax1/out", vc.Tensor(x_np).argmax(1, True).numpy())
    for name in ("sum", "mean"):
        x = vc.Tensor(x_np, requires_grad=True)
        y = x.sum() if name == "sum" else x.mean()
        y.backward()
        put(f"cfg3/{name}_all/out", y.numpy()); put(f"cfg3/{name}_all/dx/sha256", sha(x.grad.numpy()))


def cfg4():
    lg_np, tg = C.cfg4(C.SMALL["cfg4"]["logits"])
    g_np = C.uniform(10, lg_np.shape, -1.0, 1.0)
    put("cfg4/targets", tg)
    for name in ("softmax", "log_softmax"):
        x = vc.Tensor(lg_np, requires_grad=True)
        y = x.softmax(-1) if name == "softmax" else x.log_softmax(-1)
        y.backward(vc.Tensor(g_np))
        put(f"cfg4/{name}/out", y.numpy()); put(f"cfg4/{name}/dx", x.grad.numpy())
    x = vc.Tensor(lg_np, requires_grad=True)
    loss = vc.cross_entropy(x, tg)
    loss.backward()
    put("cfg4/ce/loss", loss.numpy()); put("cfg4/ce/dx", x.grad.numpy())


def cfg5():
    a_np, b_np = C.cfg5(C.SMALL["cfg5"]["a"], C.SMALL["cfg5"]["b"])
    a, b = vc.Tensor(a_np, requires_grad=True), vc.Tensor(b_np, requires_grad=True)
    out = a * b
    s = out.sum()
    s.backward()
    put("cfg5/out/sha256", sha(out.numpy())); put("cfg5/sum", s.numpy())
    put("cfg5/sum_bwd/da", a.grad.numpy()); put("cfg5/sum_bwd/db", b.grad.numpy())
    g_np = C.uniform(11, out.shape, -1.0, 1.0)
    a, b = vc.Tensor(a_np, requires_grad=True), vc.Tensor(b_np, requires_grad=True)
    (a * b).backward(vc.Tensor(g_np))
    put("cfg5/dense_bwd/da", a.grad.numpy()); put("cfg5/dense_bwd/db", b.grad.numpy())


def main():
    kat()
    cfg1("cfg1_small", C.SMALL["cfg1"]["x"], False)
    cfg1("cfg1_full", C.CFG1["x"], False)
    cfg2()
    cfg3()
    cfg4()
    cfg5()
    np.savez_compressed(OUT, **G)
    print(f"wrote {len(G)} arrays to {OUT} ({OUT.stat().st_size / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()

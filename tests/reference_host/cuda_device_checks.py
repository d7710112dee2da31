"""Checks of the `cuda` device inside the reference's own host.

Run by tests/test_gpu_reference_host.py in a child process whose PYTHONPATH
holds oracle/_ref/cuda_host (the reference built with its `cuda` device,
oracle/Makefile `host`): `import vectorcore` is then the reference's own
pybind11 module with CPU, Metal and CUDA devices. The file name keeps
pytest's default collection away from it (two builds of the module cannot
share one process).

The first group restates, for the CUDA device, what the reference's
Metal-only tests check for Metal (tests/python/test_performance_paths.py:
182-227, test_classifier_ops.py:165-196): queued execution in order without
a sync, in-place updates ordered after earlier readers, pool buffers reused
safely, synchronize(), sgd_step, the version-counter rule. The second group
compares the CUDA device's fused paths with the reference's CPU device of the
same module on the same inputs: bit-exact where the parity contract says so,
1e-5-class otherwise (tests/_util.py)."""
import numpy as np
import pytest
import vectorcore as vc

from _util import assert_bitexact, assert_rel, assert_sum_close, assert_ulp

pytestmark = pytest.mark.skipif(not vc.cuda_available(), reason="no CUDA device")

RTOL = 1e-5


def cpu_numpy(t):
    return t.to("cpu").numpy()


def both(x, rg=False):
    return vc.Tensor(x, requires_grad=rg), vc.Tensor(x, requires_grad=rg, device="cuda")


# ---- the device and its neighbours -------------------------------------------------
def test_cuda_is_a_third_device_and_metal_stays_metal():
    assert "B200" in vc.cuda_device_name()
    t = vc.Tensor([1.0, 2.0], device="cuda")
    assert t.device == "cuda"
    assert vc.Tensor([1.0]).device == "cpu"
    if not vc.metal_available():
        with pytest.raises(RuntimeError, match="Metal is unavailable"):
            vc.Tensor([1.0], device="metal")
    with pytest.raises(ValueError, match="cuda"):
        vc.Tensor([1.0], device="tpu")
    with pytest.raises(ValueError, match="device mismatch"):
        t + vc.Tensor([1.0, 2.0])
    np.testing.assert_array_equal(cpu_numpy(t * 2.0), [2.0, 4.0])


def test_to_round_trip_and_gradient_through_to():
    x = np.random.default_rng(1).normal(size=(37, 53)).astype(np.float32)
    c = vc.Tensor(x, requires_grad=True)
    g = c.to("cuda")
    assert g.device == "cuda"
    assert_bitexact(cpu_numpy(g), x)
    (g * 3.0).sum().backward()
    assert c.grad.device == "cpu"
    np.testing.assert_array_equal(c.grad.numpy(), np.full_like(x, 3.0))


# ---- asynchronous execution (the Metal-only tests, for CUDA) -------------------------
def test_long_dependency_chain_without_sync():
    x = vc.Tensor(np.zeros(1000, dtype=np.float32), device="cuda")
    for _ in range(2000):
        x = x + 1.0
    np.testing.assert_allclose(cpu_numpy(x), 2000.0)


def test_in_place_update_is_ordered():
    w = vc.Tensor(np.ones(256, dtype=np.float32), requires_grad=True, device="cuda")
    before = w * 2.0
    (w * 1.0).sum().backward()
    vc.sgd_step([w], 0.5)
    after = w * 2.0
    np.testing.assert_allclose(cpu_numpy(before), 2.0)
    np.testing.assert_allclose(cpu_numpy(after), 1.0)


def test_buffer_reuse_does_not_corrupt_results():
    rng = np.random.default_rng(7)
    expected, results = [], []
    for _ in range(200):
        size = int(rng.integers(1, 5000))
        data = rng.normal(size=size).astype(np.float32)
        t = vc.Tensor(data, device="cuda")
        tmp = (t * 3.0).relu()
        results.append((tmp - t).sum())
        expected.append(float((np.maximum(data * 3.0, 0) - data).astype(np.float64).sum()))
        del t, tmp
    for got, want in zip(results, expected):
        assert np.isclose(got.item(), want, rtol=1e-4, atol=1e-3)


def test_synchronize():
    vc.synchronize()
    y = vc.Tensor([1.0, 2.0], device="cuda") * 2.0
    vc.synchronize()
    np.testing.assert_allclose(cpu_numpy(y), [2.0, 4.0])


def test_sgd_on_cuda_matches_cpu():
    rng = np.random.default_rng(7)
    w_np = rng.normal(size=(3, 2)).astype(np.float32)
    x_np = rng.normal(size=(4, 3)).astype(np.float32)
    results = {}
    for device in ("cpu", "cuda"):
        w = vc.Tensor(w_np, requires_grad=True, device=device)
        x = vc.Tensor(x_np, device=device)
        for _ in range(5):
            loss = vc.cross_entropy(x @ w, [0, 1, 1, 0])
            loss.backward()
            vc.sgd_step([w], 0.5)
            vc.zero_grad([w])
        results[device] = cpu_numpy(w)
    np.testing.assert_allclose(results["cuda"], results["cpu"], rtol=1e-4, atol=1e-5)


def test_sgd_bumps_version_and_is_detected():
    w = vc.Tensor([[1.0], [2.0]], requires_grad=True, device="cuda")
    x = vc.Tensor([[1.0, 1.0]], device="cuda")
    stale = (w * w).sum()
    (x @ w).sum().backward()
    before = w._version
    vc.sgd_step([w], 0.1)
    assert w._version == before + 1
    with pytest.raises(RuntimeError, match="modified in place"):
        stale.backward()


# ---- the fused paths against the reference's CPU device ------------------------------
@pytest.mark.parametrize("a_shape,b_shape", [((64, 1, 32, 256), (1, 16, 1, 256)), ((300, 70), (70,)),
                                             ((40, 50, 1), (50, 7)), ((128, 96), (128, 96)), ((5, 6), ())])
def test_broadcast_gradients(a_shape, b_shape):
    rng = np.random.default_rng(len(a_shape) * 7 + len(b_shape))
    a = rng.uniform(0.5, 2.0, size=a_shape).astype(np.float32)
    b = rng.uniform(0.5, 2.0, size=b_shape).astype(np.float32)
    ops = (("add", lambda x, y: x + y), ("sub", lambda x, y: x - y), ("mul", lambda x, y: x * y),
           ("div", lambda x, y: x / y))
    for op, fn in ops:
        grads = {}
        for device in ("cpu", "cuda"):
            ta = vc.Tensor(a, requires_grad=True, device=device)
            tb = vc.Tensor(b, requires_grad=True, device=device)
            out = fn(ta, tb)
            g = vc.Tensor(rng_g(out.shape), device=device)
            out.backward(g)
            grads[device] = (cpu_numpy(out), cpu_numpy(ta.grad), cpu_numpy(tb.grad))
        assert_bitexact(grads["cuda"][0], grads["cpu"][0], "forward")
        g = rng_g(grads["cpu"][0].shape)
        terms = {"add": (g, g), "sub": (g, g), "mul": (g * b, g * a), "div": (g / b, g * a / (b * b))}[op]
        for k, name in ((1, "da"), (2, "db")):
            ref = grads["cpu"][k]
            n = max(1, int(np.prod(grads["cpu"][0].shape)) // max(1, ref.size))
            if n == 1:
                assert_bitexact(grads["cuda"][k], ref, f"{op} {name}")  # no reduction: the same float ops
            else:
                # a reduction of n terms: the reference rounds after each reduced
                # axis, the fused kernel once -- the sum tolerance class
                rms = float(np.sqrt(np.mean(np.square(terms[k - 1], dtype=np.float64))))
                assert_sum_close(grads["cuda"][k], ref, n, rms, what=f"{op} {name}")


def rng_g(shape):
    return np.random.default_rng(99).uniform(-1, 1, size=tuple(shape)).astype(np.float32)


def test_unary_gradients_bitexact():
    x = np.random.default_rng(3).uniform(-4, 4, size=(300, 257)).astype(np.float32)
    g = rng_g(x.shape)
    for fn, exact in ((lambda t: t.relu(), True), (lambda t: t.sigmoid(), False), (lambda t: -t, True),
                      (lambda t: t.exp(), False)):
        res = {}
        for device in ("cpu", "cuda"):
            t = vc.Tensor(x, requires_grad=True, device=device)
            y = fn(t)
            y.backward(vc.Tensor(g, device=device))
            res[device] = cpu_numpy(y), cpu_numpy(t.grad)
        if exact:
            assert_bitexact(res["cuda"][0], res["cpu"][0])
            assert_bitexact(res["cuda"][1], res["cpu"][1])
        else:
            assert_ulp(res["cuda"][0], res["cpu"][0], 2)
            assert_rel(res["cuda"][1], res["cpu"][1], RTOL, scale=1.0)


def test_reductions_and_max_gradient_ties():
    x = np.random.default_rng(5).normal(size=(64, 500, 33)).astype(np.float32)
    x[3, 10:20, 4] = 9.0  # ties: the first index takes the gradient
    for axis in (0, 1, 2, -1):
        res = {}
        for device in ("cpu", "cuda"):
            t = vc.Tensor(x, requires_grad=True, device=device)
            m = t.max(axis, keepdim=True)
            s = t.sum(axis)
            (m.sum() + s.sum()).backward()
            res[device] = (cpu_numpy(m), cpu_numpy(t.argmax(axis)), cpu_numpy(s), cpu_numpy(t.grad),
                           cpu_numpy(t.mean(axis)))
        assert_bitexact(res["cuda"][0], res["cpu"][0], "max")
        assert_bitexact(res["cuda"][1], res["cpu"][1], "argmax")
        assert_rel(res["cuda"][2], res["cpu"][2], RTOL, "sum")
        assert_bitexact(res["cuda"][3], res["cpu"][3], "max + sum gradient")
        assert_rel(res["cuda"][4], res["cpu"][4], RTOL, "mean")
    full = {d: vc.Tensor(x, device=d).sum().item() for d in ("cpu", "cuda")}
    assert abs(full["cuda"] - full["cpu"]) <= RTOL * abs(full["cpu"]) + 1e-3


@pytest.mark.parametrize("shape,axis", [((64, 1000), -1), ((8, 32000), 1), ((3, 7, 9), 1), ((37, 45), 0)])
def test_softmax_family_fused(shape, axis):
    x = (np.random.default_rng(11).normal(size=shape) * 2).astype(np.float32)
    g = rng_g(shape)
    for name in ("softmax", "log_softmax"):
        res = {}
        for device in ("cpu", "cuda"):
            t = vc.Tensor(x, requires_grad=True, device=device)
            y = getattr(t, name)(axis)
            y.backward(vc.Tensor(g, device=device))
            res[device] = cpu_numpy(y), cpu_numpy(t.grad)
        assert_rel(res["cuda"][0], res["cpu"][0], RTOL, name)
        assert_rel(res["cuda"][1], res["cpu"][1], RTOL, name + " backward", scale=1.0)


def test_cross_entropy_without_a_mask():
    rng = np.random.default_rng(13)
    logits = (rng.normal(size=(256, 32000)) * 2).astype(np.float32)
    targets = [int(v) for v in rng.integers(0, 32000, 256)]
    res = {}
    for device in ("cpu", "cuda"):
        t = vc.Tensor(logits, requires_grad=True, device=device)
        loss = vc.cross_entropy(t, targets)
        loss.backward()
        res[device] = loss.item(), cpu_numpy(t.grad)
    assert abs(res["cuda"][0] - res["cpu"][0]) <= RTOL * abs(res["cpu"][0])
    assert_rel(res["cuda"][1], res["cpu"][1], RTOL, "dlogits")
    bad = vc.Tensor(logits[:2], device="cuda")
    with pytest.raises(IndexError, match="out of range"):
        vc.cross_entropy(bad, [0, 32000])
    with pytest.raises(ValueError, match="targets"):
        vc.cross_entropy(bad, [0])


def test_bias_relu_sum_chain():
    x = np.random.default_rng(0).uniform(-1, 1, size=(1024, 4096)).astype(np.float32)
    b = np.random.default_rng(1).normal(size=4096).astype(np.float32)
    res = {}
    for device in ("cpu", "cuda"):
        tx = vc.Tensor(x, requires_grad=True, device=device)
        tb = vc.Tensor(b, requires_grad=True, device=device)
        loss = (tx + tb).relu().sum()
        loss.backward()
        res[device] = loss.item(), cpu_numpy(tx.grad), cpu_numpy(tb.grad)
    assert abs(res["cuda"][0] - res["cpu"][0]) <= RTOL * abs(res["cpu"][0])
    assert_bitexact(res["cuda"][1], res["cpu"][1], "dx")
    assert_rel(res["cuda"][2], res["cpu"][2], RTOL, "db")


def test_training_loop_matches_cpu():
    rng = np.random.default_rng(21)
    x_np = rng.normal(size=(128, 20)).astype(np.float32)
    y = [int(v) for v in rng.integers(0, 5, 128)]
    losses = {}
    for device in ("cpu", "cuda"):
        layer1, layer2 = vc.Linear(20, 32, seed=1), vc.Linear(32, 5, seed=2)
        params = [layer1.weight, layer1.bias, layer2.weight, layer2.bias]
        params = [p.to(device).detach() for p in params]
        for p in params:
            p.requires_grad = True
        x = vc.Tensor(x_np, device=device)
        hist = []
        for _ in range(50):
            h = (x @ params[0] + params[1]).relu()
            loss = vc.cross_entropy(h @ params[2] + params[3], y)
            loss.backward()
            vc.sgd_step(params, 0.1)
            vc.zero_grad(params)
            hist.append(loss.item())
        losses[device] = hist
    np.testing.assert_allclose(losses["cuda"], losses["cpu"], rtol=2e-3)
    assert losses["cuda"][-1] < losses["cuda"][0]

"""The reference's OWN host code driving the CUDA device.

oracle/_ref/cuda_slot/ holds the reference's unmodified C++ sources and
pybind11 bindings linked with vectorcore_b200/csrc/host/{cuda_backend,
metal_slot}.cpp in place of its Metal stub (oracle/Makefile `slot`). In that
build the reference's non-CPU device value -- spelled "metal" by its
Device::str() -- is the B200, and its `cpu` device is the reference's own CPU
path, so these tests compare the two devices inside one process through the
reference's public API: the dispatch, Tensor, autograd engine, nn and
bindings are the reference's; only the device plugin is ours.

The checks follow the reference's own test suites (broadcast paths, unary
ops, axis reductions, classifier ops, gradients, asynchronous execution,
training). Tolerances: bit-exact for add/sub/mul/div/neg/relu/max/argmax;
<= 2 ulp for exp/sigmoid/log; 1e-5-class relative for sums and the softmax
compositions (the reference's float32 GEMM-free ops only -- matmul is an
existing op and compared at the reference's own 2e-4)."""
import importlib.machinery
import importlib.util
from pathlib import Path

import numpy as np
import pytest

import _cases as C
from _util import assert_bitexact, assert_rel, assert_ulp

pytestmark = pytest.mark.gpu

SLOT = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "cuda_slot"


@pytest.fixture(scope="module")
def vc():
    libs = sorted(SLOT.glob("vectorcore*.so"))
    if not libs:
        pytest.skip("reference slot build absent (oracle/Makefile `slot` needs the reference checkout)")
    loader = importlib.machinery.ExtensionFileLoader("vectorcore", str(libs[0]))
    spec = importlib.util.spec_from_loader("vectorcore", loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    assert mod.metal_available(), "the CUDA device is not available through the reference's device slot"
    return mod


GPU = "metal"  # the reference's non-CPU device value == the CUDA device in this build


def both(vc, x, rg=False):
    return vc.Tensor(x, requires_grad=rg), vc.Tensor(x, requires_grad=rg, device=GPU)


def test_device_identity(vc):
    assert "B200" in vc.metal_device_name()
    t = vc.Tensor([1.0, 2.0], device=GPU)
    assert t.device == "metal"
    np.testing.assert_array_equal((t * 2.0).to("cpu").numpy(), [2.0, 4.0])


@pytest.mark.parametrize("a_shape,b_shape", C.BROADCAST_CASES)
def test_broadcast_paths_bitexact(vc, a_shape, b_shape):
    rng = np.random.default_rng(len(a_shape) * 13 + len(b_shape))
    a = rng.uniform(0.5, 2, size=a_shape).astype(np.float32)
    b = rng.uniform(0.5, 2, size=b_shape).astype(np.float32)
    ca, ga = both(vc, a)
    cb, gb = both(vc, b)
    for fn in (lambda x, y: x + y, lambda x, y: x - y, lambda x, y: x * y, lambda x, y: x / y):
        assert_bitexact(fn(ga, gb).to("cpu").numpy(), fn(ca, cb).numpy())


def test_unary_ops(vc):
    x = np.random.default_rng(3).uniform(-5, 5, size=(700, 300)).astype(np.float32)
    c, g = both(vc, x)
    assert_bitexact(g.relu().to("cpu").numpy(), c.relu().numpy())
    assert_bitexact((-g).to("cpu").numpy(), (-c).numpy())
    assert_ulp(g.exp().to("cpu").numpy(), c.exp().numpy(), 2)
    assert_ulp(g.sigmoid().to("cpu").numpy(), c.sigmoid().numpy(), 2)
    p = np.abs(x) + np.float32(0.1)
    cp, gp = both(vc, p)
    assert_ulp(gp.log().to("cpu").numpy(), cp.log().numpy(), 2)


def test_axis_reductions(vc):
    x = np.random.default_rng(5).normal(size=(64, 500, 33)).astype(np.float32)
    c, g = both(vc, x)
    for axis in (0, 1, 2):
        assert_rel(g.sum(axis).to("cpu").numpy(), c.sum(axis).numpy(), 1e-5)
        assert_bitexact(g.max(axis).to("cpu").numpy(), c.max(axis).numpy())
        assert_bitexact(g.argmax(axis).to("cpu").numpy(), c.argmax(axis).numpy())
    assert_rel(np.array([g.sum().item()]), np.array([c.sum().item()]), 1e-5)
    assert g.max().item() == c.max().item()


def test_classifier_ops_and_gradients(vc):
    rng = np.random.default_rng(6)
    logits = (rng.normal(size=(64, 1000)) * 2).astype(np.float32)
    targets = [int(t) for t in rng.integers(0, 1000, 64)]
    c, g = both(vc, logits, rg=True)
    lc, lg = vc.cross_entropy(c, targets), vc.cross_entropy(g, targets)
    assert_rel(np.array([lg.item()]), np.array([lc.item()]), 1e-5)
    lc.backward()
    lg.backward()
    assert_rel(g.grad.to("cpu").numpy(), c.grad.numpy(), 1e-5, scale=1.0 / 64)
    for axis in (0, 1):
        assert_rel(g.detach().softmax(axis).to("cpu").numpy(), c.detach().softmax(axis).numpy(), 1e-5)
        assert_rel(g.detach().log_softmax(axis).to("cpu").numpy(), c.detach().log_softmax(axis).numpy(), 1e-5)


def test_broadcast_gradient_reduction(vc):
    rng = np.random.default_rng(6)
    for big, small in [((8, 5, 7), (7,)), ((8, 5, 7), (5, 1)), ((8, 5, 7), (8, 1, 7)), ((8, 5, 7), (1, 1, 1)),
                       ((8, 5, 7), ())]:
        a = rng.normal(size=big).astype(np.float32)
        b = rng.normal(size=small).astype(np.float32)
        w = rng.normal(size=big).astype(np.float32)
        grads = []
        for dev in ("cpu", GPU):
            tb = vc.Tensor(b, requires_grad=True, device=dev)
            ((vc.Tensor(a, device=dev) + tb) * vc.Tensor(w, device=dev)).sum().backward()
            grads.append(tb.grad.to("cpu").numpy())
        assert_rel(grads[1], grads[0], 1e-5)


def test_max_gradient_ties_and_bias_relu(vc):
    t = vc.Tensor([[1.0, 3.0, 3.0]], requires_grad=True, device=GPU)
    t.max(1).sum().backward()
    np.testing.assert_array_equal(t.grad.to("cpu").numpy(), [[0, 1, 0]])
    x = vc.Tensor([[-1, 2, 3], [-4, 5, 6]], requires_grad=True, device=GPU)
    bias = vc.Tensor([0.5, 1.0, -2.0], requires_grad=True, device=GPU)
    (x + bias).relu().sum().backward()
    np.testing.assert_array_equal(x.grad.to("cpu").numpy(), [[0, 1, 1], [0, 1, 1]])
    np.testing.assert_array_equal(bias.grad.to("cpu").numpy(), [0, 2, 2])


def test_matmul_and_transpose(vc):
    rng = np.random.default_rng(5)
    for a_shape, b_shape in [((2, 3, 4), (2, 4, 5)), ((2, 3, 4), (4, 5)), ((1, 17, 19), (4, 19, 18)),
                             ((127, 513), (513, 129))]:
        a = rng.normal(size=a_shape).astype(np.float32)
        b = rng.normal(size=b_shape).astype(np.float32)
        got = (vc.Tensor(a, device=GPU) @ vc.Tensor(b, device=GPU)).to("cpu").numpy()
        np.testing.assert_allclose(got, np.matmul(a.astype(np.float64), b), rtol=2e-4, atol=2e-4)
    x = np.arange(24, dtype=np.float32).reshape(2, 3, 4)
    np.testing.assert_array_equal(vc.Tensor(x, device=GPU).transpose().to("cpu").numpy(), np.swapaxes(x, -1, -2))


def test_async_chain_in_place_order_and_buffer_reuse(vc):
    x = vc.Tensor(np.zeros(1000, np.float32), device=GPU)
    for _ in range(2000):
        x = x + 1.0
    np.testing.assert_array_equal(x.to("cpu").numpy(), 2000.0)
    w = vc.Tensor(np.ones(256, np.float32), requires_grad=True, device=GPU)
    before = w * 2.0
    (w * 1.0).sum().backward()
    vc.sgd_step([w], 0.5)
    after = w * 2.0
    np.testing.assert_array_equal(before.to("cpu").numpy(), 2.0)
    np.testing.assert_array_equal(after.to("cpu").numpy(), 1.0)
    rng = np.random.default_rng(7)
    for _ in range(100):
        data = rng.normal(size=int(rng.integers(1, 5000))).astype(np.float32)
        t = vc.Tensor(data, device=GPU)
        got = ((t * 3.0).relu() - t).sum().item()
        assert np.isclose(got, float((np.maximum(data * 3.0, 0) - data).astype(np.float64).sum()), rtol=1e-4,
                          atol=1e-3)
    vc.synchronize()


def test_version_counter_detects_sgd_on_the_device(vc):
    w = vc.Tensor([[1.0], [2.0]], requires_grad=True, device=GPU)
    x = vc.Tensor([[1.0, 1.0]], device=GPU)
    stale = (w * w).sum()
    (x @ w).sum().backward()
    before = w._version
    vc.sgd_step([w], 0.1)
    assert w._version == before + 1
    with pytest.raises(RuntimeError, match="modified in place"):
        stale.backward()


def test_mlp_trains_through_the_reference_host(vc):
    rng = np.random.default_rng(0)
    feats, labels = [], []
    for label in range(3):
        radius = np.linspace(0.05, 1.0, 60)
        angle = np.linspace(label * 4.0, (label + 1) * 4.0, 60) + rng.normal(scale=0.2, size=60)
        feats.append(np.column_stack([radius * np.sin(angle), radius * np.cos(angle)]))
        labels.extend([label] * 60)
    x = vc.Tensor(np.concatenate(feats).astype(np.float32), device=GPU)
    first, second = vc.Linear(2, 64, 1), vc.Linear(64, 3, 2)
    params = [p.to(GPU).detach() for p in (first.weight, first.bias, second.weight, second.bias)]
    for p in params:
        p.requires_grad = True
    first.weight, first.bias, second.weight, second.bias = params
    for _ in range(600):
        loss = vc.cross_entropy(second(first(x).relu()), labels)
        loss.backward()
        vc.sgd_step(params, 1.0)
        vc.zero_grad(params)
    pred = second(first(x).relu()).argmax(1).to("cpu").numpy().astype(int)
    assert (pred == np.array(labels)).mean() > 0.95

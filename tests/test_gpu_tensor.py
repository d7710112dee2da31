"""The reference's Python API on the cuda device (vectorcore_b200.Tensor).

These tests follow the reference's own test suites
(tests/python/test_vectorcore.py, test_classifier_ops.py,
test_autograd_correctness.py, test_performance_paths.py): the same kinds of
checks -- NumPy / PyTorch references, finite-difference gradcheck with a
random projection, version-counter rules, leaf-only gradients, async
ordering and buffer reuse -- written for device="cuda", plus parity of whole
forward/backward pipelines with the reference's own outputs (golden vectors
and the CPU oracle)."""
import zlib

import numpy as np
import pytest

import _cases as C
import oracle
import pytensor as vc
from _util import assert_bitexact, assert_sum_close, sha256

pytestmark = pytest.mark.gpu
DEV = "cuda"


def T(x, rg=False):
    return vc.Tensor(np.asarray(x, np.float32), requires_grad=rg, device=DEV)


def close(actual, expected, rtol=2e-5, atol=2e-5):
    np.testing.assert_allclose(actual.to("cpu").numpy(), np.asarray(expected, np.float32), rtol=rtol, atol=atol)


# ---- API surface ----------------------------------------------------------------------

def test_creation_metadata_and_indexing():
    v = T([[1, 2, 3], [4, 5, 6]], True)
    assert v.shape == [2, 3] and v.strides == [3, 1] and v.ndim == 2 and v.numel == 6
    assert v.device == "cuda" and v.dtype == "float32"
    assert v.at([1, 1]) == 5
    assert "requires_grad=true" in repr(v) and "device='cuda'" in repr(v)
    with pytest.raises(IndexError):
        v.at([2, 0])


def test_device_transfer_round_trip_and_gradient():
    x = np.random.default_rng(5).uniform(-1, 1, (2, 3)).astype(np.float32)
    cpu = vc.Tensor(x, requires_grad=True)
    y = (cpu.to("cuda") * 3.0).relu()
    assert y.device == "cuda"
    y.sum().backward()
    assert cpu.grad.device == "cpu"
    np.testing.assert_array_equal(cpu.grad.numpy(), np.where(x > 0, 3.0, 0.0).astype(np.float32))


def test_cpu_tensors_do_not_compute_here():
    with pytest.raises(RuntimeError):
        vc.Tensor([1.0, 2.0]).exp()
    with pytest.raises(ValueError):
        vc.Tensor([1.0]) + T([1.0])


@pytest.mark.parametrize("a_shape,b_shape", C.BROADCAST_CASES)
def test_elementwise_paths_match_numpy(a_shape, b_shape):
    rng = np.random.default_rng(len(a_shape) * 13 + len(b_shape))
    a = rng.uniform(0.5, 2, size=a_shape).astype(np.float32)
    b = rng.uniform(0.5, 2, size=b_shape).astype(np.float32)
    ta, tb = T(a), T(b)
    for vop, nop in ((lambda x, y: x + y, np.add), (lambda x, y: x - y, np.subtract),
                     (lambda x, y: x * y, np.multiply), (lambda x, y: x / y, np.divide)):
        assert_bitexact(vop(ta, tb).numpy(), nop(a, b))


def test_scalar_operators_and_reverse_ops():
    a = np.array([0.5, 1.5, -2.0], np.float32)
    t = T(a)
    close(2.0 + t * 2.0, 2 + a * 2)
    close(3.0 / t - (1.0 - t), 3 / a - (1 - a))


# ---- reductions and the classifier blocks ---------------------------------------------------

@pytest.mark.parametrize("axis", [0, 1, 2, -1, -3])
@pytest.mark.parametrize("keepdim", [False, True])
def test_axis_reductions_match_numpy(axis, keepdim):
    x = np.random.default_rng(2).normal(size=(3, 4, 5)).astype(np.float32)
    t = T(x)
    close(t.sum(axis, keepdim), x.sum(axis=axis, keepdims=keepdim), rtol=1e-5)
    close(t.mean(axis, keepdim), x.mean(axis=axis, keepdims=keepdim), rtol=1e-5)
    close(t.max(axis, keepdim), x.max(axis=axis, keepdims=keepdim))
    close(t.argmax(axis, keepdim), x.argmax(axis=axis).reshape(x.max(axis=axis, keepdims=keepdim).shape))


def test_reductions_without_axis_and_ties():
    x = np.random.default_rng(3).normal(size=(3, 4)).astype(np.float32)
    t = T(x)
    assert t.max().item() == x.max()
    assert t.argmax().item() == x.argmax()
    assert t.sum(keepdim=True).shape == [1, 1]
    close(T([[1.0, 3.0, 3.0], [2.0, 2.0, 0.0]]).argmax(1), [1, 0])
    m = T([[1.0, 3.0, 3.0]], True)
    m.max(1).sum().backward()
    close(m.grad, [[0, 1, 0]])


@pytest.mark.parametrize("axis", [0, 1, -1])
def test_softmax_and_log_softmax(axis):
    x = (np.random.default_rng(4).normal(size=(3, 5)) * 3).astype(np.float32)
    t = T(x)
    shifted = x - x.max(axis=axis, keepdims=True)
    expected = shifted - np.log(np.exp(shifted).sum(axis=axis, keepdims=True))
    close(t.log_softmax(axis), expected, rtol=1e-4, atol=1e-5)
    close(t.softmax(axis), np.exp(expected), rtol=1e-4, atol=1e-6)
    close(vc.softmax(t, axis).sum(axis), np.ones(x.sum(axis=axis).shape), rtol=1e-5)


def test_cross_entropy_matches_pytorch():
    torch = pytest.importorskip("torch")
    logits = (np.random.default_rng(6).normal(size=(6, 4)) * 2).astype(np.float32)
    targets = [0, 3, 1, 1, 2, 0]
    t = T(logits, True)
    loss = vc.cross_entropy(t, targets)
    loss.backward()
    tt = torch.tensor(logits, requires_grad=True)
    ref = torch.nn.functional.cross_entropy(tt, torch.tensor(targets))
    ref.backward()
    assert np.isclose(loss.item(), ref.item(), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(t.grad.numpy(), tt.grad.numpy(), rtol=1e-4, atol=1e-6)


def test_cross_entropy_accepts_numpy_targets_and_known_answer():
    loss = vc.cross_entropy(T(np.zeros((3, 2))), np.array([0, 1, 1], np.int64))
    assert np.isclose(loss.item(), np.log(2.0))


@pytest.mark.parametrize("call", [
    lambda: T([[1.0, 2.0]]).sum(2),
    lambda: T([[1.0, 2.0]]).max(-3),
    lambda: T(3.0).sum(0),
    lambda: T(np.zeros((2, 0))).max(1),
    lambda: T(np.zeros((2, 0))).mean(1),
    lambda: T(np.ones((2, 3, 4))) @ T(np.ones((3, 5, 2))),
    lambda: T(np.ones((2, 3))) @ T(np.ones((4, 2))),
    lambda: T([1.0, 2.0]) @ T([1.0, 2.0]),
    lambda: vc.cross_entropy(T([1.0, 2.0]), [0]),
    lambda: vc.cross_entropy(T([[1.0, 2.0]]), [0, 1]),
    lambda: vc.cross_entropy(T([[1.0, 2.0]]), [2]),
])
def test_invalid_inputs_raise(call):
    with pytest.raises((ValueError, IndexError, RuntimeError)):
        call()


def test_sum_of_empty_axis_is_zero():
    close(T(np.zeros((2, 0))).sum(1), [0.0, 0.0])


# ---- finite-difference gradcheck (the reference's CASES, on cuda) ---------------------------

def uniform(r, shape, lo=-1.0, hi=1.0):
    return r.uniform(lo, hi, size=shape).astype(np.float32)


def away_from_zero(r, shape):
    return (r.uniform(0.2, 1.0, size=shape) * r.choice([-1.0, 1.0], size=shape)).astype(np.float32)


def well_separated(r, shape):
    n = int(np.prod(shape))
    return (r.permutation(n) * 0.1 - n * 0.05).reshape(shape).astype(np.float32)


CASES = [
    ("add_broadcast_row", lambda a, b: a + b, [lambda r: uniform(r, (2, 3)), lambda r: uniform(r, (3,))]),
    ("add_broadcast_outer", lambda a, b: a + b, [lambda r: uniform(r, (2, 1)), lambda r: uniform(r, (1, 3))]),
    ("subtract_broadcast_column", lambda a, b: a - b, [lambda r: uniform(r, (2, 3)), lambda r: uniform(r, (2, 1))]),
    ("multiply_rank3_broadcast", lambda a, b: a * b, [lambda r: uniform(r, (2, 3, 4)), lambda r: uniform(r, (4,))]),
    ("divide_broadcast", lambda a, b: a / b, [lambda r: uniform(r, (2, 3)), lambda r: uniform(r, (3,), 1, 2)]),
    ("divide_scalar_tensor", lambda a, b: a / b, [lambda r: uniform(r, (2, 3)), lambda r: uniform(r, (), 1, 2)]),
    ("negate", lambda a: -a, [lambda r: uniform(r, (2, 3))]),
    ("scalar_affine", lambda a: a * 2.5 + 1.0, [lambda r: uniform(r, (4,))]),
    ("scalar_reverse", lambda a: 3.0 / a - (1.0 - a), [lambda r: uniform(r, (4,), 1, 2)]),
    ("matmul", lambda a, b: a @ b, [lambda r: uniform(r, (3, 4)), lambda r: uniform(r, (4, 2))]),
    ("transpose", lambda a: a.T, [lambda r: uniform(r, (3, 2))]),
    ("sum", lambda a: a.sum(), [lambda r: uniform(r, (2, 3))]),
    ("mean", lambda a: a.mean(), [lambda r: uniform(r, (2, 3))]),
    ("relu", lambda a: a.relu(), [lambda r: away_from_zero(r, (3, 4))]),
    ("sigmoid", lambda a: a.sigmoid(), [lambda r: uniform(r, (3, 4), -3, 3)]),
    ("reshape", lambda a: a.reshape([3, 2]) * 2.0, [lambda r: uniform(r, (2, 3))]),
    ("reused_input", lambda a: a * a + a, [lambda r: uniform(r, (5,))]),
    ("exp", lambda a: a.exp(), [lambda r: uniform(r, (2, 3))]),
    ("log", lambda a: a.log(), [lambda r: uniform(r, (2, 3), 1, 2)]),
    ("sum_axis0", lambda a: a.sum(0), [lambda r: uniform(r, (3, 4))]),
    ("sum_axis_neg1_keepdim", lambda a: a.sum(-1, keepdim=True) * a, [lambda r: uniform(r, (2, 3, 4))]),
    ("mean_axis1", lambda a: a.mean(1), [lambda r: uniform(r, (2, 3, 4))]),
    ("max_axis1", lambda a: a.max(1), [lambda r: well_separated(r, (3, 4))]),
    ("max_axis0_keepdim", lambda a: a.max(0, keepdim=True) * a, [lambda r: well_separated(r, (3, 4))]),
    ("max_all", lambda a: a.max(), [lambda r: well_separated(r, (2, 3))]),
    ("softmax_rows", lambda a: a.softmax(-1), [lambda r: uniform(r, (3, 4), -2, 2)]),
    ("softmax_axis0", lambda a: a.softmax(0), [lambda r: uniform(r, (3, 4), -2, 2)]),
    ("log_softmax_rows", lambda a: a.log_softmax(1), [lambda r: uniform(r, (3, 4), -2, 2)]),
    ("cross_entropy", lambda a: vc.cross_entropy(a, [2, 0, 3]), [lambda r: uniform(r, (3, 4), -2, 2)]),
    ("batched_matmul_broadcast_both", lambda a, b: a @ b,
     [lambda r: uniform(r, (2, 1, 3, 4)), lambda r: uniform(r, (3, 4, 2))]),
    ("linear_sigmoid", lambda x, w, b: (x @ w + b).sigmoid(),
     [lambda r: uniform(r, (4, 3)), lambda r: uniform(r, (3, 2)), lambda r: uniform(r, (2,))]),
]


def gradcheck(fn, inputs, eps=5e-3, rtol=1e-2, atol=1e-2):
    leaves = [T(x, True) for x in inputs]
    out = fn(*leaves)
    w = np.random.default_rng(99).uniform(0.5, 1.5, size=out.shape).astype(np.float32)
    (out * T(w)).sum().backward()

    def objective(values):
        return float((fn(*[T(v) for v in values]) * T(w)).sum().item())

    for idx, (leaf, base) in enumerate(zip(leaves, inputs)):
        assert leaf.grad is not None, f"input {idx} received no gradient"
        analytic = leaf.grad.numpy()
        numeric = np.zeros(base.shape, np.float64).reshape(-1)
        for pos in range(base.size):
            plus = [v.copy() for v in inputs]
            minus = [v.copy() for v in inputs]
            plus[idx].reshape(-1)[pos] += eps
            minus[idx].reshape(-1)[pos] -= eps
            numeric[pos] = (objective(plus) - objective(minus)) / (2 * eps)
        np.testing.assert_allclose(analytic, numeric.reshape(base.shape), rtol=rtol, atol=atol)


@pytest.mark.parametrize("name,fn,factories", CASES, ids=[c[0] for c in CASES])
def test_gradcheck(name, fn, factories):
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    gradcheck(fn, [f(rng) for f in factories])


def test_relu_kink_values_are_finite():
    x = T([0.0, -0.0, 1.0], True)
    x.relu().sum().backward()
    assert np.all(np.isfinite(x.grad.numpy()))


# ---- version counter, leaves, accumulation ---------------------------------------------------

def test_version_counter_and_sgd_between_forward_and_backward_is_rejected():
    w = T([2.0], True)
    x = T([3.0], True)
    loss = (w * x).sum()
    (w * 1.0).sum().backward()
    before = w._version
    vc.sgd_step([w], 1.0)
    assert w._version == before + 1
    with pytest.raises(RuntimeError, match="modified in place"):
        loss.backward()


def test_mutation_of_saved_output_is_rejected():
    x = T([0.5, -0.5], True)
    y = x.sigmoid()
    loss = y.sum()
    y_storage = y.detach()
    y_storage.requires_grad = True
    (y_storage * 1.0).sum().backward()
    vc.sgd_step([y_storage], 1.0)
    with pytest.raises(RuntimeError, match="modified in place"):
        loss.backward()


def test_only_leaves_keep_gradients_and_retain_grad():
    a = T([1.0, 2.0], True)
    hidden = a * 2.0
    kept = a * 3.0
    kept.retain_grad()
    ((hidden * hidden).sum() + kept.sum()).backward()
    assert a.is_leaf and not hidden.is_leaf and hidden.grad is None
    close(kept.grad, [1, 1])
    close(a.grad, [8 + 3, 16 + 3])
    with pytest.raises(RuntimeError):
        T([1.0]).retain_grad()


def test_gradient_accumulates_across_backward_calls():
    x = T([1.0, 2.0], True)
    (x * 3.0).sum().backward()
    (x * 4.0).sum().backward()
    close(x.grad, [7, 7])


# ---- asynchronous execution -------------------------------------------------------------------

def test_long_dependency_chain_without_sync():
    x = T(np.zeros(1000))
    for _ in range(2000):
        x = x + 1.0
    close(x, np.full(1000, 2000.0))


def test_in_place_update_is_ordered():
    w = T(np.ones(256), True)
    before = w * 2.0
    (w * 1.0).sum().backward()
    vc.sgd_step([w], 0.5)
    after = w * 2.0
    close(before, np.full(256, 2.0))
    close(after, np.full(256, 1.0))


def test_buffer_reuse_does_not_corrupt_results():
    rng = np.random.default_rng(7)
    results, expected = [], []
    for _ in range(200):
        data = rng.normal(size=int(rng.integers(1, 5000))).astype(np.float32)
        t = T(data)
        tmp = (t * 3.0).relu()
        results.append((tmp - t).sum())
        expected.append(float((np.maximum(data * 3.0, 0) - data).astype(np.float64).sum()))
        del t, tmp
    for got, want in zip(results, expected):
        assert np.isclose(got.item(), want, rtol=1e-4, atol=1e-3)


def test_synchronize():
    vc.synchronize()
    y = T([1.0, 2.0]) * 2.0
    vc.synchronize()
    close(y, [2.0, 4.0])


# ---- training ------------------------------------------------------------------------------

def make_spiral(points_per_class=60, classes=3, seed=0):
    rng = np.random.default_rng(seed)
    feats, labels = [], []
    for label in range(classes):
        radius = np.linspace(0.05, 1.0, points_per_class)
        angle = np.linspace(label * 4.0, (label + 1) * 4.0, points_per_class) + rng.normal(scale=0.2, size=points_per_class)
        feats.append(np.column_stack([radius * np.sin(angle), radius * np.cos(angle)]))
        labels.extend([label] * points_per_class)
    return np.concatenate(feats).astype(np.float32), labels


def test_mlp_learns_nonlinear_spiral():
    feats, labels = make_spiral()
    x = T(feats)
    first, second = vc.Linear(2, 64, 1), vc.Linear(64, 3, 2)
    params = first.parameters() + second.parameters()
    for _ in range(600):
        loss = vc.cross_entropy(second(first(x).relu()), labels)
        loss.backward()
        vc.sgd_step(params, 1.0)
        vc.zero_grad(params)
    pred = second(first(x).relu()).argmax(1).numpy().astype(int)
    assert (pred == np.array(labels)).mean() > 0.95


# ---- whole pipelines vs the reference's own outputs --------------------------------------------

def test_config1_pipeline_matches_reference_golden(golden):
    """relu(x + b).sum() forward and backward at the full configuration-1 shape."""
    x_np, b_np = C.cfg1()
    x, b = T(x_np, True), T(b_np, True)
    y = (x + b).relu()
    loss = y.sum()
    loss.backward()
    assert sha256(y.numpy()) == str(golden["cfg1_full/y/sha256"])
    assert sha256(x.grad.numpy()) == str(golden["cfg1_full/dx/sha256"])
    assert_sum_close(loss.item(), golden["cfg1_full/loss"], x_np.size, 1.0)
    assert_sum_close(b.grad.numpy(), golden["cfg1_full/db"], x_np.shape[0], 1.0)


def test_fused_bias_relu_sum_matches_reference_golden(golden):
    """The one-launch fused chain gives the reference's configuration-1
    results: dx and db bit for bit, the loss within the sum tolerance."""
    x_np, b_np = C.cfg1()
    x, b = T(x_np, True), T(b_np, True)
    loss = vc.bias_relu_sum(x, b)
    loss.backward()
    assert sha256(x.grad.numpy()) == str(golden["cfg1_full/dx/sha256"])
    assert_sum_close(loss.item(), golden["cfg1_full/loss"], x_np.size, 1.0)
    assert_bitexact(b.grad.numpy(), golden["cfg1_full/db"], "db")


@pytest.mark.parametrize("shape", [(1, 1), (3, 5), (65, 130), (200, 4100), (1000, 8), (1000, 16), (37, 160),
                                   (4096, 32), (4097, 64), (129, 16400)])
def test_fused_bias_relu_sum_matches_composed_ops(shape):
    """Odd column counts (scalar path), rows across several 64-row segments,
    columns across several 1024-column blocks, column strips of 16 floats
    (up to 4096 rows, then the segmented kernel) and a non-unit upstream."""
    rng = np.random.default_rng(shape[0] * 7 + shape[1])
    x_np = rng.uniform(-1, 1, shape).astype(np.float32)
    b_np = rng.normal(size=shape[1]).astype(np.float32)
    x1, b1 = T(x_np, True), T(b_np, True)
    fused = vc.bias_relu_sum(x1, b1) * 0.37
    fused.backward()
    x2, b2 = T(x_np, True), T(b_np, True)
    composed = (x2 + b2).relu().sum() * 0.37
    composed.backward()
    assert_sum_close(fused.item(), composed.item(), x_np.size, 1.0)
    assert_bitexact(x1.grad.numpy(), x2.grad.numpy(), "dx")
    # db is g times an exact row count: the same bits as the double sum
    assert_bitexact(b1.grad.numpy(), b2.grad.numpy(), "db")
    for _ in range(2):  # the ticket counters reset themselves: repeat calls agree
        again = vc.bias_relu_sum(x1, b1).item()
        assert again == vc.bias_relu_sum(x1, b1).item()


def test_config5_pipeline_matches_reference_golden(golden):
    a_np, b_np = C.cfg5(C.SMALL["cfg5"]["a"], C.SMALL["cfg5"]["b"])
    a, b = T(a_np, True), T(b_np, True)
    out = a * b
    assert sha256(out.numpy()) == str(golden["cfg5/out/sha256"])
    s = out.sum()
    s.backward()
    assert_sum_close(s.item(), golden["cfg5/sum"], out.numel, 1.0)
    assert_sum_close(a.grad.numpy(), golden["cfg5/sum_bwd/da"], 16, 1.0)
    assert_sum_close(b.grad.numpy(), golden["cfg5/sum_bwd/db"], 32, 1.0)


def test_composite_gradients_match_reference_autograd(port):
    """A graph mixing broadcast, division, reductions and a softmax: the cuda
    autograd and the reference's chain rules (CPU oracle) agree."""
    rng = np.random.default_rng(21)
    x_np = rng.uniform(-1, 1, (16, 33)).astype(np.float32)
    w_np = rng.uniform(1, 2, (33,)).astype(np.float32)
    x, w = T(x_np, True), T(w_np, True)
    z = (x / w).log_softmax(-1)
    loss = (z * x).sum()
    loss.backward()
    # the same graph, step by step on the oracle
    q = port.binary(oracle.DIV, x_np, w_np)
    zq = port.log_softmax(q)
    g_z = x_np                               # d(sum(z * x))/dz
    g_x_direct = zq                          # d/dx through the product
    g_q = port.log_softmax_backward(q, g_z)
    gx_div, gw = port.binary_backward(oracle.DIV, x_np, w_np, g_q)
    np.testing.assert_allclose(x.grad.numpy(), gx_div + g_x_direct, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(w.grad.numpy(), gw, rtol=1e-4, atol=1e-4)

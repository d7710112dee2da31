"""Tensor and reverse-mode autograd over the C ABI -- a TEST HELPER.

The reference itself runs on the cuda device through its own host
(reference_cuda_device.patch, exercised by tests/test_gpu_reference_host.py).
This Python restatement of its Tensor layer lets tests drive the fused entry
points and CUDA graphs through a Tensor-shaped API without a C++ build.

Mirrors the reference's public Tensor API (include/vectorcore/tensor.hpp,
python/bindings.cpp:63-179) -- same names, argument meaning, shapes, error
types and autograd rules (src/tensor.cpp:244-301, src/ops.cpp,
src/autograd.cpp) -- so code written against ``vectorcore`` runs on the B200
device with ``device="cuda"``. Every computation goes through the C ABI's
fused kernels (``backend.CudaBackend``): broadcast gradients are reduced in
one pass, softmax / log_softmax / cross-entropy are single kernels, and the
backward rules are fused VJPs. ``cpu`` tensors hold host values for
``to("cuda")`` / ``numpy()``; computing on them is the reference's CPU
device, not this package's (there is no CPU fallback here).
"""
from __future__ import annotations

import math
import threading
from typing import Optional, Sequence

import numpy as np

from vectorcore_b200 import backend as _B
from vectorcore_b200.backend import CudaBackend, CudaStorage

_state = threading.local()


def grad_enabled() -> bool:
    return getattr(_state, "enabled", True)


class NoGradGuard:
    """Disable graph recording in a scope (src/autograd.cpp:15-19)."""

    def __enter__(self):
        self.previous = grad_enabled()
        _state.enabled = False
        return self

    def __exit__(self, *exc):
        _state.enabled = self.previous


no_grad = NoGradGuard


def _be() -> CudaBackend:
    return CudaBackend.instance()


def parse_device(name: str) -> str:
    if name in ("cpu",):
        return "cpu"
    if name in ("cuda", "cuda:0", "gpu"):
        return "cuda"
    raise ValueError("device must be 'cpu' or 'cuda'")


class HostStorage:
    """Values of a cpu tensor (host staging) with the shared version counter."""

    __slots__ = ("values", "version")

    def __init__(self, values: np.ndarray):
        self.values = np.ascontiguousarray(values, np.float32).reshape(-1)
        self.version = 0

    @property
    def size(self):
        return self.values.size

    def bump_version(self):
        self.version += 1


class GradFn:
    __slots__ = ("parents", "backward")

    def __init__(self, parents, backward):
        self.parents = parents
        self.backward = backward


class _Impl:
    __slots__ = ("storage", "shape", "requires_grad", "leaf", "retains_grad", "grad_fn", "grad", "__weakref__")

    def __init__(self, storage, shape, requires_grad=False):
        self.storage = storage
        self.shape = tuple(int(s) for s in shape)
        self.requires_grad = requires_grad
        self.leaf = True
        self.retains_grad = False
        self.grad_fn = None
        self.grad = None


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return n


def _strides(shape):
    out, s = [], 1
    for d in reversed(shape):
        out.append(s)
        s *= int(d)
    return list(reversed(out))


def _broadcast_shape(a, b):
    rank = max(len(a), len(b))
    out = []
    for i in range(rank):
        ai = 1 if i < rank - len(a) else a[i - (rank - len(a))]
        bi = 1 if i < rank - len(b) else b[i - (rank - len(b))]
        if ai != bi and ai != 1 and bi != 1:
            raise ValueError(f"cannot broadcast shapes {list(a)} and {list(b)}")
        out.append(max(ai, bi))
    return tuple(out)


class SavedTensor:
    """A tensor captured for backward plus its storage version
    (src/autograd.cpp:23-34)."""

    __slots__ = ("tensor", "version")

    def __init__(self, t: "Tensor"):
        self.tensor = t.detach()
        self.version = t._version

    def unpack(self) -> "Tensor":
        if self.tensor._version != self.version:
            raise RuntimeError(
                "a tensor needed for gradient computation was modified in place after it was used "
                f"(saved version {self.version}, current version {self.tensor._version}); run backward() "
                "before mutating it")
        return self.tensor


def _attach(output: "Tensor", parents: Sequence["Tensor"], backward) -> None:
    """attach_grad_fn (src/autograd.cpp:36-48)."""
    if not grad_enabled():
        return
    if not any(p.requires_grad for p in parents):
        return
    impl = output._impl
    impl.grad_fn = GradFn([p._impl for p in parents], backward)
    impl.requires_grad = True
    impl.leaf = False


class Tensor:
    __slots__ = ("_impl",)

    # ---- construction ------------------------------------------------------------
    def __init__(self, values=0.0, requires_grad: bool = False, device: str = "cpu"):
        if isinstance(values, _Impl):
            self._impl = values
            return
        dev = parse_device(device)
        if isinstance(values, Tensor):
            values = values.numpy()
        arr = np.asarray(values, dtype=np.float32)
        if arr.dtype == object:
            raise ValueError("Tensor values must be a scalar or rectangular array-like object")
        shape = arr.shape
        if dev == "cuda":
            be = _be()
            if not be.available():
                raise RuntimeError(f"CUDA is unavailable: {be.last_error()}")
            storage = be.upload(arr.reshape(-1) if arr.size else np.zeros(0, np.float32))
        else:
            storage = HostStorage(arr)
        self._impl = _Impl(storage, shape, requires_grad)

    @classmethod
    def _from(cls, storage, shape, requires_grad=False) -> "Tensor":
        return cls(_Impl(storage, shape, requires_grad))

    @classmethod
    def scalar(cls, value: float, requires_grad=False, device="cpu") -> "Tensor":
        return cls(np.float32(value), requires_grad, device)

    @classmethod
    def zeros(cls, shape, requires_grad=False, device="cpu") -> "Tensor":
        shape = tuple(shape)
        if parse_device(device) == "cuda":
            return cls._from(_be().fill(_numel(shape), 0.0), shape, requires_grad)
        return cls(np.zeros(shape, np.float32), requires_grad, device)

    @classmethod
    def ones(cls, shape, requires_grad=False, device="cpu") -> "Tensor":
        shape = tuple(shape)
        if parse_device(device) == "cuda":
            return cls._from(_be().fill(_numel(shape), 1.0), shape, requires_grad)
        return cls(np.ones(shape, np.float32), requires_grad, device)

    @classmethod
    def randn(cls, shape, requires_grad=False, seed: int = 0, device="cpu") -> "Tensor":
        # Standard normal values from a seeded host generator. (The reference
        # draws them with std::mt19937_64; the values differ, the
        # distribution does not.)
        values = np.random.default_rng(seed).standard_normal(tuple(shape)).astype(np.float32)
        return cls(values, requires_grad, device)

    # ---- metadata ----------------------------------------------------------------
    @property
    def shape(self):
        return list(self._impl.shape)

    @property
    def strides(self):
        return _strides(self._impl.shape)

    @property
    def ndim(self):
        return len(self._impl.shape)

    @property
    def numel(self):
        return _numel(self._impl.shape)

    @property
    def device(self):
        return "cuda" if isinstance(self._impl.storage, CudaStorage) else "cpu"

    @property
    def dtype(self):
        return "float32"

    @property
    def is_cuda(self):
        return self.device == "cuda"

    @property
    def requires_grad(self):
        return self._impl.requires_grad

    @requires_grad.setter
    def requires_grad(self, value: bool):
        if not self._impl.leaf:
            raise RuntimeError("requires_grad can only be changed on leaf tensors")
        self._impl.requires_grad = bool(value)
        if not value:
            self._impl.grad = None

    @property
    def is_leaf(self):
        return self._impl.leaf

    @property
    def retains_grad(self):
        return self._impl.retains_grad

    @property
    def _version(self):
        return self._impl.storage.version

    def retain_grad(self):
        if not self._impl.requires_grad:
            raise RuntimeError("retain_grad() requires a tensor that requires gradients")
        if not self._impl.leaf:
            self._impl.retains_grad = True

    @property
    def grad(self) -> Optional["Tensor"]:
        g = self._impl.grad
        return Tensor(g) if g is not None else None

    # ---- host access (synchronising) -------------------------------------------------
    def numpy(self) -> np.ndarray:
        s = self._impl.storage
        n = self.numel
        if isinstance(s, HostStorage):
            return s.values[:n].reshape(self._impl.shape).copy()
        return _be().download(s, n).reshape(self._impl.shape)

    def to_vector(self):
        return self.numpy().reshape(-1).tolist()

    def item(self) -> float:
        if self.numel != 1:
            raise RuntimeError("item() requires a one-element tensor")
        return float(self.numpy().reshape(-1)[0])

    def at(self, indices) -> float:
        if len(indices) != self.ndim:
            raise IndexError("index rank does not match tensor rank")
        for i, d in zip(indices, self._impl.shape):
            if i >= d or i < 0:
                raise IndexError("tensor index out of bounds")
        return float(self.numpy()[tuple(indices)])

    def __repr__(self):
        vals = self.numpy().reshape(-1)
        shown = ", ".join(f"{v:.6g}" for v in vals[:8]) + (", ..." if vals.size > 8 else "")
        return (f"Tensor(shape={self.shape}, dtype='float32', device='{self.device}', "
                f"requires_grad={'true' if self.requires_grad else 'false'}, values=[{shown}])")

    # ---- views and devices ------------------------------------------------------------
    def detach(self) -> "Tensor":
        return Tensor._from(self._impl.storage, self._impl.shape)

    def reshape(self, shape) -> "Tensor":
        shape = tuple(int(s) for s in shape)
        if _numel(shape) != self.numel:
            raise ValueError(f"cannot reshape {self.shape} to {list(shape)}")
        out = Tensor._from(self._impl.storage, shape)
        original = self._impl.shape
        _attach(out, [self], lambda g: [g.reshape(original)])
        return out

    def flatten(self) -> "Tensor":
        return self.reshape((self.numel,))

    def to(self, device: str) -> "Tensor":
        """Copy to the other device (src/tensor.cpp:168-187), without the
        reference's intermediate host vector: cuda -> cpu downloads straight
        into the new host storage, cpu -> cuda uploads straight from the host
        values (large pageable copies are staged through page-locked buffers
        by the library)."""
        target = parse_device(device)
        if target == self.device:
            return self
        shape = self._impl.shape
        if target == "cpu":
            out = Tensor._from(HostStorage(_be().download(self._impl.storage, self.numel)), shape)
        else:
            values = self._impl.storage.values[: self.numel]
            out = Tensor._from(_be().upload(values if values.size else np.zeros(0, np.float32)), shape)
        source = self.device
        _attach(out, [self], lambda g: [g.to(source)])
        return out

    def cuda(self) -> "Tensor":
        return self.to("cuda")

    def cpu(self) -> "Tensor":
        return self.to("cpu")

    # ---- autograd ----------------------------------------------------------------------
    def zero_grad(self):
        self._impl.grad = None

    def backward(self, gradient: Optional["Tensor"] = None):
        """Reverse-mode pass in the reference engine's order
        (src/tensor.cpp:244-301): DFS topological order, gradients
        accumulated with +, released once consumed; leaves (and tensors that
        asked with retain_grad) keep .grad."""
        if gradient is None:
            if self.numel != 1:
                raise RuntimeError("backward() without a gradient requires a scalar tensor")
            gradient = Tensor.ones(self._impl.shape, False, self.device)
        if not self.requires_grad:
            raise RuntimeError("cannot call backward on a tensor without gradients")
        if tuple(gradient._impl.shape) != self._impl.shape:
            raise ValueError("backward gradient shape mismatch")
        if gradient.device != self.device:
            raise ValueError("backward gradient device mismatch")
        topo, seen = [], set()
        stack = [(self._impl, False)]
        while stack:  # iterative post-order DFS (same order as the recursive visit)
            node, done = stack.pop()
            if done:
                topo.append(node)
                continue
            if id(node) in seen:
                continue
            seen.add(id(node))
            stack.append((node, True))
            if node.grad_fn is not None:
                for parent in reversed(node.grad_fn.parents):
                    if id(parent) not in seen:
                        stack.append((parent, False))
        with NoGradGuard():
            grads = {id(self._impl): gradient.detach()}
            for node in reversed(topo):
                upstream = grads.pop(id(node), None)
                if upstream is None:
                    continue
                if node.requires_grad and (node.leaf or node.retains_grad):
                    if node.grad is not None:
                        node.grad = (Tensor(node.grad) + upstream).detach()._impl
                    else:
                        node.grad = upstream.detach()._impl
                if node.grad_fn is None:
                    continue
                parent_grads = node.grad_fn.backward(upstream)
                if len(parent_grads) != len(node.grad_fn.parents):
                    raise RuntimeError("autograd function returned the wrong number of gradients")
                for parent, pg in zip(node.grad_fn.parents, parent_grads):
                    if not parent.requires_grad or pg is None:
                        continue
                    key = id(parent)
                    if key in grads:
                        grads[key] = grads[key] + pg
                    else:
                        grads[key] = pg.detach()

    # ---- operators ------------------------------------------------------------------------
    def __add__(self, other):
        return add(self, other)

    def __radd__(self, other):
        return add(other, self)

    def __sub__(self, other):
        return subtract(self, other)

    def __rsub__(self, other):
        return subtract(other, self)

    def __mul__(self, other):
        return multiply(self, other)

    def __rmul__(self, other):
        return multiply(other, self)

    def __truediv__(self, other):
        return divide(self, other)

    def __rtruediv__(self, other):
        return divide(other, self)

    def __neg__(self):
        return negate(self)

    def __matmul__(self, other):
        return matmul(self, other)

    # ---- methods ----------------------------------------------------------------------------
    def relu(self):
        return relu(self)

    def sigmoid(self):
        return sigmoid(self)

    def exp(self):
        return exp(self)

    def log(self):
        return log(self)

    def sum(self, axis: Optional[int] = None, keepdim: bool = False):
        return _all_or_axis(self, axis, keepdim, sum_all, sum_axis)

    def mean(self, axis: Optional[int] = None, keepdim: bool = False):
        return _all_or_axis(self, axis, keepdim, mean_all, mean_axis)

    def max(self, axis: Optional[int] = None, keepdim: bool = False):
        return _all_or_axis(self, axis, keepdim, max_all, max_axis)

    def argmax(self, axis: Optional[int] = None, keepdim: bool = False):
        if axis is not None:
            return argmax(self, axis, keepdim)
        flat = argmax(self.flatten(), 0, False)
        return flat.reshape([1] * self.ndim) if keepdim else flat

    def softmax(self, axis: int = -1):
        return softmax(self, axis)

    def log_softmax(self, axis: int = -1):
        return log_softmax(self, axis)

    def matmul(self, other):
        return matmul(self, other)

    def transpose(self):
        return transpose(self)

    @property
    def T(self):
        return transpose(self)


def _all_or_axis(t, axis, keepdim, all_fn, axis_fn):
    """reduce_all_or_axis (python/bindings.cpp:53-59)."""
    if axis is not None:
        return axis_fn(t, int(axis), keepdim)
    r = all_fn(t)
    return r.reshape([1] * t.ndim) if keepdim else r


# ---------------------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------------------
def _require_cuda(*ts: Tensor) -> None:
    for t in ts:
        if t.device != "cuda":
            raise RuntimeError("vectorcore_b200 computes on the cuda device; move the tensor with .to('cuda') "
                               "(cpu tensors are computed by VectorCore's own CPU backend)")


def _same_device(a: Tensor, b: Tensor) -> None:
    if a.device != b.device:
        raise ValueError(f"tensor device mismatch: {a.device} vs {b.device}")
    _require_cuda(a, b)


def _is_scalar(x) -> bool:
    return isinstance(x, (int, float, np.floating, np.integer)) and not isinstance(x, bool)


def _out(storage, shape) -> Tensor:
    return Tensor._from(storage, shape)


def _split_axis(shape, axis: int):
    """split_axis (src/ops.cpp:63-80)."""
    rank = len(shape)
    if rank == 0:
        raise ValueError("cannot reduce a scalar along an axis")
    if axis < -rank or axis >= rank:
        raise IndexError(f"axis {axis} is out of range for shape {list(shape)}")
    ax = axis + rank if axis < 0 else axis
    outer = _numel(shape[:ax])
    inner = _numel(shape[ax + 1:])
    kept = tuple(shape[:ax]) + (1,) + tuple(shape[ax + 1:])
    removed = tuple(shape[:ax]) + tuple(shape[ax + 1:])
    return ax, outer, int(shape[ax]), inner, kept, removed


# ---------------------------------------------------------------------------------------
# elementwise (src/ops.cpp:27-52, 98-164, 360-376, 395-413)
# ---------------------------------------------------------------------------------------
_OPCODE = {"add": _B.ADD, "sub": _B.SUB, "mul": _B.MUL, "div": _B.DIV}


def _binary(name: str, a, b) -> Tensor:
    op = _OPCODE[name]
    be = _be()
    if _is_scalar(b) and isinstance(a, Tensor):
        return _binary_scalar(name, a, np.float32(b), scalar_first=False)
    if _is_scalar(a) and isinstance(b, Tensor):
        return _binary_scalar(name, b, np.float32(a), scalar_first=True)
    if not isinstance(a, Tensor) or not isinstance(b, Tensor):
        return NotImplemented
    _same_device(a, b)
    shape = _broadcast_shape(a._impl.shape, b._impl.shape)
    out = _out(be.binary(a._impl.storage, a._impl.shape, None, b._impl.storage, b._impl.shape, None, shape, op),
               shape)
    need_a, need_b = a.requires_grad, b.requires_grad
    a_shape, b_shape = a._impl.shape, b._impl.shape
    saved_a = SavedTensor(a) if name in ("mul", "div") else None
    saved_b = SavedTensor(b) if name in ("mul", "div") else None

    def backward(g: Tensor):
        ga = gb = None
        if name in ("add", "sub"):
            # the same-shape gradient aliases g (sum_to_shape returns it as is)
            if need_a:
                ga = g if a_shape == g._impl.shape else _sum_to_shape(g, a_shape)
            if need_b:
                if name == "add":
                    gb = g if b_shape == g._impl.shape else _sum_to_shape(g, b_shape)
                elif b_shape == g._impl.shape:
                    gb = _out(be.unary(g._impl.storage, g.numel, _B.NEG), b_shape)
                else:
                    gb = _out(be.binary_backward(op, None, a_shape, None, b_shape, g._impl.storage, g._impl.shape,
                                                 need_a=False)[1], b_shape)
            return [ga, gb]
        av, bv = saved_a.unpack(), saved_b.unpack()
        da, db = be.binary_backward(op, av._impl.storage, a_shape, bv._impl.storage, b_shape, g._impl.storage,
                                    g._impl.shape, need_a=need_a, need_b=need_b)
        return [_out(da, a_shape) if da is not None else None, _out(db, b_shape) if db is not None else None]

    _attach(out, [a, b], backward)
    return out


def _binary_scalar(name: str, t: Tensor, s: np.float32, scalar_first: bool) -> Tensor:
    """tensor (op) python scalar: the scalar travels by value (the reference
    uploads a one-element tensor, src/tensor.cpp:323-330; same arithmetic)."""
    _require_cuda(t)
    be = _be()
    op = _OPCODE[name]
    shape = t._impl.shape
    out = _out(be.binary_scalar(t._impl.storage, t.numel, float(s), op, scalar_first), shape)
    saved = SavedTensor(t) if (name == "div" and scalar_first) else None

    def backward(g: Tensor):
        n = g.numel
        if name == "add" or (name == "sub" and not scalar_first):
            return [g]
        if name == "sub":
            return [_out(be.unary(g._impl.storage, n, _B.NEG), shape)]
        if name == "mul":
            return [_out(be.binary_scalar(g._impl.storage, n, float(s), _B.MUL), shape)]
        if not scalar_first:  # a / s: g / s
            return [_out(be.binary_scalar(g._impl.storage, n, float(s), _B.DIV), shape)]
        # s / a: -(g * s) / (a * a)
        sdev = be.upload(np.array([s], np.float32))
        tv = saved.unpack()
        _, db = be.binary_backward(_B.DIV, sdev, (), tv._impl.storage, shape, g._impl.storage, shape,
                                   need_a=False, need_b=True)
        return [_out(db, shape)]

    _attach(out, [t], backward)
    return out


def add(a, b):
    return _binary("add", a, b)


def subtract(a, b):
    return _binary("sub", a, b)


def multiply(a, b):
    return _binary("mul", a, b)


def divide(a, b):
    return _binary("div", a, b)


def _unary(t: Tensor, op: int, save: str) -> Tensor:
    _require_cuda(t)
    be = _be()
    out = _out(be.unary(t._impl.storage, t.numel, op), t._impl.shape)
    saved = SavedTensor(out if save == "y" else t) if save else None
    shape = t._impl.shape

    def backward(g: Tensor):
        x = y = None
        if save == "y":
            y = saved.unpack()._impl.storage
        elif save == "x":
            x = saved.unpack()._impl.storage
        return [_out(be.unary_backward(op, x, y, g._impl.storage, g.numel), shape)]

    _attach(out, [t], backward)
    return out


def negate(t: Tensor) -> Tensor:
    return _unary(t, _B.NEG, "")


def exp(t: Tensor) -> Tensor:
    return _unary(t, _B.EXP, "y")


def log(t: Tensor) -> Tensor:
    return _unary(t, _B.LOG, "x")


def relu(t: Tensor) -> Tensor:
    return _unary(t, _B.RELU, "x")


def sigmoid(t: Tensor) -> Tensor:
    return _unary(t, _B.SIGMOID, "y")


def _sum_to_shape(g: Tensor, target) -> Tensor:
    """detail::sum_to_shape (src/autograd.cpp:50-72) as one fused reduce."""
    target = tuple(target)
    if g._impl.shape == target:
        return g
    return _out(_be().sum_to_shape(g._impl.storage, g._impl.shape, target), target)


def _broadcast_to(g: Tensor, target) -> Tensor:
    """detail::broadcast_to (src/autograd.cpp:74-91): g + 0 in the target shape."""
    target = tuple(target)
    if g._impl.shape == target:
        return g
    return _out(_be().broadcast_to(g._impl.storage, g._impl.shape, target), target)


# ---------------------------------------------------------------------------------------
# reductions (src/ops.cpp:288-358, 390-393)
# ---------------------------------------------------------------------------------------
def sum_all(t: Tensor) -> Tensor:
    _require_cuda(t)
    be = _be()
    out = _out(be.reduce_sum(t._impl.storage, t.numel), ())
    shape = t._impl.shape
    _attach(out, [t], lambda g: [_broadcast_to(g, shape)])
    return out


def mean_all(t: Tensor) -> Tensor:
    _require_cuda(t)
    if t.numel == 0:
        raise ValueError("mean of an empty tensor is undefined")
    be = _be()
    out = _out(be.reduce_all(t._impl.storage, t.numel, _B.REDUCE_MEAN), ())
    shape, n = t._impl.shape, t.numel
    _attach(out, [t], lambda g: [_out(be.reduce_axis_backward(_B.REDUCE_MEAN, g._impl.storage, None, 1, n, 1),
                                      shape)])
    return out


def sum_axis(t: Tensor, axis: int, keepdim: bool = False) -> Tensor:
    _require_cuda(t)
    ax, outer, length, inner, kept, removed = _split_axis(t._impl.shape, axis)
    be = _be()
    out = _out(be.reduce_axis(t._impl.storage, outer, length, inner, _B.REDUCE_SUM), kept if keepdim else removed)
    shape = t._impl.shape
    _attach(out, [t], lambda g: [_out(be.reduce_axis_backward(_B.REDUCE_SUM, g._impl.storage, None, outer, length,
                                                              inner), shape)])
    return out


def mean_axis(t: Tensor, axis: int, keepdim: bool = False) -> Tensor:
    _require_cuda(t)
    ax, outer, length, inner, kept, removed = _split_axis(t._impl.shape, axis)
    if length == 0:
        raise ValueError("mean over an empty axis is undefined")
    be = _be()
    out = _out(be.reduce_axis(t._impl.storage, outer, length, inner, _B.REDUCE_MEAN), kept if keepdim else removed)
    shape = t._impl.shape
    _attach(out, [t], lambda g: [_out(be.reduce_axis_backward(_B.REDUCE_MEAN, g._impl.storage, None, outer,
                                                              length, inner), shape)])
    return out


def max_axis(t: Tensor, axis: int, keepdim: bool = False) -> Tensor:
    _require_cuda(t)
    ax, outer, length, inner, kept, removed = _split_axis(t._impl.shape, axis)
    if length == 0:
        raise ValueError("max/argmax over an empty axis is undefined")
    be = _be()
    # one pass gives the values and the argmax the backward scatters to
    vals, idx = be.reduce_axis(t._impl.storage, outer, length, inner, _B.REDUCE_MAX, want_index=True)
    out = _out(vals, kept if keepdim else removed)
    shape = t._impl.shape
    _attach(out, [t], lambda g: [_out(be.reduce_axis_backward(_B.REDUCE_MAX, g._impl.storage, idx, outer, length,
                                                              inner), shape)])
    return out


def max_all(t: Tensor) -> Tensor:
    if t.numel == 0:
        raise ValueError("max of an empty tensor is undefined")
    return max_axis(t.flatten(), 0, False)


def argmax(t: Tensor, axis: int, keepdim: bool = False) -> Tensor:
    """Indices of the maximum as float32 (the reference's convention,
    include/vectorcore/ops.hpp:28); not differentiable."""
    _require_cuda(t)
    ax, outer, length, inner, kept, removed = _split_axis(t._impl.shape, axis)
    if length == 0:
        raise ValueError("max/argmax over an empty axis is undefined")
    return _out(_be().reduce_axis(t._impl.storage, outer, length, inner, _B.REDUCE_ARGMAX),
                kept if keepdim else removed)


def argmax_int64(t: Tensor, axis: int) -> np.ndarray:
    """int64 argmax along `axis` (an extension: the reference returns float32)."""
    _require_cuda(t)
    ax, outer, length, inner, kept, removed = _split_axis(t._impl.shape, axis)
    _, idx = _be().reduce_axis(t._impl.storage, outer, length, inner, _B.REDUCE_MAX, want_index=True)
    return _be().download(idx).reshape(removed)


# ---------------------------------------------------------------------------------------
# softmax family and cross-entropy (src/ops.cpp:378-388, src/nn.cpp:31-53)
# ---------------------------------------------------------------------------------------
def _softmax_impl(t: Tensor, axis: int, log_: bool) -> Tensor:
    _require_cuda(t)
    ax, outer, length, inner, kept, removed = _split_axis(t._impl.shape, axis)
    be = _be()
    y, m, s = be.softmax(t._impl.storage, outer, length, inner, log=log_)
    out = _out(y, t._impl.shape)
    saved = SavedTensor(t)
    shape = t._impl.shape

    def backward(g: Tensor):
        x = saved.unpack()
        return [_out(be.softmax_backward(x._impl.storage, m, s, g._impl.storage, outer, length, inner, log=log_),
                     shape)]

    _attach(out, [t], backward)
    return out


def softmax(t: Tensor, axis: int = -1) -> Tensor:
    return _softmax_impl(t, axis, False)


def log_softmax(t: Tensor, axis: int = -1) -> Tensor:
    return _softmax_impl(t, axis, True)


def cross_entropy(logits: Tensor, targets) -> Tensor:
    """Mean softmax cross-entropy of [batch, classes] logits and integer class
    targets (nn::cross_entropy, src/nn.cpp:31-53), fused: no one-hot mask."""
    if logits.ndim != 2:
        raise ValueError(f"cross_entropy expects [batch, classes] logits, got {logits.shape}")
    batch, classes = logits._impl.shape
    tg = np.asarray(targets)
    if tg.ndim != 1 or tg.shape[0] != batch:
        raise ValueError(f"cross_entropy received {tg.size} targets for a batch of {batch}")
    if batch == 0:
        raise ValueError("cross_entropy of an empty batch is undefined")
    tg = tg.astype(np.int64)
    bad = (tg < 0) | (tg >= classes)
    if bad.any():
        raise IndexError(f"target class {int(tg[bad][0])} is out of range for {classes} classes")
    _require_cuda(logits)
    be = _be()
    dt = be.upload(tg)
    loss, m, s, _ = be.cross_entropy(logits._impl.storage, dt, batch, classes)
    out = _out(loss, ())
    saved = SavedTensor(logits)

    def backward(g: Tensor):
        x = saved.unpack()
        return [_out(be.cross_entropy_backward(x._impl.storage, dt, m, s, g._impl.storage, batch, classes),
                     (batch, classes))]

    _attach(out, [logits], backward)
    return out


def bias_relu_sum(x: Tensor, b: Tensor) -> Tensor:
    """relu(x + b).sum() for x [rows, cols] and a bias b [cols], fused: one
    kernel forward, one backward (same values as the composed ops: the loss
    and db within the sum tolerance, dx bit for bit)."""
    _same_device(x, b)
    if x.ndim != 2 or b.ndim != 1 or b._impl.shape[0] != x._impl.shape[1]:
        raise ValueError(f"bias_relu_sum expects x [rows, cols] and b [cols], got {x.shape} and {b.shape}")
    rows, cols = x._impl.shape
    be = _be()
    out = _out(be.bias_relu_sum(x._impl.storage, b._impl.storage, rows, cols), ())
    saved_x, saved_b = SavedTensor(x), SavedTensor(b)

    def backward(g: Tensor):
        xs, bs = saved_x.unpack(), saved_b.unpack()
        dx, db = be.bias_relu_sum_backward(xs._impl.storage, bs._impl.storage, g._impl.storage, rows, cols)
        return [_out(dx, (rows, cols)), _out(db, (cols,))]

    _attach(out, [x, b], backward)
    return out


# ---------------------------------------------------------------------------------------
# matmul / transpose (src/ops.cpp:166-286) -- existing ops, correct not tuned
# ---------------------------------------------------------------------------------------
def _matmul_kernel(a: Tensor, b: Tensor, trans_a: bool, trans_b: bool) -> Tensor:
    _same_device(a, b)
    if a.ndim < 2 or b.ndim < 2:
        raise ValueError(f"matmul requires tensors of rank 2 or more, got {a.shape} and {b.shape}")
    as_, bs = a._impl.shape, b._impl.shape
    a_rows, a_cols = as_[-2], as_[-1]
    b_rows, b_cols = bs[-2], bs[-1]
    m = a_cols if trans_a else a_rows
    k = a_rows if trans_a else a_cols
    n = b_rows if trans_b else b_cols
    if (b_cols if trans_b else b_rows) != k:
        raise ValueError(f"matmul shape mismatch: {list(as_)} and {list(bs)}")
    a_batch, b_batch = as_[:-2], bs[:-2]
    try:
        out_batch = _broadcast_shape(a_batch, b_batch)
    except ValueError:
        raise ValueError(f"matmul batch dimensions do not broadcast: {list(as_)} and {list(bs)}") from None
    batch = _numel(out_batch)
    a_str, b_str = _strides(a_batch), _strides(b_batch)
    rank = len(out_batch)
    a_off, b_off = [], []
    for z in range(batch):
        rem, ai, bi = z, 0, 0
        for axis in range(rank - 1, -1, -1):
            c = rem % out_batch[axis]
            rem //= out_batch[axis]
            if axis >= rank - len(a_batch):
                ia = axis - (rank - len(a_batch))
                if a_batch[ia] != 1:
                    ai += c * a_str[ia]
            if axis >= rank - len(b_batch):
                ib = axis - (rank - len(b_batch))
                if b_batch[ib] != 1:
                    bi += c * b_str[ib]
        a_off.append(ai * m * k)
        b_off.append(bi * k * n)
    out_shape = tuple(out_batch) + (m, n)
    if batch == 0 or m == 0 or n == 0:
        return _out(_be().allocate(_numel(out_shape)), out_shape)
    return _out(_be().matmul(a._impl.storage, b._impl.storage, m, k, n, a_off, b_off, trans_a, trans_b), out_shape)


def matmul(a: Tensor, b: Tensor) -> Tensor:
    out = _matmul_kernel(a, b, False, False)
    sa, sb = SavedTensor(a), SavedTensor(b)
    as_, bs = a._impl.shape, b._impl.shape
    need_a, need_b = a.requires_grad, b.requires_grad

    def backward(g: Tensor):
        ga = _sum_to_shape(_matmul_kernel(g, sb.unpack(), False, True), as_) if need_a else None
        gb = _sum_to_shape(_matmul_kernel(sa.unpack(), g, True, False), bs) if need_b else None
        return [ga, gb]

    _attach(out, [a, b], backward)
    return out


def transpose(t: Tensor) -> Tensor:
    if t.ndim < 2:
        raise ValueError("transpose requires a tensor of rank 2 or more")
    _require_cuda(t)
    shape = t._impl.shape
    rows, cols = shape[-2], shape[-1]
    batch = _numel(shape[:-2])
    out_shape = tuple(shape[:-2]) + (cols, rows)
    out = _out(_be().transpose_last2(t._impl.storage, batch, rows, cols), out_shape)
    _attach(out, [t], lambda g: [transpose(g)])
    return out


__all__ = ["Tensor", "NoGradGuard", "no_grad", "grad_enabled", "add", "subtract", "multiply", "divide", "negate",
           "exp", "log", "relu", "sigmoid", "sum_all", "mean_all", "sum_axis", "mean_axis", "max_axis", "max_all",
           "argmax", "argmax_int64", "softmax", "log_softmax", "cross_entropy", "matmul", "transpose"]
_ = math

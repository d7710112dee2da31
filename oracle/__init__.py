"""Parity checkers for the CUDA device -- TEST INFRASTRUCTURE ONLY.

Two interchangeable CPU implementations of VectorCore's float32 hot path,
with identical numpy-level signatures:

* ``port()``  -- the C restatement in ``vc_oracle.c`` (built into
  ``oracle/libvc_oracle.so``); it follows the reference's CPU code
  (src/cpu/cpu_backend.cpp, src/ops.cpp, src/autograd.cpp, src/nn.cpp) step by
  step.
* ``reference()`` -- the reference's own code, compiled from its unmodified
  sources by ``oracle/Makefile`` into ``oracle/_ref/libvcref.so``.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline and
reference legs may use this package. The product (``vectorcore_b200``) never
imports it and has no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "libvc_oracle.so"
REF_DIR = HERE / "_ref"
REF_LIB = REF_DIR / "libvcref.so"

ADD, SUB, MUL, DIV = 0, 1, 2, 3
NEG, RELU, SIGMOID, RELU_GRAD, EXP, LOG = 0, 1, 2, 3, 4, 5
SUM, MAX, ARGMAX = 0, 1, 2

_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)
_szp = ctypes.POINTER(ctypes.c_size_t)


class OracleError(RuntimeError):
    pass


def _c(a, dtype=np.float32):
    """C-contiguous array of `dtype` that keeps 0-d shapes (np.ascontiguousarray
    would promote them to 1-d)."""
    return np.require(np.asarray(a, dtype), requirements="C")


def _fp(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def _shape(shape):
    shape = tuple(int(s) for s in shape)
    arr = (ctypes.c_size_t * max(1, len(shape)))(*shape)
    return arr, len(shape)


def broadcast_shape(a, b):
    return tuple(np.broadcast_shapes(tuple(a), tuple(b)))


def _split(shape, axis):
    rank = len(shape)
    ax = axis + rank if axis < 0 else axis
    outer = int(np.prod(shape[:ax], dtype=np.int64))
    inner = int(np.prod(shape[ax + 1:], dtype=np.int64))
    return outer, int(shape[ax]), inner


class _Impl:
    """Shared numpy wrappers; subclasses bind the C symbols."""

    prefix = ""

    def __init__(self, path: Path):
        if not path.exists():
            raise OracleError(f"oracle library missing: {path} (run `make -C oracle`)")
        self.lib = ctypes.CDLL(str(path))
        self.path = path

    def _fn(self, name):
        return getattr(self.lib, self.prefix + name)

    def _check(self, rc):
        if rc != 0:
            raise OracleError(self._fn("last_error")().decode())

    # ---- elementwise --------------------------------------------------
    def binary(self, op, a, b):
        a = _c(a)
        b = _c(b)
        oshape = broadcast_shape(a.shape, b.shape)
        out = np.empty(oshape, np.float32)
        sa, ra = _shape(a.shape)
        sb, rb = _shape(b.shape)
        so, ro = _shape(oshape)
        self._check(self._fn("binary")(op, _fp(a), sa, ra, _fp(b), sb, rb, _fp(out), so, ro))
        return out

    def unary(self, op, x):
        x = _c(x)
        out = np.empty_like(x)
        self._check(self._fn("unary")(op, _fp(x), _fp(out), ctypes.c_size_t(x.size)) or 0)
        return out

    def sum(self, x):
        x = _c(x)
        return np.float32(self._fn("sum")(_fp(x), ctypes.c_size_t(x.size)))

    def reduce_axis(self, op, x, outer, length, inner):
        x = _c(x)
        out = np.empty(outer * inner, np.float32)
        self._reduce_axis_call(op, x, out, outer, length, inner)
        return out

    def scatter_axis(self, values, indices, outer, length, inner):
        values = _c(values)
        indices = _c(indices)
        out = np.empty(outer * length * inner, np.float32)
        self._fn("scatter_axis")(_fp(values), _fp(indices), _fp(out), ctypes.c_size_t(outer),
                                 ctypes.c_size_t(length), ctypes.c_size_t(inner))
        return out

    def sum_to_shape(self, g, target):
        g = _c(g)
        out = np.empty(tuple(target), np.float32)
        sg, rg = _shape(g.shape)
        st, rt = _shape(target)
        self._check(self._fn("sum_to_shape")(_fp(g), sg, rg, _fp(out), st, rt))
        return out


class Port(_Impl):
    prefix = "vco_"

    def __init__(self, path: Path = PORT_LIB):
        super().__init__(path)
        L = self.lib
        L.vco_last_error.restype = ctypes.c_char_p
        L.vco_sum.restype = ctypes.c_float
        L.vco_unary.restype = None
        L.vco_scatter_axis.restype = None
        L.vco_log_softmax.restype = None
        L.vco_softmax.restype = None
        L.vco_log_softmax_backward.restype = None
        L.vco_softmax_backward.restype = None
        L.vco_unary_backward.restype = None

    def _reduce_axis_call(self, op, x, out, outer, length, inner):
        self._check(self.lib.vco_reduce_axis(op, _fp(x), _fp(out), None, ctypes.c_size_t(outer),
                                             ctypes.c_size_t(length), ctypes.c_size_t(inner)))

    def argmax_i64(self, x, outer, length, inner):
        x = _c(x)
        out = np.empty(outer * inner, np.float32)
        idx = np.empty(outer * inner, np.int64)
        self._check(self.lib.vco_reduce_axis(ARGMAX, _fp(x), _fp(out), idx.ctypes.data_as(_i64p),
                                             ctypes.c_size_t(outer), ctypes.c_size_t(length),
                                             ctypes.c_size_t(inner)))
        return idx

    def binary_backward(self, op, a, b, g, need_a=True, need_b=True):
        a = _c(a)
        b = _c(b)
        g = _c(g)
        da = np.empty(a.shape, np.float32) if need_a else None
        db = np.empty(b.shape, np.float32) if need_b else None
        sa, ra = _shape(a.shape)
        sb, rb = _shape(b.shape)
        self._check(self.lib.vco_binary_backward(op, _fp(a), sa, ra, _fp(b), sb, rb, _fp(g),
                                                 _fp(da), _fp(db)))
        return da, db

    def unary_backward(self, op, x, g):
        x = _c(x)
        g = _c(g)
        y = self.unary(op, x)
        dx = np.empty_like(x)
        self.lib.vco_unary_backward(op, _fp(x), _fp(y), _fp(g), _fp(dx), ctypes.c_size_t(x.size))
        return dx

    def unary_backward_saved(self, op, x, y, g):
        """Backward rule given the forward input x and a caller-supplied
        forward output y (so GPU and CPU use the same saved tensor)."""
        x, y, g = (_c(v) for v in (x, y, g))
        dx = np.empty_like(x)
        self.lib.vco_unary_backward(op, _fp(x), _fp(y), _fp(g), _fp(dx), ctypes.c_size_t(x.size))
        return dx

    def log_softmax(self, x, axis=-1, stats=False):
        x = _c(x)
        outer, length, inner = _split(x.shape, axis)
        out = np.empty_like(x)
        m = np.empty(outer * inner, np.float32)
        s = np.empty(outer * inner, np.float32)
        self.lib.vco_log_softmax(_fp(x), _fp(out), _fp(m), _fp(s), ctypes.c_size_t(outer),
                                 ctypes.c_size_t(length), ctypes.c_size_t(inner))
        return (out, m, s) if stats else out

    def softmax(self, x, axis=-1):
        x = _c(x)
        outer, length, inner = _split(x.shape, axis)
        out = np.empty_like(x)
        self.lib.vco_softmax(_fp(x), _fp(out), ctypes.c_size_t(outer), ctypes.c_size_t(length),
                             ctypes.c_size_t(inner))
        return out

    def log_softmax_backward(self, x, g, axis=-1):
        x = _c(x)
        g = _c(g)
        outer, length, inner = _split(x.shape, axis)
        dx = np.empty_like(x)
        self.lib.vco_log_softmax_backward(_fp(x), _fp(g), _fp(dx), ctypes.c_size_t(outer),
                                          ctypes.c_size_t(length), ctypes.c_size_t(inner))
        return dx

    def softmax_backward(self, x, g, axis=-1):
        x = _c(x)
        g = _c(g)
        outer, length, inner = _split(x.shape, axis)
        dx = np.empty_like(x)
        self.lib.vco_softmax_backward(_fp(x), _fp(g), _fp(dx), ctypes.c_size_t(outer),
                                      ctypes.c_size_t(length), ctypes.c_size_t(inner))
        return dx

    def cross_entropy(self, logits, targets, upstream=1.0, grad=True):
        logits = _c(logits)
        targets = _c(targets, np.int64)
        batch, classes = logits.shape
        loss = ctypes.c_float()
        dx = np.empty_like(logits) if grad else None
        self._check(self.lib.vco_cross_entropy(_fp(logits), ctypes.c_size_t(batch),
                                               ctypes.c_size_t(classes),
                                               targets.ctypes.data_as(_i64p),
                                               ctypes.c_float(upstream), ctypes.byref(loss),
                                               _fp(dx)))
        return np.float32(loss.value), dx

    def reduce_op(self, kind, x, axis=None, g=None):
        """kind: 'sum' | 'mean' | 'max'. Returns (out, dx or None)."""
        x = _c(x)
        k = {"sum": 0, "mean": 1, "max": 2}[kind]
        full = axis is None
        if full:
            oshape = ()
        else:
            ax = axis + x.ndim if axis < 0 else axis
            oshape = x.shape[:ax] + x.shape[ax + 1:]
        out = np.empty(oshape, np.float32)
        dx = None
        if g is not None:
            g = _c(g).reshape(oshape)
            dx = np.empty_like(x)
        s, r = _shape(x.shape)
        self._check(self.lib.vco_reduce_op(k, _fp(x), s, r, int(full), ctypes.c_long(axis or 0),
                                           _fp(out), _fp(g), _fp(dx)))
        return out, dx


class Reference(_Impl):
    prefix = "vcref_"

    def __init__(self, path: Path = REF_LIB):
        super().__init__(path)
        L = self.lib
        L.vcref_last_error.restype = ctypes.c_char_p
        L.vcref_sum.restype = ctypes.c_float
        L.vcref_threads.restype = ctypes.c_size_t
        L.vcref_scatter_axis.restype = None

    def threads(self):
        return int(self.lib.vcref_threads())

    def _reduce_axis_call(self, op, x, out, outer, length, inner):
        self._check(self.lib.vcref_reduce_axis(op, _fp(x), _fp(out), ctypes.c_size_t(outer),
                                               ctypes.c_size_t(length), ctypes.c_size_t(inner)))

    def binary_backward(self, op, a, b, g, need_a=True, need_b=True):
        a = _c(a)
        b = _c(b)
        g = _c(g)
        da = np.empty(a.shape, np.float32) if need_a else None
        db = np.empty(b.shape, np.float32) if need_b else None
        sa, ra = _shape(a.shape)
        sb, rb = _shape(b.shape)
        self._check(self.lib.vcref_binary_backward(op, _fp(a), sa, ra, _fp(b), sb, rb, _fp(g),
                                                   None, _fp(da), _fp(db)))
        return da, db

    def unary_backward(self, op, x, g):
        x = _c(x)
        g = _c(g)
        dx = np.empty_like(x)
        self._check(self.lib.vcref_unary_backward(op, _fp(x), ctypes.c_size_t(x.size), _fp(g),
                                                  None, _fp(dx)))
        return dx

    def _softmax(self, kind, x, axis, g=None):
        x = _c(x)
        out = np.empty_like(x)
        dx = None
        if g is not None:
            g = _c(g)
            dx = np.empty_like(x)
        s, r = _shape(x.shape)
        self._check(self.lib.vcref_softmax_op(kind, _fp(x), s, r, ctypes.c_long(axis), _fp(out),
                                              _fp(g), _fp(dx)))
        return out, dx

    def log_softmax(self, x, axis=-1):
        return self._softmax(0, x, axis)[0]

    def softmax(self, x, axis=-1):
        return self._softmax(1, x, axis)[0]

    def log_softmax_backward(self, x, g, axis=-1):
        return self._softmax(0, x, axis, g)[1]

    def softmax_backward(self, x, g, axis=-1):
        return self._softmax(1, x, axis, g)[1]

    def cross_entropy(self, logits, targets, upstream=1.0, grad=True):
        logits = _c(logits)
        targets = _c(targets, np.int64)
        batch, classes = logits.shape
        loss = ctypes.c_float()
        dx = np.empty_like(logits) if grad else None
        self._check(self.lib.vcref_cross_entropy(_fp(logits), ctypes.c_size_t(batch),
                                                 ctypes.c_size_t(classes),
                                                 targets.ctypes.data_as(_i64p),
                                                 ctypes.c_float(upstream), ctypes.byref(loss),
                                                 _fp(dx)))
        return np.float32(loss.value), dx

    def reduce_op(self, kind, x, axis=None, g=None):
        x = _c(x)
        k = {"sum": 0, "mean": 1, "max": 2, "argmax": 3}[kind]
        full = axis is None
        if full:
            oshape = ()
        else:
            ax = axis + x.ndim if axis < 0 else axis
            oshape = x.shape[:ax] + x.shape[ax + 1:]
        out = np.empty(oshape, np.float32)
        dx = None
        if g is not None:
            g = _c(g).reshape(oshape)
            dx = np.empty_like(x)
        s, r = _shape(x.shape)
        self._check(self.lib.vcref_reduce_op(k, _fp(x), s, r, int(full), ctypes.c_long(axis or 0),
                                             _fp(out), _fp(g), _fp(dx)))
        return out, dx


_port = None
_ref = None


def port() -> Port:
    global _port
    if _port is None:
        _port = Port()
    return _port


def reference_available() -> bool:
    return REF_LIB.exists()


def reference() -> Reference:
    global _ref
    if _ref is None:
        _ref = Reference()
    return _ref


def _configured_reference() -> str:
    """The reference checkout named by the repository's BASELINE.json
    (``reference_path``), used when VECTORCORE_REF is not set."""
    import json

    try:
        return str(json.loads((HERE.parent / "BASELINE.json").read_text()).get("reference_path") or "")
    except (OSError, ValueError):
        return ""


def build(quiet: bool = True) -> None:
    """Compile the restatement and, when the reference checkout is present
    (VECTORCORE_REF, else BASELINE.json's reference_path), the reference's
    own CPU path, its device-slot build and its build with the cuda device
    (``make -C oracle``)."""
    import subprocess

    ref = os.environ.get("VECTORCORE_REF") or _configured_reference()
    # "slot" and "host" link the reference's sources to the CUDA library, so
    # they need vectorcore_b200/_lib/libvc_cuda.so to be built first.
    targets = ["oracle"] + (["ref", "slot", "host"] if ref and Path(ref, "src").is_dir() else [])
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF={ref}", *targets], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)

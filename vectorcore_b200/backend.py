"""CudaBackend: the reference's device-plugin interface, implemented on B200.

The reference routes every non-CPU tensor operation to the abstract
``MetalBackend`` (include/vectorcore/metal_backend.hpp:13-56). ``CudaBackend``
offers the same methods with the same argument meaning -- element counts,
shapes, strides, ``[outer, length, inner]`` axis splits -- and returns
``CudaStorage`` objects (the counterpart of ``Storage``,
include/vectorcore/storage.hpp:11-27), plus the fused entry points the CUDA
device adds (backward rules, sum_to_shape, softmax family, cross-entropy).
All calls go through the C ABI (include/vc_cuda.h); failures raise the
reference's exception types and nothing falls back to the CPU.
"""
from __future__ import annotations

import ctypes
import threading

import numpy as np

from . import _abi
from ._abi import ADD, DIV, MUL, SUB  # noqa: F401  (re-exported op codes)
from ._abi import EXP, LOG, NEG, RELU, RELU_GRAD, SIGMOID  # noqa: F401
from ._abi import REDUCE_ARGMAX, REDUCE_MAX, REDUCE_MEAN, REDUCE_SUM  # noqa: F401

_F32 = 4


class CudaStorage:
    """Device buffer from the stream-ordered pool plus the in-place
    modification counter shared by every view (storage.hpp:22-23).

    ``dtype`` is float32 except for the int64 index / target buffers the
    fused kernels use."""

    __slots__ = ("ptr", "size", "dtype", "version", "__weakref__")

    def __init__(self, elements: int, dtype=np.float32):
        self.dtype = np.dtype(dtype)
        self.size = int(elements)
        self.version = 0
        self.ptr = _abi.alloc(max(self.size, 1) * self.dtype.itemsize)

    @property
    def nbytes(self) -> int:
        return self.size * self.dtype.itemsize

    def bump_version(self) -> None:
        self.version += 1

    def __del__(self):
        ptr, self.ptr = getattr(self, "ptr", 0), 0
        if ptr:
            try:
                _abi.lib.vc_cuda_free(ctypes.c_void_p(ptr))
            except Exception:  # interpreter shutdown
                pass

    def device(self) -> str:
        return "cuda"


def _p(x):
    """Raw device address of a storage (or None)."""
    return None if x is None else ctypes.c_void_p(x.ptr)


class PinnedBuffer:
    """Page-locked host memory (vc_cuda_host_alloc) viewed as a numpy array:
    the host side of the asynchronous transfers."""

    def __init__(self, elements: int, dtype=np.float32):
        self.dtype = np.dtype(dtype)
        self.size = int(elements)
        ptr = ctypes.c_void_p()
        _abi.call("vc_cuda_host_alloc", ctypes.c_size_t(max(self.size, 1) * self.dtype.itemsize), ctypes.byref(ptr))
        self.ptr = ptr.value
        buf = (ctypes.c_char * (self.size * self.dtype.itemsize)).from_address(self.ptr)
        self.array = np.frombuffer(buf, dtype=self.dtype, count=self.size)

    @property
    def nbytes(self) -> int:
        return self.size * self.dtype.itemsize

    def close(self) -> None:
        ptr, self.ptr = getattr(self, "ptr", 0), 0
        if ptr:
            self.array = None
            _abi.lib.vc_cuda_host_free(ctypes.c_void_p(ptr))

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown
            pass


class CudaGraph:
    """A replayable capture of the library stream's work (vc_cuda_graph_*).
    The pool blocks allocated while capturing stay reserved for the graph
    until close(); storages returned by the captured calls are rewritten by
    every replay."""

    def __init__(self, handle: int):
        self._h = ctypes.c_void_p(handle)

    def launch(self) -> None:
        if not self._h.value:
            raise RuntimeError("CudaGraph: launch after close()")
        _abi.call("vc_cuda_graph_launch", self._h)

    @property
    def nodes(self) -> int:
        n = ctypes.c_size_t(0)
        _abi.call("vc_cuda_graph_nodes", self._h, ctypes.byref(n))
        return int(n.value)

    def close(self) -> None:
        if self._h.value:
            _abi.call("vc_cuda_graph_destroy", self._h)
            self._h = ctypes.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CudaBackend:
    _instance = None
    _lock = threading.Lock()

    @classmethod
    def instance(cls) -> "CudaBackend":
        with cls._lock:
            if cls._instance is None:
                cls._instance = cls()
            return cls._instance

    # ---- device ---------------------------------------------------------------
    def available(self) -> bool:
        return _abi.available()

    def device_name(self) -> str:
        return _abi.device_name() if self.available() else "unavailable"

    def last_error(self) -> str:
        return _abi.last_error()

    def synchronize(self) -> None:
        _abi.synchronize()

    def capture(self, fn):
        """Run fn() under stream capture; returns (CudaGraph, fn's result).
        The captured work is NOT executed by the capture itself: launch the
        graph to run it."""
        _abi.call("vc_cuda_graph_begin")
        try:
            result = fn()
        except BaseException:
            h = ctypes.c_void_p(0)
            try:
                _abi.call("vc_cuda_graph_end", ctypes.byref(h))
            finally:
                if h.value:
                    _abi.call("vc_cuda_graph_destroy", h)
            raise
        h = ctypes.c_void_p(0)
        _abi.call("vc_cuda_graph_end", ctypes.byref(h))
        return CudaGraph(h.value), result

    # ---- memory ---------------------------------------------------------------
    def allocate(self, elements: int, dtype=np.float32) -> CudaStorage:
        return CudaStorage(elements, dtype)

    def upload(self, values: np.ndarray) -> CudaStorage:
        values = np.ascontiguousarray(values)
        if values.dtype not in (np.float32, np.int64):
            values = values.astype(np.float32)
        s = CudaStorage(values.size, values.dtype)
        _abi.call("vc_cuda_upload", ctypes.c_void_p(s.ptr), values.ctypes.data_as(ctypes.c_void_p),
                  ctypes.c_size_t(values.nbytes))
        return s

    def download(self, source: CudaStorage, elements: int | None = None) -> np.ndarray:
        n = source.size if elements is None else int(elements)
        if n > source.size:
            raise IndexError("download exceeds storage")
        out = np.empty(n, source.dtype)
        _abi.call("vc_cuda_download", out.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(source.ptr),
                  ctypes.c_size_t(out.nbytes))
        return out

    # ---- asynchronous transfers (vc_cuda_upload_async & co.) --------------------
    def upload_async(self, dst: CudaStorage, src: PinnedBuffer, nbytes: int | None = None) -> int:
        """Copy a pinned host buffer into dst on the upload copy stream; later
        work waits for it only after transfer_wait(ticket)."""
        nb = src.nbytes if nbytes is None else int(nbytes)
        if nb > dst.nbytes or nb > src.nbytes:
            raise IndexError("upload_async exceeds a buffer")
        t = ctypes.c_uint64(0)
        _abi.call("vc_cuda_upload_async", ctypes.c_void_p(dst.ptr), ctypes.c_void_p(src.ptr), ctypes.c_size_t(nb),
                  ctypes.byref(t))
        return int(t.value)

    def download_async(self, dst: PinnedBuffer, src: CudaStorage, nbytes: int | None = None) -> int:
        """Copy src into a pinned host buffer on the download copy stream,
        after the work enqueued so far; read dst after transfer_sync(ticket)."""
        nb = src.nbytes if nbytes is None else int(nbytes)
        if nb > dst.nbytes or nb > src.nbytes:
            raise IndexError("download_async exceeds a buffer")
        t = ctypes.c_uint64(0)
        _abi.call("vc_cuda_download_async", ctypes.c_void_p(dst.ptr), ctypes.c_void_p(src.ptr),
                  ctypes.c_size_t(nb), ctypes.byref(t))
        return int(t.value)

    def transfer_wait(self, ticket: int) -> None:
        _abi.call("vc_cuda_transfer_wait", ctypes.c_uint64(ticket))

    def transfer_sync(self, ticket: int) -> None:
        _abi.call("vc_cuda_transfer_sync", ctypes.c_uint64(ticket))

    # ---- MetalBackend methods ---------------------------------------------------
    def binary(self, a, a_shape, a_strides, b, b_shape, b_strides, out_shape, op) -> CudaStorage:
        out = CudaStorage(int(np.prod(out_shape, dtype=np.int64)))
        sa, ra = _abi.shape_arg(a_shape)
        sb, rb = _abi.shape_arg(b_shape)
        so, ro = _abi.shape_arg(out_shape)
        ta = _abi.shape_arg(a_strides)[0] if a_strides is not None else None
        tb = _abi.shape_arg(b_strides)[0] if b_strides is not None else None
        _abi.call("vc_cuda_binary", op, _p(a), sa, ta, ra, _p(b), sb, tb, rb, _p(out), so, ro)
        return out

    def binary_scalar(self, a, count, scalar, op, scalar_first=False) -> CudaStorage:
        out = CudaStorage(count)
        _abi.call("vc_cuda_binary_scalar", op, _p(a), ctypes.c_float(scalar), int(scalar_first), _p(out),
                  ctypes.c_size_t(count))
        return out

    def unary(self, inp, count, op) -> CudaStorage:
        out = CudaStorage(count)
        _abi.call("vc_cuda_unary", op, _p(inp), _p(out), ctypes.c_size_t(count))
        return out

    def reduce_sum(self, inp, count) -> CudaStorage:
        out = CudaStorage(1)
        _abi.call("vc_cuda_reduce_all", REDUCE_SUM, _p(inp), ctypes.c_size_t(count), _p(out), None)
        return out

    def reduce_all(self, inp, count, op, want_index=False):
        out = CudaStorage(1)
        idx = CudaStorage(1, np.int64) if want_index else None
        _abi.call("vc_cuda_reduce_all", op, _p(inp), ctypes.c_size_t(count), _p(out), _p(idx))
        return (out, idx) if want_index else out

    def reduce_axis(self, inp, outer, length, inner, op, want_index=False):
        """SUM / MEAN / MAX values, or ARGMAX as float indices (the
        reference's convention); want_index also returns int64 indices."""
        out = CudaStorage(outer * inner)
        idx = CudaStorage(outer * inner, np.int64) if want_index else None
        _abi.call("vc_cuda_reduce_axis", op, _p(inp), ctypes.c_size_t(outer), ctypes.c_size_t(length),
                  ctypes.c_size_t(inner), _p(out), _p(idx))
        return (out, idx) if want_index else out

    def scatter_axis(self, values, indices, outer, length, inner) -> CudaStorage:
        out = CudaStorage(outer * length * inner)
        f32 = indices if indices.dtype == np.float32 else None
        i64 = indices if indices.dtype == np.int64 else None
        _abi.call("vc_cuda_scatter_axis", _p(values), _p(f32), _p(i64), _p(out), ctypes.c_size_t(outer),
                  ctypes.c_size_t(length), ctypes.c_size_t(inner))
        return out

    def axpy_inplace(self, target, source, count, alpha) -> None:
        _abi.call("vc_cuda_axpy", _p(target), _p(source), ctypes.c_size_t(count), ctypes.c_float(alpha))

    def matmul(self, a, b, m, k, n, a_offsets, b_offsets, trans_a=False, trans_b=False) -> CudaStorage:
        if len(a_offsets) != len(b_offsets) or not a_offsets:
            raise ValueError("matmul needs one A and B offset per batch")
        batch = len(a_offsets)
        out = CudaStorage(batch * m * n)
        ao = (ctypes.c_size_t * batch)(*[int(v) for v in a_offsets])
        bo = (ctypes.c_size_t * batch)(*[int(v) for v in b_offsets])
        _abi.call("vc_cuda_matmul", _p(a), _p(b), _p(out), ctypes.c_size_t(m), ctypes.c_size_t(k),
                  ctypes.c_size_t(n), ao, bo, ctypes.c_size_t(batch), int(trans_a), int(trans_b))
        return out

    def transpose_last2(self, inp, batch, rows, cols) -> CudaStorage:
        out = CudaStorage(batch * rows * cols)
        _abi.call("vc_cuda_transpose_last2", _p(inp), _p(out), ctypes.c_size_t(batch), ctypes.c_size_t(rows),
                  ctypes.c_size_t(cols))
        return out

    # ---- fused entry points of the CUDA device ---------------------------------------
    def fill(self, count, value) -> CudaStorage:
        out = CudaStorage(count)
        _abi.call("vc_cuda_fill", _p(out), ctypes.c_size_t(count), ctypes.c_float(value))
        return out

    def copy(self, src: CudaStorage) -> CudaStorage:
        out = CudaStorage(src.size, src.dtype)
        _abi.call("vc_cuda_copy", _p(out), _p(src), ctypes.c_size_t(src.nbytes))
        return out

    def unary_backward(self, op, x, y, g, count) -> CudaStorage:
        out = CudaStorage(count)
        _abi.call("vc_cuda_unary_backward", op, _p(x), _p(y), _p(g), _p(out), ctypes.c_size_t(count))
        return out

    def broadcast_to(self, value, v_shape, t_shape) -> CudaStorage:
        out = CudaStorage(int(np.prod(t_shape, dtype=np.int64)))
        sv, rv = _abi.shape_arg(v_shape)
        st, rt = _abi.shape_arg(t_shape)
        _abi.call("vc_cuda_broadcast_to", _p(value), sv, rv, _p(out), st, rt)
        return out

    def sum_to_shape(self, g, g_shape, t_shape) -> CudaStorage:
        out = CudaStorage(int(np.prod(t_shape, dtype=np.int64)))
        sg, rg = _abi.shape_arg(g_shape)
        st, rt = _abi.shape_arg(t_shape)
        _abi.call("vc_cuda_sum_to_shape", _p(g), sg, rg, _p(out), st, rt)
        return out

    def binary_backward(self, op, a, a_shape, b, b_shape, g, g_shape, need_a=True, need_b=True):
        da = CudaStorage(int(np.prod(a_shape, dtype=np.int64))) if need_a else None
        db = CudaStorage(int(np.prod(b_shape, dtype=np.int64))) if need_b else None
        sa, ra = _abi.shape_arg(a_shape)
        sb, rb = _abi.shape_arg(b_shape)
        sg, rg = _abi.shape_arg(g_shape)
        _abi.call("vc_cuda_binary_backward", op, _p(a), sa, ra, _p(b), sb, rb, _p(g), sg, rg, _p(da), _p(db))
        return da, db

    def reduce_axis_backward(self, op, g, indices, outer, length, inner) -> CudaStorage:
        out = CudaStorage(outer * length * inner)
        _abi.call("vc_cuda_reduce_axis_backward", op, _p(g), _p(indices), _p(out), ctypes.c_size_t(outer),
                  ctypes.c_size_t(length), ctypes.c_size_t(inner))
        return out

    def softmax(self, x, outer, length, inner, log=False, stats=True):
        y = CudaStorage(outer * length * inner)
        m = CudaStorage(outer * inner) if stats else None
        s = CudaStorage(outer * inner) if stats else None
        _abi.call("vc_cuda_log_softmax" if log else "vc_cuda_softmax", _p(x), _p(y), _p(m), _p(s),
                  ctypes.c_size_t(outer), ctypes.c_size_t(length), ctypes.c_size_t(inner))
        return y, m, s

    def softmax_backward(self, x, m, s, g, outer, length, inner, log=False) -> CudaStorage:
        dx = CudaStorage(outer * length * inner)
        _abi.call("vc_cuda_log_softmax_backward" if log else "vc_cuda_softmax_backward", _p(x), _p(m), _p(s),
                  _p(g), _p(dx), ctypes.c_size_t(outer), ctypes.c_size_t(length), ctypes.c_size_t(inner))
        return dx

    def cross_entropy(self, logits, targets, batch, classes, batch_total=0):
        loss = CudaStorage(1)
        m = CudaStorage(batch)
        s = CudaStorage(batch)
        part = CudaStorage(1, np.float64)
        _abi.call("vc_cuda_cross_entropy", _p(logits), _p(targets), ctypes.c_size_t(batch),
                  ctypes.c_size_t(classes), ctypes.c_size_t(batch_total), _p(loss), _p(m), _p(s), _p(part))
        return loss, m, s, part

    def cross_entropy_backward(self, logits, targets, m, s, upstream, batch, classes, batch_total=0):
        dx = CudaStorage(batch * classes)
        _abi.call("vc_cuda_cross_entropy_backward", _p(logits), _p(targets), _p(m), _p(s), _p(upstream),
                  ctypes.c_size_t(batch), ctypes.c_size_t(classes), ctypes.c_size_t(batch_total), _p(dx))
        return dx

    # ---- fused chain relu(x + b).sum() (one launch each way) ----------------
    def bias_relu_sum(self, x, b, rows, cols):
        """loss storage (1 element) = relu(x + b).sum() for x [rows, cols], b [cols]."""
        loss = CudaStorage(1)
        _abi.call("vc_cuda_bias_relu_sum", _p(x), _p(b), ctypes.c_size_t(rows), ctypes.c_size_t(cols), _p(loss),
                  None)
        return loss

    def bias_relu_sum_backward(self, x, b, upstream, rows, cols):
        """(dx, db) of relu(x + b).sum() given the upstream scalar gradient."""
        dx = CudaStorage(rows * cols)
        db = CudaStorage(cols)
        _abi.call("vc_cuda_bias_relu_sum_backward", _p(x), _p(b), _p(upstream), ctypes.c_size_t(rows),
                  ctypes.c_size_t(cols), _p(dx), _p(db), None)
        return dx, db

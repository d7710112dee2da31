"""ctypes binding of the C ABI in include/vc_cuda.h (libvc_cuda.so).

This is the Python side of the drop-in boundary: the same entry points a C++
host binds. Status codes become the exception types the reference's pybind11
module raises for the corresponding C++ exceptions (std::invalid_argument ->
ValueError, std::out_of_range -> IndexError, std::overflow_error ->
OverflowError, std::runtime_error -> RuntimeError), with the message from
vc_cuda_last_error().

There is no fallback: if the library is missing, importing this module
raises ImportError.
"""
from __future__ import annotations

import ctypes
import re
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

from . import build as _build

LIB_PATH = _build.library_path()
HEADER = _build.INCLUDE / "vc_cuda.h"

if not LIB_PATH.exists():
    raise ImportError(
        f"vectorcore_b200: the CUDA device library {LIB_PATH} is not built; run "
        "`python vectorcore_b200/build.py` (nvcc for sm_100a). There is no CPU fallback.")

lib = ctypes.CDLL(str(LIB_PATH))

VC_OK, VC_ERR_INVALID, VC_ERR_OUT_OF_RANGE, VC_ERR_OVERFLOW = 0, 1, 2, 3
VC_ERR_RUNTIME, VC_ERR_OOM, VC_ERR_TIMEOUT = 4, 5, 6

ADD, SUB, MUL, DIV = 0, 1, 2, 3
NEG, RELU, SIGMOID, RELU_GRAD, EXP, LOG = 0, 1, 2, 3, 4, 5
REDUCE_SUM, REDUCE_MAX, REDUCE_ARGMAX, REDUCE_MEAN = 0, 1, 2, 3


class CudaDeviceError(RuntimeError):
    """A failure reported by the CUDA device (RuntimeError, like the reference)."""

    def __init__(self, status, message):
        super().__init__(message)
        self.status = status


class DeviceOutOfMemory(CudaDeviceError):
    pass


class DeviceTimeout(CudaDeviceError):
    pass


_EXC = {
    VC_ERR_INVALID: ValueError,
    VC_ERR_OUT_OF_RANGE: IndexError,
    VC_ERR_OVERFLOW: OverflowError,
}

_szp = POINTER(c_size_t)
_f = c_void_p  # device float* (raw address)

_SIGS = {
    "vc_cuda_available": (c_int, []),
    "vc_cuda_init": (c_int, [c_int]),
    "vc_cuda_last_error": (c_char_p, []),
    "vc_cuda_device_name": (c_int, [c_char_p, c_size_t]),
    "vc_cuda_synchronize": (c_int, []),
    "vc_cuda_stream": (c_void_p, []),
    "vc_cuda_set_stream": (c_int, [c_void_p]),
    "vc_cuda_sm_count": (c_int, []),
    "vc_cuda_alloc": (c_int, [c_size_t, POINTER(c_void_p)]),
    "vc_cuda_free": (c_int, [c_void_p]),
    "vc_cuda_pool_stats": (c_int, [_szp, _szp, _szp, _szp]),
    "vc_cuda_pool_trim": (c_int, []),
    "vc_cuda_host_alloc": (c_int, [c_size_t, POINTER(c_void_p)]),
    "vc_cuda_host_free": (c_int, [c_void_p]),
    "vc_cuda_upload": (c_int, [c_void_p, c_void_p, c_size_t]),
    "vc_cuda_download": (c_int, [c_void_p, c_void_p, c_size_t]),
    "vc_cuda_upload_async": (c_int, [c_void_p, c_void_p, c_size_t, POINTER(c_uint64)]),
    "vc_cuda_download_async": (c_int, [c_void_p, c_void_p, c_size_t, POINTER(c_uint64)]),
    "vc_cuda_transfer_wait": (c_int, [c_uint64]),
    "vc_cuda_transfer_sync": (c_int, [c_uint64]),
    "vc_cuda_copy": (c_int, [c_void_p, c_void_p, c_size_t]),
    "vc_cuda_fill": (c_int, [_f, c_size_t, c_float]),
    "vc_cuda_binary": (c_int, [c_int, _f, _szp, _szp, c_int, _f, _szp, _szp, c_int, _f, _szp, c_int]),
    "vc_cuda_binary_scalar": (c_int, [c_int, _f, c_float, c_int, _f, c_size_t]),
    "vc_cuda_unary": (c_int, [c_int, _f, _f, c_size_t]),
    "vc_cuda_unary_backward": (c_int, [c_int, _f, _f, _f, _f, c_size_t]),
    "vc_cuda_broadcast_to": (c_int, [_f, _szp, c_int, _f, _szp, c_int]),
    "vc_cuda_axpy": (c_int, [_f, _f, c_size_t, c_float]),
    "vc_cuda_sum_to_shape": (c_int, [_f, _szp, c_int, _f, _szp, c_int]),
    "vc_cuda_binary_backward": (c_int, [c_int, _f, _szp, c_int, _f, _szp, c_int, _f, _szp, c_int, _f, _f]),
    "vc_cuda_reduce_all": (c_int, [c_int, _f, c_size_t, _f, c_void_p]),
    "vc_cuda_reduce_axis": (c_int, [c_int, _f, c_size_t, c_size_t, c_size_t, _f, c_void_p]),
    "vc_cuda_scatter_axis": (c_int, [_f, _f, c_void_p, _f, c_size_t, c_size_t, c_size_t]),
    "vc_cuda_reduce_axis_backward": (c_int, [c_int, _f, c_void_p, _f, c_size_t, c_size_t, c_size_t]),
    "vc_cuda_log_softmax": (c_int, [_f, _f, _f, _f, c_size_t, c_size_t, c_size_t]),
    "vc_cuda_softmax": (c_int, [_f, _f, _f, _f, c_size_t, c_size_t, c_size_t]),
    "vc_cuda_log_softmax_backward": (c_int, [_f, _f, _f, _f, _f, c_size_t, c_size_t, c_size_t]),
    "vc_cuda_softmax_backward": (c_int, [_f, _f, _f, _f, _f, c_size_t, c_size_t, c_size_t]),
    "vc_cuda_cross_entropy": (c_int, [_f, c_void_p, c_size_t, c_size_t, c_size_t, _f, _f, _f, c_void_p]),
    "vc_cuda_cross_entropy_backward": (c_int, [_f, c_void_p, _f, _f, _f, c_size_t, c_size_t, c_size_t, _f]),
    "vc_cuda_bias_relu_sum": (c_int, [_f, _f, c_size_t, c_size_t, _f, c_void_p]),
    "vc_cuda_graph_begin": (c_int, []),
    "vc_cuda_graph_end": (c_int, [POINTER(c_void_p)]),
    "vc_cuda_graph_launch": (c_int, [c_void_p]),
    "vc_cuda_graph_nodes": (c_int, [c_void_p, POINTER(c_size_t)]),
    "vc_cuda_graph_destroy": (c_int, [c_void_p]),
    "vc_cuda_bias_relu_sum_backward": (c_int, [_f, _f, _f, c_size_t, c_size_t, _f, _f, c_void_p]),
    "vc_cuda_matmul": (c_int, [_f, _f, _f, c_size_t, c_size_t, c_size_t, _szp, _szp, c_size_t, c_int, c_int]),
    "vc_cuda_transpose_last2": (c_int, [_f, _f, c_size_t, c_size_t, c_size_t]),
    "vc_cuda_reduce_sum_noalloc": (c_int, [_f, c_size_t, _f]),
    "vc_cuda_selftest_wait_timeout": (c_int, [c_int64]),
    "vc_cuda_reduce_axis_partial": (c_int, [c_int, _f, c_size_t, c_size_t, c_size_t, c_int64, c_int, c_void_p,
                                            _f, c_void_p]),
    "vc_cuda_binary_backward_partial": (c_int, [c_int, _f, _szp, c_int, _f, _szp, c_int, _f, _szp, c_int, c_void_p,
                                                c_void_p]),
    "vc_cuda_combine_partials": (c_int, [c_int, c_void_p, _f, c_void_p, c_int, c_size_t, c_float, c_int, _f,
                                         c_void_p]),
    "vc_cuda_comm_unique_id": (c_int, [c_void_p, c_size_t]),
    "vc_cuda_comm_init": (c_int, [c_int, c_int, c_void_p, c_size_t, c_int]),
    "vc_cuda_comm_allgather": (c_int, [c_void_p, c_void_p, c_size_t]),
    "vc_cuda_comm_allgather_group": (c_int, [POINTER(c_void_p), POINTER(c_void_p), _szp, c_int]),
    "vc_cuda_comm_synchronize": (c_int, [c_int]),
    "vc_cuda_comm_destroy": (c_int, []),
    "vc_cuda_comm_size": (c_int, []),
    "vc_cuda_comm_rank": (c_int, []),
}


def header_symbols() -> list[str]:
    """Every entry point declared in include/vc_cuda.h."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(vc_cuda_\w+)\s*\(", text)))


for _name, (_res, _args) in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


def last_error() -> str:
    msg = lib.vc_cuda_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str = "") -> None:
    if status == VC_OK:
        return
    msg = last_error() or what
    if status in _EXC:
        raise _EXC[status](msg)
    if status == VC_ERR_OOM:
        raise DeviceOutOfMemory(status, msg)
    if status == VC_ERR_TIMEOUT:
        raise DeviceTimeout(status, msg)
    raise CudaDeviceError(status, msg)


def call(name: str, *args) -> None:
    check(getattr(lib, name)(*args), name)


def shape_arg(shape):
    shape = [int(s) for s in shape]
    return (c_size_t * max(1, len(shape)))(*shape), len(shape)


def available() -> bool:
    return bool(lib.vc_cuda_available())


def device_name() -> str:
    buf = ctypes.create_string_buffer(256)
    check(lib.vc_cuda_device_name(buf, 256))
    return buf.value.decode()


def synchronize() -> None:
    check(lib.vc_cuda_synchronize())


def alloc(nbytes: int) -> int:
    p = c_void_p()
    check(lib.vc_cuda_alloc(c_size_t(nbytes), ctypes.byref(p)))
    return int(p.value or 0)


def free(ptr: int) -> None:
    check(lib.vc_cuda_free(c_void_p(ptr)))


def pool_stats() -> dict:
    vals = [c_size_t() for _ in range(4)]
    check(lib.vc_cuda_pool_stats(*[ctypes.byref(v) for v in vals]))
    return dict(zip(("cached_bytes", "in_use_bytes", "hits", "misses"), (v.value for v in vals)))


__all__ = ["lib", "check", "call", "shape_arg", "available", "device_name", "synchronize", "alloc",
           "free", "pool_stats", "header_symbols", "last_error", "CudaDeviceError",
           "DeviceOutOfMemory", "DeviceTimeout"]
_ = (c_double, c_int64, Path)

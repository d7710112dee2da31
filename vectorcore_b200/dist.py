"""Leading-axis sharding across the GPUs of one box (one process per GPU).

The reference is single-device; this is the multi-GPU path of the CUDA
device. A global tensor of R rows is split into contiguous, balanced row
shards (``RowShard``), rank r holding rows [start, stop). Elementwise and
broadcast ops need no communication. A reduction over the sharded axis
computes an unrounded per-rank partial on the device, all-gathers the
partials over NCCL (NVLink / NVSwitch) and combines them in rank order
0..R-1 on every rank (``vc_cuda_combine_partials``), so the result is the
same on every rank and independent of the collective's internal order.
Reductions along other axes, softmax rows and the per-row work of
cross-entropy stay local.

``Communicator.from_torch()`` bootstraps the NCCL communicator through an
initialised ``torch.distributed`` process group (any backend -- the 128-byte
id is all that travels over it).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _abi
from . import backend as _B
from .backend import CudaBackend, CudaStorage
from .tensor import Tensor, _attach, _out, _require_cuda

UNIQUE_ID_BYTES = 128


@dataclass(frozen=True)
class RowShard:
    """Rows [start, stop) of a global extent `rows` owned by `rank` of
    `world`: contiguous, in rank order, the first rows % world ranks holding
    one extra row."""

    rows: int
    world: int
    rank: int

    def __post_init__(self):
        if self.world < 1 or not 0 <= self.rank < self.world or self.rows < 0:
            raise ValueError(f"bad shard: rows={self.rows} world={self.world} rank={self.rank}")

    @property
    def start(self) -> int:
        base, extra = divmod(self.rows, self.world)
        return self.rank * base + min(self.rank, extra)

    @property
    def count(self) -> int:
        base, extra = divmod(self.rows, self.world)
        return base + (1 if self.rank < extra else 0)

    @property
    def stop(self) -> int:
        return self.start + self.count


def exchange_unique_id(make_id, group=None) -> bytes:
    """Rank 0 calls make_id(); every rank returns its bytes (torch.distributed
    broadcast of a Python object over the given group)."""
    import torch.distributed as dist

    obj = [make_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
    return obj[0]


class Communicator:
    """The CUDA device's NCCL communicator (one per process)."""

    def __init__(self, world: int, rank: int, unique_id: bytes, timeout_ms: int = 60_000):
        if len(unique_id) != UNIQUE_ID_BYTES:
            raise ValueError("the NCCL unique id is 128 bytes")
        buf = ctypes.create_string_buffer(unique_id, UNIQUE_ID_BYTES)
        _abi.call("vc_cuda_comm_init", world, rank, buf, UNIQUE_ID_BYTES, timeout_ms)
        self.world, self.rank, self.timeout_ms = world, rank, timeout_ms

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(UNIQUE_ID_BYTES)
        _abi.call("vc_cuda_comm_unique_id", buf, UNIQUE_ID_BYTES)
        return buf.raw

    @classmethod
    def from_torch(cls, group=None, timeout_ms: int = 60_000) -> "Communicator":
        import torch.distributed as dist

        uid = exchange_unique_id(cls.unique_id, group)
        return cls(dist.get_world_size(group), dist.get_rank(group), uid, timeout_ms)

    def allgather(self, send: CudaStorage, nbytes: int, dtype=np.uint8) -> CudaStorage:
        itemsize = np.dtype(dtype).itemsize
        recv = CudaStorage(self.world * nbytes // itemsize, dtype)
        _abi.call("vc_cuda_comm_allgather", ctypes.c_void_p(send.ptr), ctypes.c_void_p(recv.ptr),
                  ctypes.c_size_t(nbytes))
        return recv

    def synchronize(self, timeout_ms: int | None = None) -> None:
        _abi.call("vc_cuda_comm_synchronize", int(timeout_ms or self.timeout_ms))

    def close(self) -> None:
        _abi.call("vc_cuda_comm_destroy")


def _be() -> CudaBackend:
    return CudaBackend.instance()


def _p(s):
    return None if s is None else ctypes.c_void_p(s.ptr)


def _sum_over_shards(comm: Communicator, partial: CudaStorage, count: int, divisor: float = 0.0,
                     negate: bool = False) -> CudaStorage:
    gathered = comm.allgather(partial, count * 8, np.float64)
    out = CudaStorage(count)
    _abi.call("vc_cuda_combine_partials", _B.REDUCE_SUM, _p(gathered), None, None, comm.world,
              ctypes.c_size_t(count), ctypes.c_float(divisor), int(negate), _p(out), None)
    return out


def sum_axis0(x: Tensor, comm: Communicator, mean_rows: int = 0) -> Tensor:
    """Sum (or mean over `mean_rows` global rows) of the row-sharded `x` over
    its leading axis; the same result on every rank. Backward: the upstream
    gradient broadcast to this rank's rows (no communication)."""
    _require_cuda(x)
    be = _be()
    shape = x._impl.shape
    rows_local, rest = shape[0], tuple(shape[1:])
    count = int(np.prod(rest, dtype=np.int64))
    partial = CudaStorage(count, np.float64)
    _abi.call("vc_cuda_reduce_axis_partial", _B.REDUCE_SUM, _p(x._impl.storage), ctypes.c_size_t(1),
              ctypes.c_size_t(rows_local), ctypes.c_size_t(count), ctypes.c_int64(0), 0, _p(partial), None, None)
    out = _out(_sum_over_shards(comm, partial, count, float(mean_rows) if mean_rows else 0.0), rest)
    op = _B.REDUCE_MEAN if mean_rows else _B.REDUCE_SUM

    def backward(g):
        if mean_rows:
            # g / R_global then broadcast: scale by the GLOBAL row count
            scaled = be.binary_scalar(g._impl.storage, count, float(mean_rows), _B.DIV)
            return [_out(be.reduce_axis_backward(_B.REDUCE_SUM, scaled, None, 1, rows_local, count), shape)]
        return [_out(be.reduce_axis_backward(op, g._impl.storage, None, 1, rows_local, count), shape)]

    _attach(out, [x], backward)
    return out


def max_axis0(x: Tensor, comm: Communicator, shard: RowShard):
    """Max over the sharded leading axis and its global argmax (int64 numpy
    array), with the reference's scan semantics across shards (first maximal
    row wins; a NaN only wins at global row 0). Not differentiable here."""
    _require_cuda(x)
    shape = x._impl.shape
    rows_local, rest = shape[0], tuple(shape[1:])
    count = int(np.prod(rest, dtype=np.int64))
    pv, pi = CudaStorage(count), CudaStorage(count, np.int64)
    _abi.call("vc_cuda_reduce_axis_partial", _B.REDUCE_MAX, _p(x._impl.storage), ctypes.c_size_t(1),
              ctypes.c_size_t(rows_local), ctypes.c_size_t(count), ctypes.c_int64(shard.start),
              int(shard.rank > 0), None, _p(pv), _p(pi))
    gv = comm.allgather(pv, count * 4, np.float32)
    gi = comm.allgather(pi, count * 8, np.int64)
    out, idx = CudaStorage(count), CudaStorage(count, np.int64)
    _abi.call("vc_cuda_combine_partials", _B.REDUCE_MAX, None, _p(gv), _p(gi), comm.world, ctypes.c_size_t(count),
              ctypes.c_float(0.0), 0, _p(out), _p(idx))
    return _out(out, rest), _be().download(idx).reshape(rest)


def sum_all(x: Tensor, comm: Communicator, mean_numel: int = 0) -> Tensor:
    """Sum (or mean over `mean_numel` global elements) of every element of the
    sharded tensor. Backward: the upstream broadcast over this rank's shard."""
    _require_cuda(x)
    be = _be()
    n = x.numel
    partial = CudaStorage(1, np.float64)
    _abi.call("vc_cuda_reduce_axis_partial", _B.REDUCE_SUM, _p(x._impl.storage), ctypes.c_size_t(1),
              ctypes.c_size_t(n), ctypes.c_size_t(1), ctypes.c_int64(0), 0, _p(partial), None, None)
    out = _out(_sum_over_shards(comm, partial, 1, float(mean_numel) if mean_numel else 0.0), ())
    shape = x._impl.shape

    def backward(g):
        gs = g._impl.storage
        if mean_numel:
            gs = be.binary_scalar(gs, 1, float(mean_numel), _B.DIV)
        return [_out(be.reduce_axis_backward(_B.REDUCE_SUM, gs, None, 1, n, 1), shape)]

    _attach(out, [x], backward)
    return out


def cross_entropy(logits: Tensor, targets, comm: Communicator, global_batch: int) -> Tensor:
    """Mean softmax cross-entropy over a row-sharded batch: each rank's row
    terms are summed on the device, the per-rank sums are combined in rank
    order, and loss = -(sum) / global_batch. Backward is local (each row's
    gradient needs only its own logits and the global batch size)."""
    if logits.ndim != 2:
        raise ValueError(f"cross_entropy expects [batch, classes] logits, got {logits.shape}")
    _require_cuda(logits)
    be = _be()
    batch, classes = logits._impl.shape
    tg = np.asarray(targets).astype(np.int64)
    if tg.shape != (batch,):
        raise ValueError(f"cross_entropy received {tg.size} targets for a batch of {batch}")
    bad = (tg < 0) | (tg >= classes)
    if bad.any():
        raise IndexError(f"target class {int(tg[bad][0])} is out of range for {classes} classes")
    dt = be.upload(tg)
    _, m, s, part = be.cross_entropy(logits._impl.storage, dt, batch, classes, global_batch)
    out = _out(_sum_over_shards(comm, part, 1, float(global_batch), negate=True), ())
    x = logits.detach()

    def backward(g):
        return [_out(be.cross_entropy_backward(x._impl.storage, dt, m, s, g._impl.storage, batch, classes,
                                               global_batch), (batch, classes))]

    _attach(out, [logits], backward)
    return out


__all__ = ["RowShard", "Communicator", "exchange_unique_id", "sum_axis0", "max_axis0", "sum_all", "cross_entropy"]

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

The functions work at the device-plugin level (``CudaStorage`` + shapes, like
``backend.CudaBackend``): each returns the combined result, identical on
every rank, and the backward of a sharded reduction needs no communication
(the upstream gradient is broadcast over the rank's own rows). Every rank
must make the same calls in the same order: each is a collective.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _abi
from . import backend as _B
from .backend import CudaBackend, CudaStorage

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

    def allgather_group(self, items) -> list:
        """Several all-gathers as ONE NCCL group (one launch): items are
        (send storage, bytes per rank, dtype); returns the receive storages
        ([world * bytes] each, rank-major)."""
        recvs = [CudaStorage(self.world * nb // np.dtype(dt).itemsize, dt) for _, nb, dt in items]
        n = len(items)
        sends = (ctypes.c_void_p * n)(*[s.ptr for s, _, _ in items])
        rps = (ctypes.c_void_p * n)(*[r.ptr for r in recvs])
        sizes = (ctypes.c_size_t * n)(*[nb for _, nb, _ in items])
        _abi.call("vc_cuda_comm_allgather_group", sends, rps, sizes, n)
        return recvs

    def synchronize(self, timeout_ms: int | None = None) -> None:
        _abi.call("vc_cuda_comm_synchronize", int(timeout_ms or self.timeout_ms))

    def close(self) -> None:
        _abi.call("vc_cuda_comm_destroy")


def _be() -> CudaBackend:
    return CudaBackend.instance()


def _p(s):
    return None if s is None else ctypes.c_void_p(s.ptr)


def _combine_sum(world: int, gathered: CudaStorage, count: int, divisor: float = 0.0,
                 negate: bool = False) -> CudaStorage:
    out = CudaStorage(count)
    _abi.call("vc_cuda_combine_partials", _B.REDUCE_SUM, _p(gathered), None, None, world, ctypes.c_size_t(count),
              ctypes.c_float(divisor), int(negate), _p(out), None)
    return out


def _combine_max(world: int, gv: CudaStorage, gi: CudaStorage, count: int):
    out, idx = CudaStorage(count), CudaStorage(count, np.int64)
    _abi.call("vc_cuda_combine_partials", _B.REDUCE_MAX, None, _p(gv), _p(gi), world, ctypes.c_size_t(count),
              ctypes.c_float(0.0), 0, _p(out), _p(idx))
    return out, idx


def _combine_sums(comm: Communicator, partial: CudaStorage, count: int, divisor: float = 0.0,
                  negate: bool = False) -> CudaStorage:
    """All-gather `count` double partials per rank and add them in rank order."""
    return _combine_sum(comm.world, comm.allgather(partial, count * 8, np.float64), count, divisor, negate)


def _partial_sum(x: CudaStorage, rows_local: int, count: int) -> CudaStorage:
    partial = CudaStorage(count, np.float64)
    _abi.call("vc_cuda_reduce_axis_partial", _B.REDUCE_SUM, _p(x), ctypes.c_size_t(1), ctypes.c_size_t(rows_local),
              ctypes.c_size_t(count), ctypes.c_int64(0), 0, _p(partial), None, None)
    return partial


def _partial_max(x: CudaStorage, rows_local: int, count: int, shard: RowShard):
    pv, pi = CudaStorage(count), CudaStorage(count, np.int64)
    _abi.call("vc_cuda_reduce_axis_partial", _B.REDUCE_MAX, _p(x), ctypes.c_size_t(1), ctypes.c_size_t(rows_local),
              ctypes.c_size_t(count), ctypes.c_int64(shard.start), int(shard.rank > 0), None, _p(pv), _p(pi))
    return pv, pi


def sum_axis0(x: CudaStorage, rows_local: int, count: int, comm: Communicator, mean_rows: int = 0) -> CudaStorage:
    """Sum (or the mean over `mean_rows` global rows) over the sharded leading
    axis of x [rows_local, count]: [count] floats, the same on every rank.
    The backward is local: ``sum_axis0_backward``."""
    return _combine_sums(comm, _partial_sum(x, rows_local, count), count, float(mean_rows) if mean_rows else 0.0)


def sum_axis0_backward(g: CudaStorage, rows_local: int, count: int, mean_rows: int = 0) -> CudaStorage:
    """dx [rows_local, count] of sum_axis0 for the upstream g [count]: g + 0
    broadcast over this rank's rows (g / R_global + 0 for the mean, scaled by
    the GLOBAL row count)."""
    be = _be()
    if mean_rows:
        g = be.binary_scalar(g, count, float(mean_rows), _B.DIV)
    return be.reduce_axis_backward(_B.REDUCE_SUM, g, None, 1, rows_local, count)


def max_axis0(x: CudaStorage, rows_local: int, count: int, comm: Communicator, shard: RowShard):
    """Max over the sharded leading axis of x [rows_local, count] and its
    global argmax (int64), with the reference's scan semantics across
    shards: the first maximal row wins (a lower rank wins ties) and a NaN
    only wins at global row 0. Returns (values [count], indices [count])."""
    pv, pi = _partial_max(x, rows_local, count, shard)
    gv, gi = comm.allgather_group([(pv, count * 4, np.float32), (pi, count * 8, np.int64)])
    return _combine_max(comm.world, gv, gi, count)


def sum_all(x: CudaStorage, n_local: int, comm: Communicator, mean_numel: int = 0) -> CudaStorage:
    """Sum (or the mean over `mean_numel` global elements) of every element
    of the sharded tensor: one float, the same on every rank. The backward is
    the upstream broadcast over this rank's shard (``broadcast_to``)."""
    return _combine_sums(comm, _partial_total(x, n_local), 1, float(mean_numel) if mean_numel else 0.0)


def _partial_total(x: CudaStorage, n_local: int) -> CudaStorage:
    partial = CudaStorage(1, np.float64)
    _abi.call("vc_cuda_reduce_axis_partial", _B.REDUCE_SUM, _p(x), ctypes.c_size_t(1), ctypes.c_size_t(n_local),
              ctypes.c_size_t(1), ctypes.c_int64(0), 0, _p(partial), None, None)
    return partial


def axis0_reductions(x: CudaStorage, rows_local: int, count: int, comm: Communicator, shard: RowShard):
    """The axis-0 sum, the axis-0 max with its argmax and the full sum of the
    row-sharded x [rows_local, count] with ONE grouped all-gather of the
    four partials (one NCCL launch per call instead of four). Returns
    (sum [count], (max [count], argmax int64 [count]), total [1]), each the
    same on every rank and equal to the separate calls' results."""
    ps = _partial_sum(x, rows_local, count)
    pv, pi = _partial_max(x, rows_local, count, shard)
    pt = _partial_total(x, rows_local * count)
    gs, gv, gi, gt = comm.allgather_group([(ps, count * 8, np.float64), (pv, count * 4, np.float32),
                                           (pi, count * 8, np.int64), (pt, 8, np.float64)])
    return _combine_sum(comm.world, gs, count), _combine_max(comm.world, gv, gi, count), \
        _combine_sum(comm.world, gt, 1)


def cross_entropy(logits: CudaStorage, targets: CudaStorage, batch_local: int, classes: int,
                  comm: Communicator, global_batch: int):
    """Mean softmax cross-entropy over a row-sharded batch: each rank's row
    terms are summed on the device, the per-rank sums combined in rank order,
    loss = -(sum) / global_batch. Returns (loss, row_max, row_sum); the
    backward is local: ``cross_entropy_backward`` with the same
    global_batch."""
    _, m, s, part = _be().cross_entropy(logits, targets, batch_local, classes, global_batch)
    return _combine_sums(comm, part, 1, float(global_batch), negate=True), m, s


def cross_entropy_backward(logits, targets, row_max, row_sum, upstream, batch_local, classes, global_batch):
    return _be().cross_entropy_backward(logits, targets, row_max, row_sum, upstream, batch_local, classes,
                                        global_batch)


def binary_backward(op: int, a: CudaStorage, a_shape, b: CudaStorage, b_shape, g: CudaStorage, g_shape,
                    comm: Communicator):
    """Gradients of out = a (op) b when a and g are sharded along the leading
    axis and b is replicated (broadcast along it, e.g. a bias, or config 5's
    b [1,Q,1,L]): da is local; db sums over every rank's rows, so each rank
    writes an unrounded double partial in the same fused pass and the
    partials are combined in rank order. Returns (da, db), db identical on
    every rank."""
    da = CudaStorage(int(np.prod(a_shape, dtype=np.int64)))
    nb = int(np.prod(b_shape, dtype=np.int64))
    da_part, db_part = CudaStorage(da.size, np.float64), CudaStorage(nb, np.float64)
    sa, ra = _abi.shape_arg(a_shape)
    sb, rb = _abi.shape_arg(b_shape)
    sg, rg = _abi.shape_arg(g_shape)
    _abi.call("vc_cuda_binary_backward_partial", op, _p(a), sa, ra, _p(b), sb, rb, _p(g), sg, rg, _p(da_part),
              _p(db_part))
    # da has no cross-rank sum: round this rank's partial (one combine of one rank)
    _abi.call("vc_cuda_combine_partials", _B.REDUCE_SUM, _p(da_part), None, None, 1, ctypes.c_size_t(da.size),
              ctypes.c_float(0.0), 0, _p(da), None)
    return da, _combine_sums(comm, db_part, nb)


def bias_relu_sum(x: CudaStorage, b: CudaStorage, rows_local: int, cols: int, comm: Communicator) -> CudaStorage:
    """relu(x + b).sum() of a row-sharded x [rows_local, cols] and a
    replicated bias b [cols]: the fused forward's double partial per rank,
    combined in rank order."""
    part = CudaStorage(1, np.float64)
    _abi.call("vc_cuda_bias_relu_sum", _p(x), _p(b), ctypes.c_size_t(rows_local), ctypes.c_size_t(cols), None,
              _p(part))
    return _combine_sums(comm, part, 1)


def bias_relu_sum_backward(x, b, upstream, rows_local: int, cols: int, comm: Communicator):
    """(dx, db) of the sharded relu(x + b).sum(): dx local (bit-exact with one
    GPU), db from per-rank double partials combined in rank order."""
    dx = CudaStorage(rows_local * cols)
    part = CudaStorage(cols, np.float64)
    _abi.call("vc_cuda_bias_relu_sum_backward", _p(x), _p(b), _p(upstream), ctypes.c_size_t(rows_local),
              ctypes.c_size_t(cols), _p(dx), None, _p(part))
    return dx, _combine_sums(comm, part, cols)


__all__ = ["RowShard", "Communicator", "exchange_unique_id", "sum_axis0", "sum_axis0_backward", "max_axis0",
           "sum_all", "axis0_reductions", "cross_entropy", "cross_entropy_backward", "binary_backward",
           "bias_relu_sum", "bias_relu_sum_backward"]

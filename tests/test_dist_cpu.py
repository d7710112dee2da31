"""Multi-GPU host logic on CPU: row sharding, the NCCL-id exchange over a
torch.distributed group, and failure detection when a rank dies. The ranks
are gloo processes (world size 2) started with the spawn method; no GPU is
touched. The device-side path (partials, NCCL all-gather, rank-order
combine) is tests/test_gpu_dist.py."""
import os
import socket
import time

import pytest

from vectorcore_b200.dist import RowShard


@pytest.mark.parametrize("rows", [0, 1, 7, 1000, 1003, 8192])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_row_shards_cover_the_rows_once_in_rank_order(rows, world):
    shards = [RowShard(rows, world, r) for r in range(world)]
    assert shards[0].start == 0 and shards[-1].stop == rows
    for a, b in zip(shards, shards[1:]):
        assert a.stop == b.start
    counts = [s.count for s in shards]
    assert max(counts) - min(counts) <= 1
    assert sorted(counts, reverse=True) == counts  # the extra rows go to the lowest ranks


def test_row_shard_rejects_bad_ranks():
    with pytest.raises(ValueError):
        RowShard(10, 2, 2)
    with pytest.raises(ValueError):
        RowShard(10, 0, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, queue):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    from vectorcore_b200.dist import exchange_unique_id

    try:
        if mode == "ok":
            uid = exchange_unique_id(lambda: bytes(range(128)))
            queue.put((rank, "ok", uid == bytes(range(128))))
        elif mode == "rank1_dies":
            if rank == 1:
                os._exit(3)  # leaves before the collective, without a goodbye
            t0 = time.monotonic()
            try:
                exchange_unique_id(lambda: bytes(128))
                queue.put((rank, "no error", time.monotonic() - t0))
            except Exception as exc:  # the peer never joined: a bounded error, not a hang
                queue.put((rank, "error", time.monotonic() - t0, type(exc).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode, world=2):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, queue)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a gloo rank did not finish within 120 s")
    out = []
    while not queue.empty():
        out.append(queue.get())
    return sorted(out), procs


def test_unique_id_reaches_every_rank_over_gloo():
    out, procs = _run("ok")
    assert [o[:3] for o in out] == [(0, "ok", True), (1, "ok", True)]
    assert all(p.exitcode == 0 for p in procs)


def test_a_rank_that_dies_is_detected_not_waited_for():
    out, procs = _run("rank1_dies")
    by_rank = {o[0]: o for o in out}
    assert procs[1].exitcode == 3
    assert by_rank[0][1] == "error", by_rank[0]
    assert by_rank[0][2] < 60.0  # bounded by the process group's timeout

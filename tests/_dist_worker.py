"""One rank of the row-sharded multi-GPU check (run by tests/test_gpu_dist.py
under torch.distributed.run, one process per GPU).

Every rank holds its RowShard of the same seeded global tensors, computes the
sharded reductions (per-rank partials, the CUDA device's NCCL all-gather,
rank-order combine: vectorcore_b200.dist) and gathers its results to rank 0
over the host group. Rank 0 computes the same ops on the whole tensors on its
own GPU and checks: bit-exact for max/argmax (also against the CPU oracle),
the scan's cross-shard rules and every local backward; within 1e-5 for sums,
means and cross-entropy. Covered: axis-0 sum / mean / max / argmax, the full
sum, cross-entropy's mean over a sharded batch and its dlogits, the gradient
of a replicated broadcast operand (configuration 5's b [1,Q,1,L]) and the
fused relu(x + b).sum() chain with its bias gradient."""
import datetime
import json
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def main():
    import torch.distributed as dist

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=90))
    import oracle
    from vectorcore_b200 import _abi
    from vectorcore_b200 import backend as B
    from vectorcore_b200 import dist as vdist

    _abi.check(_abi.lib.vc_cuda_init(local))
    be = B.CudaBackend.instance()
    comm = vdist.Communicator.from_torch(timeout_ms=60_000)
    out = {}

    # ---- reductions over the sharded leading axis --------------------------------
    rows, cols = 1003, 4099
    x = np.random.default_rng(4).normal(size=(rows, cols)).astype(np.float32)
    shards = [vdist.RowShard(rows, world, r) for r in range(world)]
    x[:, 0] = 0.0
    x[5, 0] = 7.0                      # equal maxima in the first and the last shard:
    x[rows - 5, 0] = 7.0               # the lower row (lower rank) must win
    x[0, 1] = np.nan                   # NaN at global row 0 wins its column
    x[shards[-1].start, 2] = np.nan    # NaN at a later shard's first row must not
    x[:, 3] = -0.0
    x[shards[-1].start, 3] = 0.0       # a zero maximum keeps the first zero's sign
    sh = shards[rank]
    xl = be.upload(x[sh.start:sh.stop])
    s = vdist.sum_axis0(xl, sh.count, cols, comm)
    mean = vdist.sum_axis0(xl, sh.count, cols, comm, mean_rows=rows)
    mx, mi = vdist.max_axis0(xl, sh.count, cols, comm, sh)
    tot = vdist.sum_all(xl, sh.count * cols, comm)
    w = np.random.default_rng(12).uniform(-1, 1, size=cols).astype(np.float32)
    dw = be.upload(w)
    dx = vdist.sum_axis0_backward(dw, sh.count, cols)
    dxm = vdist.sum_axis0_backward(dw, sh.count, cols, mean_rows=rows)
    s3, (mx3, mi3), tot3 = vdist.axis0_reductions(xl, sh.count, cols, comm, sh)  # one grouped all-gather
    out.update(s=be.download(s), mean=be.download(mean), mx=be.download(mx), mi=be.download(mi),
               tot=float(be.download(tot)[0]), dx=be.download(dx), dxm=be.download(dxm))
    # the planted NaNs make some sums NaN: compare NaN-aware, bit for bit otherwise
    grouped_same = (np.array_equal(be.download(s3), out["s"], equal_nan=True) and
                    np.array_equal(be.download(mx3), out["mx"], equal_nan=True) and
                    np.array_equal(be.download(mi3), out["mi"]) and
                    np.array_equal(be.download(tot3), np.array([out["tot"]], np.float32), equal_nan=True))
    out["grouped_same"] = bool(grouped_same)

    # ---- cross-entropy over a sharded batch -----------------------------------------
    batch, classes = 513, 1000
    logits = np.random.default_rng(5).normal(0, 2, size=(batch, classes)).astype(np.float32)
    targets = np.random.default_rng(6).integers(0, classes, batch).astype(np.int64)
    ls = vdist.RowShard(batch, world, rank)
    lg, tg = be.upload(logits[ls.start:ls.stop]), be.upload(targets[ls.start:ls.stop])
    loss, m, ssum = vdist.cross_entropy(lg, tg, ls.count, classes, comm, batch)
    one = be.upload(np.ones(1, np.float32))
    dlg = vdist.cross_entropy_backward(lg, tg, m, ssum, one, ls.count, classes, batch)
    out.update(loss=float(be.download(loss)[0]), dlogits=be.download(dlg))

    # ---- gradient of a replicated broadcast operand (configuration 5's b) ----------
    # (16 rows of b: the TMA-fed kernel, with double db partials per shard)
    P, Q, R, L = 5, 16, 24, 64
    a5 = np.random.default_rng(7).uniform(-1, 1, (P, 1, R, L)).astype(np.float32)
    b5 = np.random.default_rng(8).uniform(-1, 1, (1, Q, 1, L)).astype(np.float32)
    g5 = np.random.default_rng(9).uniform(-1, 1, (P, Q, R, L)).astype(np.float32)
    ps = vdist.RowShard(P, world, rank)
    da5, db5 = vdist.binary_backward(B.MUL, be.upload(a5[ps.start:ps.stop]), (ps.count, 1, R, L), be.upload(b5),
                                     b5.shape, be.upload(g5[ps.start:ps.stop]), (ps.count, Q, R, L), comm)
    out.update(da5=be.download(da5), db5=be.download(db5))

    # ---- relu(x + b).sum() with a sharded batch and a replicated bias ---------------
    br, bc = 1000, 512
    xb = np.random.default_rng(0).uniform(-1, 1, (br, bc)).astype(np.float32)
    bb = np.random.default_rng(1).normal(size=bc).astype(np.float32)
    bs = vdist.RowShard(br, world, rank)
    dxb_, dbb_ = be.upload(xb[bs.start:bs.stop]), be.upload(bb)
    lb = vdist.bias_relu_sum(dxb_, dbb_, bs.count, bc, comm)
    gxb, gbb = vdist.bias_relu_sum_backward(dxb_, dbb_, one, bs.count, bc, comm)
    out.update(lb=float(be.download(lb)[0]), gxb=be.download(gxb), gbb=be.download(gbb))
    comm.synchronize()

    gathered = [None] * world
    dist.all_gather_object(gathered, out)
    if rank == 0:
        checks = {}
        same = lambda a, b: bool(np.array_equal(np.asarray(a), np.asarray(b), equal_nan=True))
        rel = lambda a, b, t=1e-5: bool(np.allclose(a, b, rtol=t, atol=t * np.nanmax(np.abs(b)) + 1e-30,
                                                    equal_nan=True))
        dxf = be.upload(x)
        full_s = be.download(be.reduce_axis(dxf, 1, rows, cols, B.REDUCE_SUM))
        full_mean = be.download(be.reduce_axis(dxf, 1, rows, cols, B.REDUCE_MEAN))
        full_tot = float(be.download(be.reduce_sum(dxf, rows * cols))[0])
        full_dx = be.download(be.reduce_axis_backward(B.REDUCE_SUM, dw, None, 1, rows, cols))
        full_dxm = be.download(be.reduce_axis_backward(B.REDUCE_MEAN, dw, None, 1, rows, cols))
        for r, res in enumerate(gathered):
            checks[f"rank{r}_sum_axis0"] = rel(res["s"], full_s)
            checks[f"rank{r}_mean_axis0"] = rel(res["mean"], full_mean)
            checks[f"rank{r}_sum_all"] = rel(np.array([res["tot"]]), np.array([full_tot]))
            checks[f"rank{r}_grouped_allgather_same"] = res["grouped_same"]
            checks[f"rank{r}_max_same_on_every_rank"] = same(res["mx"], gathered[0]["mx"]) and same(res["mi"], gathered[0]["mi"])
        Pt = oracle.port()
        ref_max = Pt.reduce_axis(oracle.MAX, x, 1, rows, cols)
        ref_arg = Pt.argmax_i64(x, 1, rows, cols)
        mx0, mi0 = gathered[0]["mx"], gathered[0]["mi"]
        checks["max_axis0_bitexact"] = same(mx0.view(np.uint32), ref_max.view(np.uint32)) or same(mx0, ref_max)
        checks["argmax_axis0"] = same(mi0, ref_arg)
        checks["argmax_tie_lower_rank"] = bool(int(mi0[0]) == 5)
        checks["nan_row0_wins"] = bool(int(mi0[1]) == 0 and np.isnan(mx0[1]))
        checks["nan_later_shard_ignored"] = bool(int(mi0[2]) != shards[-1].start)
        checks["zero_max_first_sign"] = bool(int(mi0[3]) == 0 and mx0.view(np.uint32)[3] == np.float32(-0.0).view(np.uint32))
        checks["sum_axis0_backward_bitexact"] = same(np.concatenate([res["dx"] for res in gathered]), full_dx)
        checks["mean_axis0_backward_bitexact"] = same(np.concatenate([res["dxm"] for res in gathered]), full_dxm)

        dlf, dtf = be.upload(logits), be.upload(targets)
        floss, fm, fs, _ = be.cross_entropy(dlf, dtf, batch, classes)
        full_loss = float(be.download(floss)[0])
        full_dlg = be.download(be.cross_entropy_backward(dlf, dtf, fm, fs, one, batch, classes))
        for r, res in enumerate(gathered):
            checks[f"rank{r}_ce_loss"] = rel(np.array([res["loss"]]), np.array([full_loss]))
        checks["ce_dlogits"] = rel(np.concatenate([res["dlogits"] for res in gathered]), full_dlg)

        fda5, fdb5 = be.binary_backward(B.MUL, be.upload(a5), a5.shape, be.upload(b5), b5.shape, be.upload(g5),
                                        g5.shape)
        checks["bcast_da_local"] = rel(np.concatenate([res["da5"] for res in gathered]), be.download(fda5))
        for r, res in enumerate(gathered):
            checks[f"rank{r}_bcast_db_combined"] = rel(res["db5"], be.download(fdb5))

        dxbf, dbbf = be.upload(xb), be.upload(bb)
        flb = float(be.download(be.bias_relu_sum(dxbf, dbbf, br, bc))[0])
        fgx, fgb = be.bias_relu_sum_backward(dxbf, dbbf, one, br, bc)
        for r, res in enumerate(gathered):
            checks[f"rank{r}_bias_relu_sum_loss"] = rel(np.array([res["lb"]]), np.array([flb]))
            checks[f"rank{r}_bias_relu_sum_db"] = rel(res["gbb"], be.download(fgb))
        checks["bias_relu_sum_dx_bitexact"] = same(np.concatenate([res["gxb"] for res in gathered]),
                                                   be.download(fgx))
        print(json.dumps({"world": world, "checks": checks}), flush=True)
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

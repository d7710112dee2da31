"""One rank of the row-sharded multi-GPU check (launched by
tests/test_gpu_dist.py through torch.distributed.run; not collected by
pytest). The NCCL id travels over a gloo process group; the partials travel
over the CUDA device's own NCCL communicator. Rank 0 compares every sharded
result with the same computation done whole on its own GPU and prints one
JSON line of checks."""
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
    import vectorcore_b200 as vc
    from vectorcore_b200 import _abi
    from vectorcore_b200 import dist as vdist

    _abi.check(_abi.lib.vc_cuda_init(local))
    comm = vdist.Communicator.from_torch(timeout_ms=60_000)

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
    shard = shards[rank]
    xl = vc.Tensor(x[shard.start:shard.stop], requires_grad=True, device="cuda")
    s = vdist.sum_axis0(xl, comm)
    mean = vdist.sum_axis0(xl, comm, mean_rows=rows)
    mx, mi = vdist.max_axis0(xl, comm, shard)
    tot = vdist.sum_all(xl, comm)
    w = np.random.default_rng(12).uniform(-1, 1, size=cols).astype(np.float32)
    (s * vc.Tensor(w, device="cuda")).sum().backward()

    batch, classes = 513, 1000
    logits = np.random.default_rng(5).normal(0, 2, size=(batch, classes)).astype(np.float32)
    targets = np.random.default_rng(6).integers(0, classes, batch)
    ls = vdist.RowShard(batch, world, rank)
    lg = vc.Tensor(logits[ls.start:ls.stop], requires_grad=True, device="cuda")
    loss = vdist.cross_entropy(lg, targets[ls.start:ls.stop], comm, batch)
    loss.backward()
    comm.synchronize()

    local = {"dx": xl.grad.numpy(), "dlogits": lg.grad.numpy(), "s": s.numpy(), "mean": mean.numpy(),
             "mx": mx.numpy(), "mi": mi, "tot": tot.item(), "loss": loss.item()}
    gathered = [None] * world
    dist.all_gather_object(gathered, local)
    if rank == 0:
        checks = {}
        xf = vc.Tensor(x, requires_grad=True, device="cuda")
        sf = xf.sum(0)
        (sf * vc.Tensor(w, device="cuda")).sum().backward()
        same = lambda a, b: bool(np.array_equal(np.asarray(a), np.asarray(b), equal_nan=True))
        rel = lambda a, b, t=1e-5: bool(np.allclose(a, b, rtol=t, atol=t * np.max(np.abs(b)) + 1e-30,
                                                    equal_nan=True))
        for r, res in enumerate(gathered):
            checks[f"rank{r}_sum_axis0"] = rel(res["s"], sf.numpy())
            checks[f"rank{r}_mean_axis0"] = rel(res["mean"], xf.mean(0).numpy())
            checks[f"rank{r}_tot"] = rel(np.array([res["tot"]]), np.array([xf.sum().item()]))
        P = oracle.port()
        ref_max = P.reduce_axis(oracle.MAX, x, 1, rows, cols)
        ref_arg = P.argmax_i64(x, 1, rows, cols)
        checks["max_axis0_bitexact"] = bool(np.array_equal(gathered[0]["mx"].view(np.uint32), ref_max.view(np.uint32))
                                            or same(gathered[0]["mx"], ref_max))
        checks["argmax_axis0"] = same(gathered[0]["mi"], ref_arg)
        checks["argmax_tie_lower_rank"] = bool(int(gathered[0]["mi"][0]) == 5)
        checks["nan_row0_wins"] = bool(int(gathered[0]["mi"][1]) == 0 and np.isnan(gathered[0]["mx"][1]))
        checks["nan_later_shard_ignored"] = bool(int(gathered[0]["mi"][2]) != shards[-1].start)
        checks["zero_max_first_sign"] = bool(int(gathered[0]["mi"][3]) == 0 and
                                             gathered[0]["mx"].view(np.uint32)[3] == np.float32(-0.0).view(np.uint32))
        dx_full = np.concatenate([res["dx"] for res in gathered])
        checks["dx_backward_bitexact"] = same(dx_full, xf.grad.numpy())
        lf = vc.Tensor(logits, requires_grad=True, device="cuda")
        lossf = vc.cross_entropy(lf, targets)
        lossf.backward()
        checks["ce_loss"] = all(rel(np.array([res["loss"]]), np.array([lossf.item()])) for res in gathered)
        checks["ce_dlogits"] = rel(np.concatenate([res["dlogits"] for res in gathered]), lf.grad.numpy())
        print(json.dumps({"world": world, "checks": checks}), flush=True)
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

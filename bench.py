"""Benchmark of VectorCore's CUDA device on B200 (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg2|cfg1|cfg3|cfg4|cfg5] [--rows R]

Metric: effective HBM GB/s per op and elements/s. A step is
one pass of the hot path over one batch of the workload; `value` = the sum of
the ops' ALGORITHMIC bytes (count-once traffic, benchmark table) over all
ranks / device time of the step, from CUDA events on the library's stream,
max over ranks.

Default workload (the one the driver runs): benchmark configuration 2 -- the
same-shape elementwise sweep on a, b, g of [16384, 16384] float32 (2^28
elements, 1.07 GB each, larger than the 126 MB L2, and L2 flushed before
every timed op by a 256 MiB read): add, sub, mul, div, neg, exp, log, relu,
sigmoid and a * 0.5, each forward and backward. Multi-GPU: strong scaling,
as configuration 2 states -- ONE global [16384, 16384] tensor sharded along
axis 0, rank r computing its 16384/N rows (elementwise work needs no
communication). The global tensors are generated block-wise (1024-row blocks,
each from its own seed) so every N sees the same data.

The same line carries
* `sharded_reduction`: configuration 3's axis-0 sum, max / argmax and full
  sum over a row-sharded [8192, 32768] at N GPUs -- per-rank partials, the
  CUDA device's NCCL all-gather, rank-order combine -- timed, split into the
  local reduction and the collective + combine, and checked on every rank
  against the 1-GPU result;
* `per_config` (N = 1): per-op GB/s of configurations 1, 3, 4 and 5;
* `e2e`: the sweep through the C ABI with host buffers (uploads and the
  result's download inside the timed region);
* `cpu_baseline`: the reference's own CPU path on a bounded sample.

`--workload cfg1|cfg3|cfg4|cfg5` makes another configuration the headline;
`--rows` shrinks the leading dimension (small profiling cases).

Only bench.py's cpu_baseline leg and the --impl reference arm touch oracle/
(the reference's own CPU path compiled from its sources, oracle/_ref).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
TRAFFIC_FILE = ROOT / "profiles" / "traffic.json"
FALLBACK_HBM_GBS = 6650.0


def hbm_peak():
    try:
        p = json.loads(PEAKS_FILE.read_text())
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.lines: list[str] = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, power, smax, reasons = [], [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


# --------------------------------------------------------------------------------------
# Workloads. Each op: (name, algorithmic bytes, callable returning the outputs).
# --------------------------------------------------------------------------------------
class Ctx:
    def __init__(self, be, B, abi, rank, rows, torch, world=1):
        self.be, self.B, self.abi, self.rank, self.rows, self.torch = be, B, abi, rank, rows, torch
        self.world = world
        self.launches = 0

    def L(self, x, k=1):
        self.launches += k
        return x

    def from_torch(self, t):
        """Copy a torch CUDA tensor into a pool buffer (setup only)."""
        self.torch.cuda.synchronize()
        s = self.be.allocate(t.numel(), np.float32 if t.dtype.is_floating_point else np.int64)
        self.abi.call("vc_cuda_copy", ctypes.c_void_p(s.ptr), ctypes.c_void_p(t.data_ptr()),
                      ctypes.c_size_t(t.numel() * t.element_size()))
        self.be.synchronize()
        return s


GEN_BLOCK = 1024  # rows per generator block of the global tensors


def block_rows(seed, r0, r1, cols, draw, block=GEN_BLOCK):
    """Rows [r0, r1) of a global float32 tensor whose 1024-row block k is
    draw(default_rng([seed, k]), size): any rank can produce exactly its
    shard, and every shard layout sees the same global tensor."""
    out = np.empty((r1 - r0, cols), np.float32)
    for k in range(r0 // block, (r1 + block - 1) // block if r1 > r0 else r0 // block):
        lo, hi = k * block, (k + 1) * block
        vals = draw(np.random.default_rng([seed, k]), (block, cols)).astype(np.float32)
        a, b = max(lo, r0), min(hi, r1)
        out[a - r0:b - r0] = vals[a - lo:b - lo]
    return out


def uniform_rows(seed, lo, hi, r0, r1, cols):
    return block_rows(seed, r0, r1, cols, lambda g, size: g.uniform(lo, hi, size=size))


def normal_rows(seed, std, r0, r1, cols):
    return block_rows(seed, r0, r1, cols, lambda g, size: g.normal(0.0, std, size=size))


CFG2_ROWS, CFG2_COLS = 16384, 16384


def wl_cfg2(c: Ctx):
    be, B = c.be, c.B
    from vectorcore_b200.dist import RowShard

    cols = CFG2_COLS
    sh = RowShard(c.rows or CFG2_ROWS, c.world, c.rank)
    rows = sh.count
    n = rows * cols
    shape = (rows, cols)
    a_np = uniform_rows(2, 0.1, 2.0, sh.start, sh.stop, cols).reshape(-1)
    b_np = uniform_rows(3, 0.1, 2.0, sh.start, sh.stop, cols).reshape(-1)
    g_np = uniform_rows(9, -1.0, 1.0, sh.start, sh.stop, cols).reshape(-1)
    a, b, g = be.upload(a_np), be.upload(b_np), be.upload(g_np)
    s_neg = be.binary_scalar(a, n, 1.0, B.SUB)  # a - 1: signed inputs for neg / relu / sigmoid
    saved = {}

    def save(k, v):
        saved[k] = v
        return v

    L = c.L
    ops = [
        ("add.fwd", 12 * n, lambda: L(be.binary(a, shape, None, b, shape, None, shape, B.ADD))),
        ("sub.fwd", 12 * n, lambda: L(be.binary(a, shape, None, b, shape, None, shape, B.SUB))),
        ("mul.fwd", 12 * n, lambda: L(be.binary(a, shape, None, b, shape, None, shape, B.MUL))),
        ("div.fwd", 12 * n, lambda: L(be.binary(a, shape, None, b, shape, None, shape, B.DIV))),
        ("neg.fwd", 8 * n, lambda: L(be.unary(s_neg, n, B.NEG))),
        ("exp.fwd", 8 * n, lambda: save("exp", L(be.unary(a, n, B.EXP)))),
        ("log.fwd", 8 * n, lambda: L(be.unary(a, n, B.LOG))),
        ("relu.fwd", 8 * n, lambda: L(be.unary(s_neg, n, B.RELU))),
        ("sigmoid.fwd", 8 * n, lambda: save("sigmoid", L(be.unary(s_neg, n, B.SIGMOID)))),
        ("scalar_mul.fwd", 8 * n, lambda: L(be.binary_scalar(a, n, 0.5, B.MUL))),
        # backward given a dense upstream g (the add gradients alias g: no kernel, 0 bytes)
        ("sub.bwd", 8 * n, lambda: L(be.unary(g, n, B.NEG))),  # da aliases g; db = -g
        ("mul.bwd", 20 * n, lambda: L(be.binary_backward(B.MUL, a, shape, b, shape, g, shape))),
        ("div.bwd", 20 * n, lambda: L(be.binary_backward(B.DIV, a, shape, b, shape, g, shape))),
        ("neg.bwd", 8 * n, lambda: L(be.unary_backward(B.NEG, None, None, g, n))),
        ("exp.bwd", 12 * n, lambda: L(be.unary_backward(B.EXP, None, saved["exp"], g, n))),
        ("log.bwd", 12 * n, lambda: L(be.unary_backward(B.LOG, a, None, g, n))),
        ("relu.bwd", 12 * n, lambda: L(be.unary_backward(B.RELU, s_neg, None, g, n))),
        ("sigmoid.bwd", 12 * n, lambda: L(be.unary_backward(B.SIGMOID, None, saved["sigmoid"], g, n))),
        ("scalar_mul.bwd", 8 * n, lambda: L(be.binary_scalar(g, n, 0.5, B.MUL))),
    ]
    host = {"a": a_np, "b": b_np, "g": g_np}
    dev = {"a": a, "b": b, "g": g}
    desc = (f"cfg2: same-shape elementwise sweep, a,b,g [{sh.rows},{cols}] f32 sharded along axis 0 "
            f"({rows} rows per GPU), add/sub/mul/div/neg/exp/log/relu/sigmoid/a*0.5 fwd+bwd")
    # first op that reads each uploaded input (g only from the backward ops on)
    first_use = {"a": 0, "b": 0, "g": [name for name, _, _ in ops].index("sub.bwd")}
    return {"ops": ops, "elements": n, "elements_global": sh.rows * cols, "desc": desc, "host": host, "dev": dev,
            "e2e_result": "last", "first_use": first_use,
            "metric": "effective HBM GB/s (config 2 elementwise sweep, fwd+bwd)"}


def wl_cfg1(c: Ctx):
    """relu(x + b).sum() forward and backward, x [1024, 4096], b [4096] (L2-resident),
    through the fused chain (vc.bias_relu_sum): one launch each way."""
    be = c.be
    rows = c.rows or 1024
    cols = 4096
    n = rows * cols
    x_np = np.random.default_rng(0).uniform(-1, 1, (rows, cols)).astype(np.float32)
    b_np = np.random.default_rng(1).normal(size=cols).astype(np.float32)
    x, b = be.upload(x_np), be.upload(b_np)
    one = be.upload(np.ones(1, np.float32))
    L = c.L
    # Each op is captured once as a CUDA graph (after one eager call, which
    # does the first-call set-up) and replayed: the step is launch-bound, and
    # a graph replay is one launch whatever the host does.
    def chain():
        loss = be.bias_relu_sum(x, b, rows, cols)
        dx, db = be.bias_relu_sum_backward(x, b, one, rows, cols)
        return loss, dx, db

    chain()
    be.synchronize()
    graph, _ = be.capture(chain)
    kernels = graph.nodes
    c.keep = graph

    def fwd_bwd():
        return L(graph.launch(), kernels)

    # algorithmic bytes: fwd reads x, b; bwd reads x, b and writes dx, db
    ops = [("bias_relu_sum.fwd+bwd", 4 * (n + cols) + 4 * (2 * n + 2 * cols), fwd_bwd)]
    return {"ops": ops, "elements": n, "desc": f"cfg1: relu(x+b).sum() fwd+bwd, x [{rows},{cols}], b [{cols}] "
                                              "(16.8 MB, L2-resident: launch-bound); fused chain, one kernel each "
                                              "way, the step replayed as one captured CUDA graph",
            "metric": "effective GB/s (config 1 bias+relu+sum, fwd+bwd)"}


def wl_cfg3(c: Ctx):
    be, B, torch = c.be, c.B, c.torch
    rows = c.rows or 8192
    cols = 32768
    n = rows * cols
    gen = torch.Generator(device="cuda").manual_seed(4)
    x = c.from_torch(torch.randn(rows, cols, device="cuda", generator=gen))
    g1 = c.from_torch(torch.rand(rows, device="cuda", generator=gen) * 2 - 1)
    one = be.upload(np.ones(1, np.float32))
    st = {}
    L = c.L
    R = B.REDUCE_SUM

    def max1():
        v, i = be.reduce_axis(x, rows, cols, 1, B.REDUCE_MAX, want_index=True)
        st["idx1"] = i
        return L((v, i))

    ops = [
        ("sum_axis1.fwd", 4 * n, lambda: L(be.reduce_axis(x, rows, cols, 1, R))),
        ("mean_axis1.fwd", 4 * n, lambda: L(be.reduce_axis(x, rows, cols, 1, B.REDUCE_MEAN))),
        ("max_argmax_axis1.fwd", 4 * n, max1),
        ("argmax_axis1.fwd", 4 * n, lambda: L(be.reduce_axis(x, rows, cols, 1, B.REDUCE_ARGMAX))),
        ("sum_axis0.fwd", 4 * n, lambda: L(be.reduce_axis(x, 1, rows, cols, R), 2)),
        ("max_axis0.fwd", 4 * n, lambda: L(be.reduce_axis(x, 1, rows, cols, B.REDUCE_MAX), 2)),
        ("sum_all.fwd", 4 * n, lambda: L(be.reduce_sum(x, n), 2)),
        ("mean_all.fwd", 4 * n, lambda: L(be.reduce_all(x, n, B.REDUCE_MEAN), 2)),
        ("sum_axis1.bwd", 4 * n, lambda: L(be.reduce_axis_backward(R, g1, None, rows, cols, 1))),
        ("mean_axis1.bwd", 4 * n, lambda: L(be.reduce_axis_backward(B.REDUCE_MEAN, g1, None, rows, cols, 1))),
        ("max_axis1.bwd", 4 * n, lambda: L(be.reduce_axis_backward(B.REDUCE_MAX, g1, st["idx1"], rows, cols, 1))),
        ("sum_all.bwd", 4 * n, lambda: L(be.broadcast_to(one, (), (rows, cols)))),
    ]
    return {"ops": ops, "elements": n, "desc": f"cfg3: reductions of x [{rows},{cols}] ~ N(0,1)",
            "metric": "effective HBM GB/s (config 3 reductions, fwd+bwd)"}


def wl_cfg4(c: Ctx):
    be, B, torch = c.be, c.B, c.torch
    rows = c.rows or 65536
    cols = 32000
    n = rows * cols
    gen = torch.Generator(device="cuda").manual_seed(5)
    lg = c.from_torch(torch.randn(rows, cols, device="cuda", generator=gen) * 2)
    tg = c.from_torch(torch.randint(0, cols, (rows,), device="cuda", generator=gen, dtype=torch.int64))
    g = c.from_torch(torch.rand(rows, cols, device="cuda", generator=gen) * 2 - 1)
    one = be.upload(np.ones(1, np.float32))
    st = {}
    L = c.L

    def ce_fwd():
        loss, m, s, part = be.cross_entropy(lg, tg, rows, cols)
        st["ce"] = (m, s)
        return L(loss, 2)

    def sm_fwd():
        y, m, s = be.softmax(lg, rows, 1 * cols, 1, log=False)
        st["sm"] = (m, s)
        return L(y)

    def lsm_fwd():
        y, m, s = be.softmax(lg, rows, cols, 1, log=True)
        st["lsm"] = (m, s)
        return L(y)

    ops = [
        ("softmax.fwd", 8 * n, sm_fwd),
        ("log_softmax.fwd", 8 * n, lsm_fwd),
        ("cross_entropy.fwd", 4 * n + 8 * rows, ce_fwd),
        ("cross_entropy.bwd", 8 * n + 8 * rows, lambda: L(be.cross_entropy_backward(lg, tg, *st["ce"], one, rows, cols))),
        ("softmax.bwd", 12 * n, lambda: L(be.softmax_backward(lg, *st["sm"], g, rows, cols, 1, log=False))),
        ("log_softmax.bwd", 12 * n, lambda: L(be.softmax_backward(lg, *st["lsm"], g, rows, cols, 1, log=True))),
    ]
    return {"ops": ops, "elements": n, "desc": f"cfg4: logits [{rows},{cols}] ~ N(0,2), int64 targets",
            "metric": "effective HBM GB/s (config 4 softmax / cross-entropy, fwd+bwd)"}


def wl_cfg5(c: Ctx):
    be, B, torch = c.be, c.B, c.torch
    d0 = c.rows or 64
    a_shape, b_shape = (d0, 1, 512, 1024), (1, 128, 1, 1024)
    o_shape = (d0, 128, 512, 1024)
    n = int(np.prod(o_shape))
    a_np = np.random.default_rng(7).uniform(-1, 1, a_shape).astype(np.float32)
    b_np = np.random.default_rng(8).uniform(-1, 1, b_shape).astype(np.float32)
    a, b = be.upload(a_np), be.upload(b_np)
    gen = torch.Generator(device="cuda").manual_seed(11)
    g = c.from_torch(torch.rand(*o_shape, device="cuda", generator=gen) * 2 - 1)
    one = be.upload(np.ones(1, np.float32))
    st = {}
    L = c.L

    def fwd():
        st["out"] = L(be.binary(a, a_shape, None, b, b_shape, None, o_shape, B.MUL))
        return st["out"]

    ab = 4 * (a_np.size + b_np.size)
    ops = [
        ("bcast_mul.fwd", 4 * n + ab, fwd),
        ("sum.fwd", 4 * n, lambda: L(be.reduce_sum(st["out"], n), 2)),
        ("bcast_mul.bwd_dense_g", 4 * n + 2 * ab, lambda: L(be.binary_backward(B.MUL, a, a_shape, b, b_shape, g, o_shape), 4)),
        ("bcast_mul.bwd_sum_upstream", 2 * ab, lambda: L(be.binary_backward(B.MUL, a, a_shape, b, b_shape, one, ()), 4)),
    ]
    return {"ops": ops, "elements": n, "desc": f"cfg5: a {a_shape} * b {b_shape} -> {o_shape}, then sum; "
                                              "backward for a dense g and for the sum's scalar upstream",
            "metric": "effective HBM GB/s (config 5 strided broadcast multiply, fwd+bwd)"}


WORKLOADS = {"cfg1": wl_cfg1, "cfg2": wl_cfg2, "cfg3": wl_cfg3, "cfg4": wl_cfg4, "cfg5": wl_cfg5}


# --------------------------------------------------------------------------------------
# Our arm
# --------------------------------------------------------------------------------------
class Timer:
    """Per-op CUDA events on the library's stream, with an L2 flush (a read of
    256 MiB) before every timed op unless the workload is L2-resident by
    design (configuration 1), and a GPU sleep of `lead_cycles` between the
    flush and the op's start event."""

    def __init__(self, torch, vstream, flush_l2=True, lead_cycles=400_000):
        self.torch, self.vstream, self.lead_cycles = torch, vstream, lead_cycles
        self.flush_buf = torch.ones(64 << 20, dtype=torch.float32, device="cuda") if flush_l2 else None
        self.flush_out = torch.empty((), dtype=torch.float32, device="cuda")

    def flush(self):
        if self.flush_buf is not None:
            with self.torch.cuda.stream(self.vstream):
                self.torch.sum(self.flush_buf, dim=0, out=self.flush_out)

    def run(self, ops, steps, warmup, barrier):
        """Per-op device milliseconds summed over `steps` timed steps."""
        torch = self.torch
        for _ in range(warmup):
            for _, _, fn in ops:
                fn()
        barrier()
        ev = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in ops]
        per_op_ms = [0.0] * len(ops)
        for _ in range(steps):
            for i, (_, _, fn) in enumerate(ops):
                self.flush()
                # keep the GPU busy while the host queues the op, so its
                # events hold no host launch latency (outside the events, like
                # the flush; with one lead per step instead, the first op of
                # every step read up to 10% slow)
                with torch.cuda.stream(self.vstream):
                    torch.cuda._sleep(self.lead_cycles)
                ev[i][0].record(self.vstream)
                fn()
                ev[i][1].record(self.vstream)
            torch.cuda.synchronize()
            for i in range(len(ops)):
                per_op_ms[i] += ev[i][0].elapsed_time(ev[i][1])
        barrier()
        return per_op_ms


def release(be, torch):
    """Hand cached device memory back between workloads."""
    be.synchronize()
    from vectorcore_b200 import _abi

    _abi.call("vc_cuda_pool_trim")
    torch.cuda.empty_cache()


def run_ours(args):
    import torch

    from vectorcore_b200 import _abi
    from vectorcore_b200 import backend as B

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        # The sweep has no data-path collective (each rank owns a row shard).
        # The host group carries the barrier, the max-over-ranks of the
        # timings and the NCCL unique id of the CUDA device's communicator
        # (the sharded reductions' all-gather runs over NCCL, not this group).
        torch.cuda.set_device(local)
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    _abi.check(_abi.lib.vc_cuda_init(local))
    torch.cuda.set_device(local)
    be = B.CudaBackend.instance()
    vstream = torch.cuda.ExternalStream(_abi.lib.vc_cuda_stream())
    ctx = Ctx(be, B, _abi, rank, args.rows, torch, world)
    if args.config_only:
        print(json.dumps(measure_config(args.config_only, ctx, torch, vstream, args, torch.cuda.synchronize)))
        return
    wl = WORKLOADS[args.workload](ctx)
    torch.cuda.empty_cache()  # inputs generated with torch now live in the library's pool
    ops = wl["ops"]
    n = wl["elements"]

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    timer = Timer(torch, vstream, flush_l2=args.workload != "cfg1")
    # warm-up, then the timed steps (launches counted in the timed steps only)
    timer.run(ops, 0, args.warmup, barrier)
    ctx.launches = 0
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record(vstream)
        per_op_ms = timer.run(ops, args.steps, 0, barrier)
        stop.record(vstream)
        barrier()
    total_ms = start.elapsed_time(stop)
    gpu_launches = ctx.launches
    step_ms_local = sum(per_op_ms) / args.steps  # device time of the ops (no host readback gaps)
    t = torch.tensor([step_ms_local], dtype=torch.float64)  # host tensor: gloo
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms = float(t.item())
    bytes_per_step = sum(nb for _, nb, _ in ops)  # this rank's
    n_global = wl.get("elements_global", world * n)
    bytes_global = bytes_per_step * n_global / n
    value = bytes_global / (step_ms * 1e-3) / 1e9
    per_op = {name: {"ms": round(per_op_ms[i] / args.steps, 4),
                     "gbs": round(nb / (per_op_ms[i] / args.steps * 1e-3) / 1e9, 1)}
              for i, (name, nb, _) in enumerate(ops)}
    peak, peak_kind = hbm_peak()
    dom = max(range(len(ops)), key=lambda i: per_op_ms[i])
    dom_name, dom_bytes, _ = ops[dom]
    dom_ms = per_op_ms[dom] / args.steps
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    traffic = None
    try:
        tr = json.loads(TRAFFIC_FILE.read_text())
        key = f"{args.workload}:{dom_name}"
        if key in tr.get("bytes_per_element", {}):
            traffic = round(tr["bytes_per_element"][key] * n)
    except Exception:
        pass

    e2e = None
    if not args.no_e2e and "host" in wl:
        # a second device set of the same inputs for the double-buffered loop
        wl2 = WORKLOADS[args.workload](ctx)
        e2e = measure_e2e(args, [wl, wl2], barrier, dist, torch, bytes_global, world, n)
        del wl2
    desc, metric, nops = wl["desc"], wl["metric"], len(ops)
    del wl, ops
    release(be, torch)

    sharded = None
    if not args.no_sharded:
        sharded = sharded_reduction(args, ctx, timer, barrier, dist, world, rank)
        release(be, torch)

    per_config = None
    if world == 1 and not args.no_per_config and args.workload == "cfg2" and not args.rows:
        # each configuration in a process of its own, as `--workload cfgN`
        # runs it: timed after this process's sweep, configuration 4's kernels
        # all measured 5-9% slower on the same box, for a reason in the
        # process's state that was not found (not host latency, allocation
        # churn, clocks or temperature)
        per_config = {}
        for name in ("cfg1", "cfg3", "cfg4", "cfg5"):
            per_config[name] = config_in_child(name, args)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "cfg2":
        cpu = reference_cpu_sample(repeats=2)

    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": metric,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4),
        "higher_is_better": True,
        "scaling": "strong" if args.workload == "cfg2" else "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded generators with the benchmark table's shapes and distributions)",
        "config": {"workload": desc, "elements_global": n_global,
                   "elements_per_gpu": n,
                   "l2": "inputs larger than the 126 MB L2, and L2 flushed before every timed op (a 256 MiB read)"
                   if args.workload != "cfg1"
                   else "16.8 MB working set stays in L2 by design (launch-bound configuration)",
                   "parallelism": f"axis-0 shards of the global tensor over {world} GPU(s), no data-path "
                                  "communication" if args.workload == "cfg2" else f"replicas x{world}"},
        "elements_per_s": round(nops * n_global / (step_ms * 1e-3), 1),
        "pct_of_peak": round(100 * value / world / peak, 1),
        "per_op": per_op,
        "roofline": {"bound": "hbm", "kernel": dom_name, "achieved": round(achieved, 1), "peak": peak,
                     "peak_kind": f"{peak_kind} hbm_gbs (copy, burst)", "unit": "GB/s",
                     "frac": round(achieved / peak, 3), "traffic": traffic,
                     "algorithmic_bytes_per_launch": dom_bytes},
        "clocks": clocks.summary(),
        "gpu_launches": gpu_launches,
        "e2e": e2e,
        "cpu_baseline": cpu,
        "sharded_reduction": sharded,
        "per_config": per_config,
        "wall_ms_timed_region": round(total_ms, 2),
    }
    print(json.dumps(line), flush=True)


def wl_metric(name):
    return {"cfg1": "effective GB/s (config 1 bias+relu+sum, fwd+bwd)",
            "cfg2": "effective HBM GB/s (config 2 elementwise sweep, fwd+bwd)",
            "cfg3": "effective HBM GB/s (config 3 reductions, fwd+bwd)",
            "cfg4": "effective HBM GB/s (config 4 softmax / cross-entropy, fwd+bwd)",
            "cfg5": "effective HBM GB/s (config 5 strided broadcast multiply, fwd+bwd)"}[name]


def config_in_child(name, args):
    """measure_config(name) in a fresh process on this process's GPU."""
    cmd = [sys.executable, str(ROOT / "bench.py"), "--config-only", name, "--steps", str(args.steps)]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env, cwd=str(ROOT))
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    if out.returncode != 0 or not lines:
        raise RuntimeError(f"per-configuration run of {name} failed (exit {out.returncode}): {out.stderr[-2000:]}")
    return json.loads(lines[-1])


def measure_config(name, ctx, torch, vstream, args, barrier):
    """Per-op GB/s of another configuration at its full shape on this GPU
    (same timing rules as the headline: warm-up, CUDA events, L2 flush)."""
    wl = WORKLOADS[name](ctx)
    torch.cuda.empty_cache()  # as the headline path: the inputs now live in the library's pool
    ops = wl["ops"]
    steps = max(1, min(args.steps, 5))
    per_op_ms = Timer(torch, vstream, flush_l2=name != "cfg1").run(ops, steps, 3, barrier)
    step_ms = sum(per_op_ms) / steps
    nbytes = sum(nb for _, nb, _ in ops)
    peak, _ = hbm_peak()
    res = {"metric": wl_metric(name), "workload": wl["desc"], "steps": steps, "warmup": 3,
           "ms_per_step": round(step_ms, 4), "value": round(nbytes / (step_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
           "per_op": {op: {"ms": round(per_op_ms[i] / steps, 4),
                           "gbs": round(nb / (per_op_ms[i] / steps * 1e-3) / 1e9, 1),
                           "frac": round(nb / (per_op_ms[i] / steps * 1e-3) / 1e9 / peak, 3)}
                      for i, (op, nb, _) in enumerate(ops)}}
    if name == "cfg1":
        res["us_per_step"] = round(step_ms * 1e3, 2)
        res["roofline_l2"] = l2_roofline(torch, vstream, nbytes, step_ms, per_op_ms, steps, ops)
    return res


def l2_roofline(torch, vstream, nbytes, step_ms, per_op_ms, steps, ops):
    """Configuration 1's 16.8 MB stays in the 126 MB L2, so its ceiling is L2
    bandwidth, not HBM: measured here as one CUDA graph of 100 back-to-back
    copies between two 32 MiB buffers that stay L2-resident (read + write
    bytes / replay time), together with the floor of one empty kernel between
    the same pair of events (the step is two kernels, replayed as one graph)."""
    src = torch.ones(8 << 20, dtype=torch.float32, device="cuda")
    dst = torch.empty_like(src)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            dst.copy_(src)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    reps = 100
    with torch.cuda.graph(graph, stream=side):
        for _ in range(reps):
            dst.copy_(src)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(vstream):
        graph.replay()
        times = []
        for _ in range(5):
            e0.record(vstream)
            graph.replay()
            e1.record(vstream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
    l2_gbs = reps * 2 * src.numel() * 4 / (min(times) * 1e-3) / 1e9
    del graph
    tiny = torch.zeros(1, dtype=torch.float32, device="cuda")
    lat = []
    with torch.cuda.stream(vstream):
        for _ in range(50):
            e0.record(vstream)
            tiny.add_(1.0)
            e1.record(vstream)
            torch.cuda.synchronize()
            lat.append(e0.elapsed_time(e1))
    floor_us = statistics.median(lat) * 1e3
    achieved = nbytes / (step_ms * 1e-3) / 1e9
    return {"bound": "l2", "achieved": round(achieved, 1), "peak": round(l2_gbs, 1), "unit": "GB/s",
            "peak_kind": "measured L2-resident copy (one graph of 100 copies between two 32 MiB buffers)",
            "frac": round(achieved / l2_gbs, 3), "bytes_per_step": nbytes,
            "l2_time_floor_us": round(nbytes / (l2_gbs * 1e9) * 1e6, 2),
            "empty_kernel_us": round(floor_us, 2), "us_per_step": round(step_ms * 1e3, 2),
            "note": "the step (one graph of two kernels) against the L2 copy rate; an empty kernel between the "
                    "same events shows the per-launch floor that dominates a step this small"}


def sharded_reduction(args, ctx, timer, barrier, dist, world, rank):
    """Configuration 3's reductions over the sharded axis at `world` GPUs:
    x [8192, 32768] ~ N(0,1) row-sharded; per step the axis-0 sum, the
    axis-0 max with its argmax and the full sum, each as a per-rank partial
    (vc_cuda_reduce_axis_partial), the CUDA device's NCCL all-gather and the
    rank-order combine (vc_cuda_combine_partials). Timed with CUDA events
    (max over ranks); a second loop times the local partials alone, so the
    difference is the collective + combine. Every rank checks its results
    against the 1-GPU reduction of the whole tensor (computed on rank 0):
    bit for bit for max / argmax, within 1e-5 for the sums."""
    import torch

    from vectorcore_b200 import dist as vdist

    be, B, abi = ctx.be, ctx.B, ctx.abi
    rows, cols = 8192, 32768
    sh = vdist.RowShard(rows, world, rank)
    xl = be.upload(normal_rows(4, 1.0, sh.start, sh.stop, cols))
    if world > 1:
        comm = vdist.Communicator.from_torch(timeout_ms=120_000)
    else:
        comm = vdist.Communicator(1, 0, vdist.Communicator.unique_id(), timeout_ms=120_000)
    res = {}

    def full_op():
        res["sum0"], res["max0"], res["sum"] = vdist.axis0_reductions(xl, sh.count, cols, comm, sh)

    def p(st):
        return None if st is None else ctypes.c_void_p(st.ptr)

    ps, pv, pi, pt = (be.allocate(cols, np.float64), be.allocate(cols), be.allocate(cols, np.int64),
                      be.allocate(1, np.float64))

    def local_op():
        abi.call("vc_cuda_reduce_axis_partial", B.REDUCE_SUM, p(xl), ctypes.c_size_t(1), ctypes.c_size_t(sh.count),
                 ctypes.c_size_t(cols), ctypes.c_int64(0), 0, p(ps), None, None)
        abi.call("vc_cuda_reduce_axis_partial", B.REDUCE_MAX, p(xl), ctypes.c_size_t(1), ctypes.c_size_t(sh.count),
                 ctypes.c_size_t(cols), ctypes.c_int64(sh.start), int(sh.rank > 0), None, p(pv), p(pi))
        abi.call("vc_cuda_reduce_axis_partial", B.REDUCE_SUM, p(xl), ctypes.c_size_t(1),
                 ctypes.c_size_t(sh.count * cols), ctypes.c_size_t(1), ctypes.c_int64(0), 0, p(pt), None, None)

    steps = max(1, args.steps)
    # a 2 ms lead (GPU sleep) before each step hides the host's enqueue of
    # the step (partials, the NCCL group, combines) from the device timing
    dev_timer = Timer(torch, timer.vstream, flush_l2=True, lead_cycles=4_000_000)
    ms_full = dev_timer.run([("sharded", 0, full_op)], steps, max(3, args.warmup), barrier)[0] / steps
    ms_local = dev_timer.run([("local", 0, local_op)], steps, 3, barrier)[0] / steps
    barrier()
    t0 = time.perf_counter()  # host wall time of back-to-back synchronous steps, for context
    for _ in range(steps):
        full_op()
        comm.synchronize()
    ms_wall = (time.perf_counter() - t0) * 1e3 / steps
    t = torch.tensor([ms_full, ms_local, ms_wall], dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_full, ms_local, ms_wall = float(t[0]), float(t[1]), float(t[2])
    got = {"sum0": be.download(res["sum0"]), "max0": be.download(res["max0"][0]),
           "arg0": be.download(res["max0"][1]), "sum": be.download(res["sum"])}
    # the 1-GPU results of the whole tensor, on rank 0
    expect = [None]
    if rank == 0:
        xf = be.upload(normal_rows(4, 1.0, 0, rows, cols))
        v, i = be.reduce_axis(xf, 1, rows, cols, B.REDUCE_MAX, want_index=True)
        expect[0] = {"sum0": be.download(be.reduce_axis(xf, 1, rows, cols, B.REDUCE_SUM)), "max0": be.download(v),
                     "arg0": be.download(i), "sum": be.download(be.reduce_sum(xf, rows * cols))}
        del xf
    if dist is not None:
        dist.broadcast_object_list(expect, src=0)
    e = expect[0]
    ok = {"sum_axis0": bool(np.allclose(got["sum0"], e["sum0"], rtol=1e-5, atol=1e-5 * np.sqrt(rows))),
          "max_axis0_bitexact": bool(np.array_equal(got["max0"].view(np.uint32), e["max0"].view(np.uint32))),
          "argmax_axis0": bool(np.array_equal(got["arg0"], e["arg0"])),
          "sum_all": bool(abs(float(got["sum"][0]) - float(e["sum"][0])) <= 1e-5 * np.sqrt(rows * cols))}
    oks = [ok]
    if dist is not None:
        oks = [None] * world
        dist.all_gather_object(oks, ok)
    comm.close()
    n_global = rows * cols
    nbytes = 3 * 4 * n_global  # each of the three reductions reads the global tensor once
    return {"workload": f"cfg3: x [{rows},{cols}] f32 sharded along axis 0 over {world} GPU(s) ({sh.count} rows "
                        "on rank 0): axis-0 sum, axis-0 max+argmax, full sum -- per-rank partials, NCCL "
                        "all-gather, rank-order combine",
            "n_gpus": world, "steps": steps, "ms_per_step": round(ms_full, 4),
            "value": round(nbytes / (ms_full * 1e-3) / 1e9, 1), "unit": "GB/s",
            "elements_per_s": round(3 * n_global / (ms_full * 1e-3), 1),
            "local_reduce_ms": round(ms_local, 4),
            "collective_and_combine_ms": round(max(0.0, ms_full - ms_local), 4),
            "host_wall_ms_per_step": round(ms_wall, 4),
            "limiter": ("collective + combine" if ms_full - ms_local > ms_local else "local reduction"),
            "collective": f"one grouped NCCL all-gather of the four partials per step over {world} rank(s) "
                          "(vc_cuda_comm_allgather_group)",
            "matches_1gpu": {f"rank{r}": o for r, o in enumerate(oks)}}


def measure_e2e(args, sets, barrier, dist, torch, bytes_global, world, n):
    """The same step through the public API with host buffers: every step
    uploads its inputs from page-locked host memory and reads its final
    result back. The copies are asynchronous (vc_cuda_upload_async /
    vc_cuda_download_async) and the inputs double-buffered like a
    prefetching loader: step i+1's inputs upload into the other device set
    while step i computes, each op waits only for the inputs it reads
    (transfer_wait before its first use), and step i's result download
    overlaps the following uploads. One untimed warm-up step, then timed on
    the host from the first upload to the last byte read."""
    from vectorcore_b200 import backend as B

    be = B.CudaBackend.instance()
    wl = sets[0]
    pins = {}
    for k, arr in wl["host"].items():
        pins[k] = B.PinnedBuffer(arr.size, arr.dtype)
        pins[k].array[:] = arr
    out_pin = B.PinnedBuffer(n)
    first_use = wl.get("first_use", {k: 0 for k in pins})

    def upload(s):
        return {k: be.upload_async(s["dev"][k], pins[k]) for k in pins}

    def run(s, tickets):
        outs = []
        for i, (_, _, fn) in enumerate(s["ops"]):
            for k, first in first_use.items():
                if first == i:
                    be.transfer_wait(tickets[k])
            outs.append(fn())
        last = outs[-1]
        be.download_async(out_pin, last, last.nbytes)

    def loop(steps):
        tickets = upload(sets[0])
        for i in range(steps):
            nxt = upload(sets[(i + 1) % len(sets)]) if i + 1 < steps else None  # prefetch
            run(sets[i % len(sets)], tickets)
            tickets = nxt
        be.synchronize()

    loop(1)  # warm-up: copy streams, events, staging of the first tickets
    # the pipeline fills with one step's upload and drains with one step's
    # compute and download: time 40 steps (~2.6 s) so the steady state
    # dominates, as in a long-running loader
    steps = 40
    barrier()
    t0 = time.perf_counter()
    loop(steps)
    barrier()
    secs = (time.perf_counter() - t0) / steps
    if dist is not None:
        te = torch.tensor([secs], dtype=torch.float64)
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
        secs = float(te.item())
    h2d = sum(p.nbytes for p in pins.values())
    for p in pins.values():
        p.close()
    out_pin.close()
    return {"value": round(bytes_global / secs / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": n * 4 * world,
            "h2d_bytes_per_step_per_gpu": h2d, "d2h_bytes_per_step_per_gpu": n * 4, "steps": steps,
            "note": "page-locked host inputs uploaded and the step's last gradient read back every step through "
                    "the C ABI: asynchronous copies, inputs double-buffered (the next step's upload overlaps this "
                    "step's compute), each op waits only for the inputs it reads"}


# --------------------------------------------------------------------------------------
# Reference arm: the reference's own CPU path (oracle/_ref, compiled from its sources)
# --------------------------------------------------------------------------------------
REF_SAMPLE = (4096, 16384)  # 2^26 elements (256 MB per tensor, beyond CPU caches)
SWEEP_BYTES_PER_ELEMENT = 208  # sum of the cfg2 ops' algorithmic bytes per element


def _ref_module():
    ref_dir = ROOT / "oracle" / "_ref"
    if not any(ref_dir.glob("vectorcore*.so")):
        return None, f"reference CPU module not built in {ref_dir} (make -C oracle ref)"
    sys.path.insert(0, str(ref_dir))
    import vectorcore as vc  # the reference's own pybind11 module

    return vc, None


def reference_sweep_once(vc, a, b, g, a1):
    """One config-2 sweep through the reference's public Python API: each op
    forward, then backward with the dense upstream g."""
    ops = [
        ("add", lambda x, y: x + y, 2), ("sub", lambda x, y: x - y, 2), ("mul", lambda x, y: x * y, 2),
        ("div", lambda x, y: x / y, 2), ("neg", lambda x: -x, 1), ("exp", lambda x: x.exp(), 1),
        ("log", lambda x: x.log(), 1), ("relu", lambda x: x.relu(), 1), ("sigmoid", lambda x: x.sigmoid(), 1),
        ("scalar_mul", lambda x: x * 0.5, 1),
    ]
    for name, fn, arity in ops:
        if arity == 2:
            y = fn(a, b)
        else:
            y = fn(a if name in ("exp", "log", "scalar_mul") else a1)
        y.backward(g)
        for t in (a, b, a1):
            t.zero_grad()


def _ref_inputs(vc, rows):
    """The first `rows` rows of the benchmark's global a, b, g (the same
    block-wise generators as our arm) as the reference's own tensors; a1 =
    a - 1 is the signed input of neg / relu / sigmoid."""
    c = CFG2_COLS
    a_np = uniform_rows(2, 0.1, 2.0, 0, rows, c)
    a = vc.Tensor(a_np, requires_grad=True)
    b = vc.Tensor(uniform_rows(3, 0.1, 2.0, 0, rows, c), requires_grad=True)
    g = vc.Tensor(uniform_rows(9, -1.0, 1.0, 0, rows, c))
    a1 = vc.Tensor(a_np - np.float32(1.0), requires_grad=True)
    return a, b, g, a1


def _ref_threads():
    try:
        import oracle

        return oracle.reference().threads() if oracle.reference_available() else os.cpu_count()
    except Exception:
        return os.cpu_count()


def reference_cpu_sample(repeats=2):
    vc, why = _ref_module()
    if vc is None:
        return {"value": None, "unit": "GB/s", "cores": os.cpu_count(), "kind": "reference", "sample": why}
    a, b, g, a1 = _ref_inputs(vc, REF_SAMPLE[0])
    reference_sweep_once(vc, a, b, g, a1)  # warm-up (page faults, pool threads)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        reference_sweep_once(vc, a, b, g, a1)
        times.append(time.perf_counter() - t0)
    secs = statistics.median(times)
    n = REF_SAMPLE[0] * REF_SAMPLE[1]
    return {"value": round(SWEEP_BYTES_PER_ELEMENT * n / secs / 1e9, 2), "unit": "GB/s",
            "cores": _ref_threads(), "kind": "reference",
            "sample": f"config-2 sweep fwd+bwd on [{REF_SAMPLE[0]},{REF_SAMPLE[1]}] (2^26 elements), median of "
                      f"{repeats} after 1 warm-up; the reference's thread pool uses hardware_concurrency() threads"}


def run_reference(args):
    """The reference's own CPU path (its pybind11 module over its thread
    pool, compiled from its sources into oracle/_ref) on the full
    configuration-2 workload: the [16384, 16384] sweep, forward and backward
    through its public Python API. Rank 0 alone runs it."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    vc, why = _ref_module()
    if vc is None:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return
    rows = args.rows or CFG2_ROWS
    a, b, g, a1 = _ref_inputs(vc, rows)
    for _ in range(args.warmup):
        reference_sweep_once(vc, a, b, g, a1)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        reference_sweep_once(vc, a, b, g, a1)
    secs = (time.perf_counter() - t0) / args.steps
    n = rows * CFG2_COLS
    value = SWEEP_BYTES_PER_ELEMENT * n / secs / 1e9
    threads = _ref_threads()
    line = {
        "impl": "reference",
        "metric": "effective HBM GB/s (config 2 elementwise sweep, fwd+bwd)",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(secs * 1e3, 2), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (the same block-wise seeded generators as our arm)",
        "config": {"workload": f"cfg2: same-shape elementwise sweep, a,b,g [{rows},{CFG2_COLS}] f32, "
                               "add/sub/mul/div/neg/exp/log/relu/sigmoid/a*0.5 fwd+bwd, on the reference's CPU "
                               "path (its thread pool on the host's cores)",
                   "elements_global": n},
        "cpu_baseline": {"value": round(value, 2), "unit": "GB/s", "cores": threads, "kind": "reference",
                         "sample": f"the full [{rows},{CFG2_COLS}] sweep per step"},
        "e2e": {"value": round(value, 2), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="cfg2", choices=sorted(WORKLOADS))
    ap.add_argument("--rows", type=int, default=0, help="shrink the leading dimension (profiling cases)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sharded", action="store_true", help="skip the sharded-reduction block")
    ap.add_argument("--no-per-config", action="store_true", help="skip the other configurations (N = 1)")
    ap.add_argument("--config-only", choices=sorted(WORKLOADS), default=None,
                    help="time one configuration as the per_config block does and print its JSON (the default "
                         "run starts one such process per extra configuration)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    args.warmup = max(args.warmup, 3)
    run_ours(args)


if __name__ == "__main__":
    main()

"""Seeded synthetic inputs for the five benchmark configurations.

The reference publishes no dataset for this path; every input is drawn with
numpy ``default_rng(seed)`` as float32, exactly as the configuration table of
the benchmark describes (distribution, shape, seed). ``scale`` shrinks the
shapes for CPU-sized parity cases while keeping the layout (which axes
broadcast, which are reduced) of the full configuration.
"""
from __future__ import annotations

import numpy as np


def uniform(seed, shape, low, high):
    return np.random.default_rng(seed).uniform(low, high, size=shape).astype(np.float32)


def normal(seed, shape, mean=0.0, std=1.0):
    return np.random.default_rng(seed).normal(mean, std, size=shape).astype(np.float32)


def integers(seed, high, size):
    return np.random.default_rng(seed).integers(0, high, size=size).astype(np.int64)


# ---- configuration shapes ------------------------------------------------

CFG1 = {"x": (1024, 4096), "b": (4096,)}
CFG2 = {"a": (16384, 16384)}
CFG3 = {"x": (8192, 32768)}
CFG4 = {"logits": (65536, 32000)}
CFG5 = {"a": (64, 1, 512, 1024), "b": (1, 128, 1, 1024)}


def cfg1(shape_x=CFG1["x"]):
    """Bias + ReLU + sum: x ~ U(-1,1) seed 0, b ~ N(0,1) seed 1."""
    x = uniform(0, shape_x, -1.0, 1.0)
    b = normal(1, (shape_x[-1],))
    return x, b


def cfg2(shape=CFG2["a"]):
    """Same-shape sweep: a, b ~ U(0.1, 2) seeds 2/3; upstream g ~ U(-1,1) seed 9."""
    return uniform(2, shape, 0.1, 2.0), uniform(3, shape, 0.1, 2.0), uniform(9, shape, -1.0, 1.0)


def cfg3(shape=CFG3["x"]):
    """Reductions: x ~ N(0,1) seed 4."""
    return normal(4, shape)


def cfg4(shape=CFG4["logits"]):
    """Softmax / cross-entropy: logits ~ N(0, 2) seed 5; targets U{0..C-1} seed 6."""
    logits = normal(5, shape, 0.0, 2.0)
    targets = integers(6, shape[1], shape[0])
    return logits, targets


def cfg5(shape_a=CFG5["a"], shape_b=CFG5["b"]):
    """Strided broadcast multiply: a, b ~ U(-1,1) seeds 7/8."""
    return uniform(7, shape_a, -1.0, 1.0), uniform(8, shape_b, -1.0, 1.0)


# Small-scale shapes used for golden fixtures and CPU-sized parity runs.
SMALL = {
    "cfg1": {"x": (256, 512)},
    "cfg2": {"a": (32, 64)},
    "cfg3": {"x": (32, 256)},
    "cfg4": {"logits": (8, 1000)},
    "cfg5": {"a": (4, 1, 8, 64), "b": (1, 16, 1, 64)},
}

# Broadcast layouts of the reference's own tests
# (tests/python/test_performance_paths.py:106-116).
BROADCAST_CASES = [
    ((1000, 300), (1000, 300)),
    ((1000, 300), ()),
    ((), (1000, 300)),
    ((1000, 300), (300,)),
    ((1000, 300), (1000, 1)),
    ((1000, 1), (1, 300)),
    ((40, 1, 300), (1, 50, 300)),
    ((40, 50, 1), (50, 7)),
    ((3,), (2, 1)),
    # long rows (the warp-per-row path): two leading dims, a row-constant
    # operand, and rows long enough for its four-deep unrolled loop
    ((16, 1, 1000), (1, 9, 1000)),
    ((5, 7, 1, 2052), (7, 3, 2052)),
    ((60, 1), (1, 1028)),
    # operand reuse along a leading dim (one operand constant along it): a
    # partial run of the reused dim and a partial column chunk; the operand
    # kept in registers chosen by footprint, the other constant along rows
    ((3, 1, 40, 516), (1, 33, 1, 516)),
    ((2, 20, 1, 260), (2, 1, 17, 1)),
]

# sum_to_shape layouts (tests/python/test_performance_paths.py:162-176) plus
# the two benchmark layouts.
SUM_TO_SHAPE_CASES = [
    ((8, 5, 7), (7,)),
    ((8, 5, 7), (5, 1)),
    ((8, 5, 7), (8, 1, 7)),
    ((8, 5, 7), (1, 1, 1)),
    ((8, 5, 7), ()),
    ((256, 512), (512,)),
    ((4, 16, 8, 64), (4, 1, 8, 64)),
    ((4, 16, 8, 64), (1, 16, 1, 64)),
]

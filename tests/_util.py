"""Comparison helpers with the tolerance classes of the parity contract.

* bit-exact: add, sub, mul, div, neg, relu, max, argmax (NaNs compare equal
  whatever their payload: glibc and CUDA encode NaN differently);
* <= 2 ulp: exp, log, sigmoid (CUDA expf/logf vs glibc);
* sums, means, softmax, cross-entropy: relative 1e-5, with the reference
  magnitude floored at the random-walk scale sqrt(n) * rms of the summed
  terms (SUM_RTOL below).
"""
import hashlib

import numpy as np

SUM_RTOL = 1e-5
ULP_MAX = 2


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def assert_bitexact(got, ref, what=""):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    both_nan = np.isnan(got) & np.isnan(ref)
    same = (bits(got) == bits(ref)) | both_nan
    if not same.all():
        idx = np.flatnonzero(~same.reshape(-1))
        i = idx[0]
        raise AssertionError(f"{what}: {idx.size} of {got.size} elements differ bitwise; first at {i}: "
                             f"got {got.reshape(-1)[i]!r} ref {ref.reshape(-1)[i]!r}")


def ulp_distance(got, ref):
    """Distance in units in the last place between float32 arrays (NaN vs
    NaN = 0; NaN vs number = huge)."""
    g = np.ascontiguousarray(got, np.float32).view(np.int32).astype(np.int64)
    r = np.ascontiguousarray(ref, np.float32).view(np.int32).astype(np.int64)
    # map to a monotonic integer line
    g = np.where(g < 0, -(g & 0x7FFFFFFF), g)
    r = np.where(r < 0, -(r & 0x7FFFFFFF), r)
    d = np.abs(g - r)
    gn, rn = np.isnan(got), np.isnan(ref)
    d = np.where(gn & rn, 0, d)
    d = np.where(gn ^ rn, 1 << 40, d)
    return d


def assert_ulp(got, ref, max_ulp=ULP_MAX, what=""):
    d = ulp_distance(got, ref)
    worst = int(d.max()) if d.size else 0
    assert worst <= max_ulp, f"{what}: max ulp distance {worst} > {max_ulp}"
    return worst


def assert_sum_close(got, ref, n, rms, rtol=SUM_RTOL, what=""):
    """|got - ref| <= rtol * max(|ref|, sqrt(n) * rms) elementwise."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = np.maximum(np.abs(ref), np.sqrt(max(n, 1)) * rms)
    err = np.abs(got - ref)
    bad = err > rtol * scale + 1e-30
    assert not bad.any(), (f"{what}: {int(bad.sum())} elements outside tolerance; worst rel "
                           f"{float(np.max(err / np.maximum(scale, 1e-30))):.3e}")


def assert_rel(got, ref, rtol=SUM_RTOL, what="", scale=None):
    """|got - ref| <= rtol * (|ref| + floor): relative, with a floor for
    entries far below the scale of the terms that produced them. The floor is
    1e-3 * max|ref|, or 0.1 * `scale` when given -- backward results are sums
    g + de*e whose terms have the magnitude of the upstream gradient, so a
    near-cancellation leaves an absolute error of a few ulp of `scale`."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    both_nan = np.isnan(got) & np.isnan(ref)
    floor = 1e-3 * (np.max(np.abs(ref[np.isfinite(ref)])) if np.isfinite(ref).any() else 0.0)
    if scale is not None:
        floor = max(floor, 0.1 * float(scale))
    err = np.where(both_nan, 0.0, np.abs(got - ref))
    bad = err > rtol * (np.abs(ref) + floor)
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {got.size} outside rtol {rtol}; worst abs err "
                           f"{float(np.nanmax(err)):.3e}")


def sha256(a):
    return hashlib.sha256(np.ascontiguousarray(a, np.float32).tobytes()).hexdigest()

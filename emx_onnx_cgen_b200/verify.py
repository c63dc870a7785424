"""Output comparison with the reference's verification metric.

The reference's ``verify`` command accepts a floating output when its worst
element-wise ULP distance to the expected output is at most ``--max-ulp``
(default 100), skipping pairs whose absolute difference is within
``atol_eps * eps(dtype)`` (default 1.0); verification.py:25-60 and
shared/ulp.py:26-58 define it:

* same sign: the distance of the two bit patterns as unsigned integers;
* opposite signs: ulp(0, |a|) + ulp(0, |b|) + 1;
* NaN against NaN: 0; NaN against a number: the largest unsigned value.

Integer and boolean outputs must match exactly.  This module computes the
same numbers vectorised (uint64 arithmetic, so fp64 distances do not wrap).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

_UINT = {np.dtype(np.float16): np.uint16, np.dtype(np.float32): np.uint32, np.dtype(np.float64): np.uint64}


def ulp_distance(actual: np.ndarray, expected: np.ndarray, atol_eps: float = 1.0) -> np.ndarray:
    """Per-element distance (uint64 array, ``expected``'s shape) in the dtype
    of ``expected``; pairs within the absolute tolerance count 0."""
    expected = np.asarray(expected)
    actual = np.asarray(actual)
    if actual.shape != expected.shape:
        raise ValueError(f"shape mismatch for ULP calculation: {actual.shape} vs {expected.shape}")
    dt = expected.dtype
    if dt not in _UINT:
        raise ValueError(f"unsupported floating dtype for ULP calculation: {dt}")
    ut = _UINT[dt]
    a = np.ascontiguousarray(actual.astype(dt, copy=False)).reshape(-1)
    b = np.ascontiguousarray(expected).reshape(-1)
    nbits = np.dtype(ut).itemsize * 8
    sign = np.uint64(1) << np.uint64(nbits - 1)
    ia = a.view(ut).astype(np.uint64)
    ib = b.view(ut).astype(np.uint64)
    ma, mb = ia & (sign - np.uint64(1)), ib & (sign - np.uint64(1))
    same = (ia & sign) == (ib & sign)
    d = np.where(same, np.where(ia > ib, ia - ib, ib - ia), ma + mb + np.uint64(1))
    na, nb = np.isnan(a), np.isnan(b)
    d = np.where(na & nb, np.uint64(0), np.where(na | nb, np.uint64(np.iinfo(ut).max), d))
    with np.errstate(invalid="ignore", over="ignore"):
        close = np.abs(a.astype(np.float64) - b.astype(np.float64)) <= float(np.finfo(dt).eps) * atol_eps
    return np.where(close, np.uint64(0), d).reshape(expected.shape)


@dataclass
class OutputCheck:
    name: str
    ok: bool
    max_ulp: int | None        # floating outputs
    mismatches: int            # elements over the limit (floating) or unequal (integer)
    worst: tuple | None        # (index, actual, expected) of the worst element
    message: str


def check_output(name: str, actual: np.ndarray, expected: np.ndarray, max_ulp: int = 100,
                 atol_eps: float = 1.0) -> OutputCheck:
    actual, expected = np.asarray(actual), np.asarray(expected)
    if actual.shape != expected.shape:
        return OutputCheck(name, False, None, -1, None, f"{name}: shape {actual.shape}, expected {expected.shape}")
    if expected.dtype in _UINT:
        d = ulp_distance(actual, expected, atol_eps)
        worst_ulp = int(d.max()) if d.size else 0
        over = int((d > np.uint64(max_ulp)).sum())
        worst = None
        if d.size and worst_ulp:
            idx = np.unravel_index(int(np.argmax(d)), d.shape)
            worst = (tuple(int(i) for i in idx), float(actual[idx]), float(expected[idx]))
        ok = worst_ulp <= max_ulp
        msg = f"{name}: max ULP {worst_ulp}" + ("" if ok else f" > {max_ulp} ({over} elements; worst at {worst})")
        return OutputCheck(name, ok, worst_ulp, over, worst, msg)
    neq = actual != expected
    n = int(neq.sum())
    worst = None
    if n:
        idx = np.unravel_index(int(np.argmax(neq)), neq.shape)
        worst = (tuple(int(i) for i in idx), actual[idx].item(), expected[idx].item())
    return OutputCheck(name, n == 0, None, n, worst,
                       f"{name}: exact" if n == 0 else f"{name}: {n} elements differ (first at {worst})")

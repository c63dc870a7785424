"""Shared helpers for the GPU parity tests (they call the C-ABI library)."""
from __future__ import annotations

import numpy as np
import pytest

from emx_onnx_cgen_b200 import lowering
from emx_onnx_cgen_b200.plan import B200PlanEmitter


def require_gpu():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from emx_onnx_cgen_b200.runtime import load_library
    load_library()  # fails loudly if libemx_b200.so is missing


def plan_for(workload, **kw):
    return B200PlanEmitter(**kw).emit_plan(lowering.lower(workload.graph))


def assert_bitexact(got: np.ndarray, ref: np.ndarray, what: str = ""):
    """Identical bits, except that any NaN equals any NaN (x86 and the GPU
    produce different NaN payloads; the reference's ULP metric treats NaN/NaN
    as equal, shared/ulp.py:26-50)."""
    assert got.shape == ref.shape and got.dtype == ref.dtype, (got.shape, ref.shape, got.dtype, ref.dtype)
    if got.dtype.kind == "f":
        gn, rn = np.isnan(got), np.isnan(ref)
        assert np.array_equal(gn, rn), f"{what}: NaN positions differ"
        got = np.where(gn, 0, got).astype(got.dtype)
        ref = np.where(rn, 0, ref).astype(ref.dtype)
    if not np.array_equal(got.view(np.uint8), ref.view(np.uint8)):
        diff = np.argwhere(got != ref)
        raise AssertionError(f"{what}: {len(diff)} of {got.size} elements differ; first at {diff[:5].tolist()}: "
                             f"got {got[tuple(diff[0])]} expected {ref[tuple(diff[0])]}")


def ulp_diff_f16(got: np.ndarray, ref: np.ndarray, atol_eps: float = 1.0) -> np.ndarray:
    """Per-element ULP distance of fp16 arrays as the reference's verify
    metric defines it (shared/ulp.py:26-50, verification.py:30-50): same sign
    |bits(a) - bits(b)|, opposite signs ulp(0,|a|) + ulp(0,|b|) + 1, NaN/NaN 0,
    NaN/number 0xFFFF; pairs with |a - b| <= atol_eps * eps(fp16) count 0."""
    a = np.ascontiguousarray(got, np.float16).reshape(-1)
    b = np.ascontiguousarray(ref, np.float16).reshape(-1)
    ia = a.view(np.uint16).astype(np.int64)
    ib = b.view(np.uint16).astype(np.int64)
    mag_a, mag_b = ia & 0x7FFF, ib & 0x7FFF
    same = (ia >> 15) == (ib >> 15)
    d = np.where(same, np.abs(mag_a - mag_b), mag_a + mag_b + 1)
    na, nb = np.isnan(a), np.isnan(b)
    d = np.where(na & nb, 0, np.where(na | nb, 0xFFFF, d))
    with np.errstate(invalid="ignore"):
        close = np.abs(a.astype(np.float64) - b.astype(np.float64)) <= atol_eps * float(np.finfo(np.float16).eps)
    return np.where(close & ~(na | nb), 0, d).reshape(np.shape(got))


def ulp_diff_f32(got: np.ndarray, ref: np.ndarray, atol_eps: float = 1.0) -> np.ndarray:
    """fp32 counterpart of ulp_diff_f16 (shared/ulp.py:26-50 metric)."""
    a = np.ascontiguousarray(got, np.float32).reshape(-1)
    b = np.ascontiguousarray(ref, np.float32).reshape(-1)
    ia = a.view(np.uint32).astype(np.int64)
    ib = b.view(np.uint32).astype(np.int64)
    mag_a, mag_b = ia & 0x7FFFFFFF, ib & 0x7FFFFFFF
    same = (ia >> 31) == (ib >> 31)
    d = np.where(same, np.abs(mag_a - mag_b), mag_a + mag_b + 1)
    na, nb = np.isnan(a), np.isnan(b)
    d = np.where(na & nb, 0, np.where(na | nb, 0xFFFFFFFF, d))
    with np.errstate(invalid="ignore"):
        close = np.abs(a.astype(np.float64) - b.astype(np.float64)) <= atol_eps * float(np.finfo(np.float32).eps)
    return np.where(close & ~(na | nb), 0, d).reshape(np.shape(got))

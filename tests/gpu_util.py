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

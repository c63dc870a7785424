"""The int8 GEMM's zero-point algebra on the CPU (csrc/qgemm.cu header).

The tensor cores sum the raw 8-bit products; the epilogue restores the zero
points as  raw - zb * rowsum(A) - za * colsum(B) + K * za * zb  in uint32
arithmetic.  That must equal the reference's int32 sum of (a - za)(b - zb)
(oracle.matmul_integer) bit for bit, for every signedness and zero point, and
the raw sums must stay below 2^31 for K <= 32768 (no accumulator wraps).
"""
import numpy as np
import pytest

from oracle import oracle


def _epilogue(a: np.ndarray, b: np.ndarray, za: int, zb: int) -> np.ndarray:
    """The kernel's arithmetic: raw int32 products, then the uint32 correction."""
    k = a.shape[1]
    raw = (a.astype(np.int64) @ b.astype(np.int64)).astype(np.int32)     # tensor-core sums (int32)
    rowsum = a.astype(np.int64).sum(axis=1).astype(np.int32)             # prep launch
    colsum = b.astype(np.int64).sum(axis=0).astype(np.int32)             # planner / prep launch
    u32 = lambda v: np.asarray(v, np.int64).astype(np.uint32)
    kzz = u32(k) * u32(za) * u32(zb)
    row_corr = kzz - u32(zb) * rowsum.astype(np.uint32)
    acc = raw.astype(np.uint32) + row_corr[:, None] - u32(za) * colsum.astype(np.uint32)[None, :]
    return acc.view(np.int32)


@pytest.mark.parametrize("a_dt,b_dt,za,zb", [
    (np.uint8, np.int8, 128, 0), (np.uint8, np.int8, 0, 3), (np.uint8, np.uint8, 255, 255),
    (np.int8, np.int8, -128, 127), (np.int8, np.uint8, 5, 250), (np.uint8, np.int8, 0, 0),
])
def test_zero_point_restoration_matches_reference(a_dt, b_dt, za, zb):
    rng = np.random.default_rng(3)
    m, k, n = 37, 272, 29
    lo = lambda dt: -128 if dt == np.int8 else 0
    a = rng.integers(lo(a_dt), lo(a_dt) + 256, (m, k)).astype(a_dt)
    b = rng.integers(lo(b_dt), lo(b_dt) + 256, (k, n)).astype(b_dt)
    ref = oracle.matmul_integer(a, b, np.asarray(za, a_dt), np.asarray(zb, b_dt))
    assert np.array_equal(_epilogue(a, b, za, zb), ref)


def test_raw_sums_fit_int32_up_to_k_32768():
    k = 32768
    assert 255 * 255 * k < 2 ** 31          # u8 x u8, the largest products
    assert 128 * 128 * k < 2 ** 31          # s8 x s8: (-128)^2 * K = 2^29
    a = np.full((2, k), 255, np.uint8)
    b = np.full((k, 3), 255, np.uint8)
    ref = oracle.matmul_integer(a, b, np.asarray(0, np.uint8), np.asarray(0, np.uint8))
    assert np.array_equal(_epilogue(a, b, 0, 0), ref)

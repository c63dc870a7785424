"""fp32 Gemm -> Relu -> Gemm on the B200 kernels: bit-exact against the
reference's generated C (golden fixtures) and the CPU restatement, including
the full [64,1024] x [4096,1024]^T x [1024,4096]^T workload."""
import numpy as np
import pytest

from emx_onnx_cgen_b200 import workloads as W
from emx_onnx_cgen_b200.runtime import Session
from golden_util import cases, load
from gpu_util import assert_bitexact, plan_for, require_gpu
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(n for n in cases() if n.startswith("mlp")))
def test_golden(name):
    require_gpu()
    wl, inputs, ref = load(name)
    out = Session(plan_for(wl)).run(inputs)
    assert_bitexact(out["Y"], ref["Y"], name)


# beyond the default MLP: ragged rows / columns with many full 64-wide K stages and a partial
# last one, through the long-chain 32x16 tile (k 1100 -> hidden 1000; hidden 4000 -> 1000) and
# the 16x32 and 8x16 tiles
@pytest.mark.parametrize("kw", [dict(), dict(m=7, k=33, hidden=65), dict(m=300, k=16, hidden=40),
                                dict(m=1, k=1, hidden=1), dict(m=40, k=1100, hidden=1000),
                                dict(m=64, k=1000, hidden=4000)])
def test_vs_port(kw):
    require_gpu()
    wl = W.mlp_fp32(**kw)
    x = wl.make_inputs(5)
    ref = oracle.run_graph(wl.graph, x)["Y"]
    out = Session(plan_for(wl)).run(x)["Y"]
    assert_bitexact(out, ref, str(kw))


def test_signed_zero_and_specials():
    """-0.0 / inf / nan propagate exactly as in the reference loop."""
    require_gpu()
    wl = W.mlp_fp32(m=4, k=8, hidden=16)
    x = wl.make_inputs(0)["X"]
    x[0, :] = -0.0
    x[1, 3] = np.inf
    x[2, 5] = np.nan
    ref = oracle.run_graph(wl.graph, {"X": x})["Y"]
    out = Session(plan_for(wl)).run({"X": x})["Y"]
    assert_bitexact(out, ref, "specials")


def test_row_slices():
    require_gpu()
    wl = W.mlp_fp32(m=16, k=64, hidden=128)
    x = wl.make_inputs(9)["X"]
    ref = oracle.run_graph(wl.graph, {"X": x})["Y"]
    s = Session(plan_for(wl))
    y = np.zeros_like(ref)
    s.run_ptrs([x.ctypes.data], [y.ctypes.data], batch_begin=5, batch_count=7)
    s.sync()
    assert_bitexact(y[5:12], ref[5:12], "rows 5..11")

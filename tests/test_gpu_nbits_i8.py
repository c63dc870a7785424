"""com.microsoft MatMulNBits at accuracy_level 4 (the int8 activation path,
templates/matmul_nbits_int8_op.c.j2) on the B200: bit-exact against the
reference's generated C (golden fixtures) and the CPU restatement.  The
activations are quantised with the reference's float statements, the block
sums are exact int32 and every output repeats the reference's per-block
float steps in block order, so no tolerance applies (NaN equals NaN)."""
import numpy as np
import pytest

from emx_onnx_cgen_b200 import workloads as W
from emx_onnx_cgen_b200.runtime import Session
from golden_util import cases, load
from gpu_util import assert_bitexact, plan_for, require_gpu
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(n for n in cases() if n.startswith("nbits8_")))
def test_golden(name):
    require_gpu()
    wl, inputs, ref = load(name)
    plan = plan_for(wl)
    assert [o.kernel for o in plan.ops] == [25]  # K_NBITS_I8
    got = Session(plan).run(inputs)
    for k, v in ref.items():
        assert_bitexact(got[k], v, f"{name}:{k}")


@pytest.mark.parametrize("kw", [
    dict(m=64, k=512, n=192, block=32, zero_points="block", bias=True),
    dict(m=33, k=1000, n=72, block=32, zero_points="column"),
    dict(m=130, k=256, n=136, block=64),
    dict(m=7, k=4096, n=200, block=128, zero_points="block"),
])
def test_against_port(kw):
    require_gpu()
    wl = W.matmul_nbits_f16(accuracy_level=4, **kw)
    sess = Session(plan_for(wl))
    for seed in (0, 1):
        x = wl.make_inputs(seed)
        assert_bitexact(sess.run(x)["Y"], oracle.run_graph(wl.graph, x)["Y"], f"{kw} seed {seed}")


def test_specials():
    """Zero rows, +-inf and NaN activations, huge and tiny magnitudes."""
    require_gpu()
    wl = W.matmul_nbits_f16(m=8, k=96, n=40, block=32, zero_points="block", bias=True, accuracy_level=4)
    a = wl.make_inputs(4)["A"].copy()
    a[0] = 0.0
    a[1, 5] = np.inf
    a[2, 40] = -np.inf
    a[3, 7] = np.nan
    a[4] *= np.float16(6000.0)
    a[5] = np.float16(1e-7)
    a[6, :32] = np.float16(-0.0)
    got = Session(plan_for(wl)).run({"A": a})["Y"]
    assert_bitexact(got, oracle.run_graph(wl.graph, {"A": a})["Y"], "specials")

"""Failure detection on the GPU without a GPU fault: the bounded device waits.

A chained convolution stack (one persistent launch whose CTAs wait on each
other's per-tile progress words) runs with the failure-detection hook that
drops every progress publication -- a flag that nothing sets -- and a 20 ms
wait budget.  The waits run out, the kernels return, emx_b200_sync reports
EMX_ERR_DEVICE_TIMEOUT, and the same plan, hook off and default budget, then
runs bit-exact against the oracle again (the context stays usable and the
chain's epoch protocol recovers).  Nothing faults, traps or hangs: every wait
in the kernels is bounded.
"""
import time

import numpy as np
import pytest

from emx_onnx_cgen_b200 import kernel_ids as K
from emx_onnx_cgen_b200 import workloads as W
from emx_onnx_cgen_b200.runtime import FAULT_DROP_CHAIN_PROGRESS, EmxError, Session
from gpu_util import assert_bitexact, plan_for, require_gpu
from oracle import oracle

pytestmark = pytest.mark.gpu

EMX_ERR_DEVICE_TIMEOUT = 6


@pytest.mark.parametrize("use_graphs", [True, False])
def test_dropped_progress_times_out_and_recovers(use_graphs):
    require_gpu()
    wl = W.qconv_stack_int8(batch=2, height=16, width=16, wscale_range=(0.0001, 0.001))
    plan = plan_for(wl)
    assert any(op.kernel == K.K_QCONV_TC and op.ip.get(K.QC_CHAIN, 0) > 1 for op in plan.ops), "needs a chain"
    x = wl.make_inputs(5)
    ref = oracle.run_graph(wl.graph, x)["Y"]
    sess = Session(plan)
    sess.set_graphs(use_graphs)
    assert_bitexact(sess.run(x)["Y"], ref, "before")

    sess.set_wait_budget(20_000_000)  # 20 ms
    sess.set_fault(FAULT_DROP_CHAIN_PROGRESS)
    t0 = time.perf_counter()
    with pytest.raises(EmxError) as ei:
        sess.run(x)
    elapsed = time.perf_counter() - t0
    assert ei.value.status == EMX_ERR_DEVICE_TIMEOUT, str(ei.value)
    assert "gave up" in str(ei.value)
    assert elapsed < 1.5, f"the 20 ms budget was not applied ({elapsed:.2f} s)"

    sess.set_fault(0)
    sess.set_wait_budget(0)
    for k in range(3):  # the epoch protocol recovers: stale progress words are never trusted
        assert_bitexact(sess.run(x)["Y"], ref, f"after recovery, run {k + 1}")
    sess.close()


def test_unknown_hook_is_rejected():
    require_gpu()
    wl = W.qconv_stack_int8(batch=1, height=8, width=8, n_convs=2)
    sess = Session(plan_for(wl))
    with pytest.raises(EmxError) as ei:
        sess.set_fault(1 << 7)
    assert ei.value.status == 1
    sess.close()

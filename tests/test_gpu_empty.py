"""Graphs with a zero extent (the reference accepts zero dimensions) run
through the C ABI: the plan launches nothing, every output comes back with
its empty shape, and a graph of the same plan kind with rows still runs
afterwards in the same process."""
import numpy as np
import pytest

from emx_onnx_cgen_b200 import workloads as W
from emx_onnx_cgen_b200.runtime import Session
from gpu_util import assert_bitexact, plan_for, require_gpu
from test_plan import EMPTY_EXTENT_CASES

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(EMPTY_EXTENT_CASES))
def test_empty_extent_runs_without_launches(name):
    require_gpu()
    wl = EMPTY_EXTENT_CASES[name]()
    plan = plan_for(wl)
    s = Session(plan)
    try:
        before = s.launch_count()
        for _ in range(2):  # once through the graph capture path's first use, once after
            out = s.run(wl.make_inputs(0))
            for n, shp in zip(plan.output_names, plan.output_shapes):
                assert out[n].shape == tuple(shp) and out[n].size == 0, n
        assert s.launch_count() == before
    finally:
        s.close()


def test_rows_after_an_empty_plan():
    require_gpu()
    from oracle import oracle
    empty = Session(plan_for(EMPTY_EXTENT_CASES["mlp_rows0"]()))
    empty.run(EMPTY_EXTENT_CASES["mlp_rows0"]().make_inputs(0))
    empty.close()
    wl = W.mlp_fp32(m=3, k=8, hidden=16)
    s = Session(plan_for(wl))
    x = wl.make_inputs(1)
    got = s.run(x)
    s.close()
    ref = oracle.run_graph(wl.graph, x)
    for n in ref:
        assert_bitexact(got[n], np.asarray(ref[n]), f"mlp after an empty plan {n}")

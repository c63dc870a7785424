"""int8 QLinearConv / QLinearAdd stack on the B200 kernels vs the reference:
bit-exact against the reference's generated C (golden fixtures) and against
the CPU restatement at sizes and parameters the fixtures do not cover."""
import numpy as np
import pytest

from emx_onnx_cgen_b200 import kernel_ids as K, workloads as W
from emx_onnx_cgen_b200.runtime import Session
from golden_util import cases, load
from gpu_util import assert_bitexact, plan_for, require_gpu
from oracle import oracle

pytestmark = pytest.mark.gpu

QCONV_CASES = sorted(n for n in cases() if n.startswith("qconv"))


@pytest.mark.parametrize("name", QCONV_CASES)
def test_golden(name):
    require_gpu()
    wl, inputs, ref = load(name)
    s = Session(plan_for(wl))
    out = s.run(inputs)
    assert_bitexact(out["Y"], ref["Y"], name)


@pytest.mark.parametrize("name", QCONV_CASES)
def test_golden_generic_kernel(name):
    """The CUDA-core fallback kernels must match too (plan without tensor cores)."""
    require_gpu()
    wl, inputs, ref = load(name)
    s = Session(plan_for(wl, use_tensor_cores=False))
    assert_bitexact(s.run(inputs)["Y"], ref["Y"], name)


@pytest.mark.parametrize("kw", [
    dict(batch=3, channels=64, height=56, width=56),
    dict(batch=2, channels=64, height=56, width=56, wscale_range=(0.0001, 0.001)),
    dict(batch=2, channels=128, height=9, width=23, wscale_range=(0.00002, 0.0002)),
    dict(batch=5, channels=32, height=3, width=130, wscale_range=(0.0001, 0.001)),
    dict(batch=1, channels=64, height=1, width=1),
])
def test_vs_port(kw):
    require_gpu()
    wl = W.qconv_stack_int8(**kw)
    x = wl.make_inputs(7)
    ref = oracle.run_graph(wl.graph, x)["Y"]
    plan = plan_for(wl)
    assert any(op.kernel == 2 for op in plan.ops), "tensor-core conv path not selected"
    out = Session(plan).run(x)["Y"]
    assert_bitexact(out, ref, str(kw))
    sat = np.mean((ref == 0) | (ref == 255))
    assert sat < 1.0  # not a trivially saturated comparison


def test_batch_slices_and_device_pointers():
    require_gpu()
    import torch
    wl = W.qconv_stack_int8(batch=4, height=20, width=20, wscale_range=(0.0001, 0.001))
    x = wl.make_inputs(3)["X"]
    ref = oracle.run_graph(wl.graph, {"X": x})["Y"]
    s = Session(plan_for(wl))
    # host pointers, a slice of rows [1, 3)
    y = np.zeros_like(ref)
    s.run_ptrs([x.ctypes.data], [y.ctypes.data], batch_begin=1, batch_count=2)
    s.sync()
    assert_bitexact(y[1:3], ref[1:3], "slice")
    assert not y[0].any() and not y[3].any()
    # device pointers on a torch stream
    xd = torch.from_numpy(x).cuda()
    yd = torch.zeros(ref.shape, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream()
    s.run_ptrs([xd.data_ptr()], [yd.data_ptr()], stream=st.cuda_stream)
    s.sync()
    assert_bitexact(yd.cpu().numpy(), ref, "device pointers")
    # the layout kernel, then the four convolutions as one chain launch
    assert s.info().launches_per_run == sum(1 for op in s.plan.ops if op.ip.get(K.QC_CHAIN, 0) >= 0) == 2


def test_graph_replay_matches_direct_launches():
    """Graph replay (default) and one-by-one launches give the same bits; a
    run with new I/O addresses captures a new graph instead of reusing the old
    one."""
    require_gpu()
    import torch
    wl = W.qconv_stack_int8(batch=3, height=30, width=30, wscale_range=(0.0001, 0.001))
    s = Session(plan_for(wl))
    outs = []
    for seed in (1, 2):
        x = torch.from_numpy(wl.make_inputs(seed)["X"]).cuda()
        y = torch.zeros_like(x)
        s.run_ptrs([x.data_ptr()], [y.data_ptr()])
        s.sync()
        outs.append((x, y.cpu().numpy()))
    s.set_graphs(False)
    for x, y_graph in outs:
        y = torch.zeros_like(x)
        s.run_ptrs([x.data_ptr()], [y.data_ptr()])
        s.sync()
        assert_bitexact(y.cpu().numpy(), y_graph, "graph vs direct")
        ref = oracle.run_graph(wl.graph, {"X": x.cpu().numpy()})["Y"]
        assert_bitexact(y_graph, ref, "graph vs oracle")


def test_repeated_runs_are_identical():
    require_gpu()
    wl = W.qconv_stack_int8(batch=2, height=56, width=56)
    s = Session(plan_for(wl))
    x = wl.make_inputs(11)
    a = s.run(x)["Y"]
    for _ in range(3):
        assert_bitexact(s.run(x)["Y"], a, "rerun")


@pytest.mark.parametrize("kw", [
    dict(batch=4, channels=64, height=56, width=56, n_convs=5, wscale_range=(0.0001, 0.001)),
    dict(batch=3, channels=64, height=20, width=20, n_convs=2),
    dict(batch=2, channels=32, height=7, width=130, n_convs=3, wscale_range=(0.0001, 0.001)),
    dict(batch=1, channels=128, height=9, width=23, n_convs=4, wscale_range=(0.00002, 0.0002)),
    dict(batch=33, channels=64, height=8, width=8, n_convs=6, wscale_range=(0.0001, 0.001)),
    # more tiles than SMs: every CTA owns several tiles per layer (rounds), so
    # layers overlap across CTAs and the progress words order them
    dict(batch=16, channels=64, height=56, width=56, n_convs=4, wscale_range=(0.0001, 0.001)),
    dict(batch=12, channels=32, height=40, width=52, n_convs=5, wscale_range=(0.0001, 0.001)),
])
def test_chain_matches_separate_launches_and_port(kw):
    """A conv stack run as one persistent launch (layers ordered by per-tile
    progress words) gives the bytes of one launch per conv and of the CPU
    restatement, on every run (the progress words carry a run epoch)."""
    require_gpu()
    wl = W.qconv_stack_int8(**kw)
    x = wl.make_inputs(5)
    ref = oracle.run_graph(wl.graph, x)["Y"]
    chained = plan_for(wl)
    heads = [op for op in chained.ops if op.ip.get(K.QC_CHAIN, 0) > 1]
    assert len(heads) == 1 and heads[0].ip[K.QC_CHAIN] == kw["n_convs"], chained.describe()
    s = Session(chained)
    for run in range(3):
        assert_bitexact(s.run(x)["Y"], ref, f"chained run {run} {kw}")
    sep = plan_for(wl, chain_convs=False)
    assert not any(op.ip.get(K.QC_CHAIN, 0) for op in sep.ops)
    assert_bitexact(Session(sep).run(x)["Y"], ref, f"separate {kw}")
    # a second input through the same chained session: nothing of the first run leaks
    x2 = wl.make_inputs(6)
    assert_bitexact(s.run(x2)["Y"], oracle.run_graph(wl.graph, x2)["Y"], f"chained second input {kw}")

"""Pipelined host I/O: runs with page-locked host buffers split their rows
into slices whose uploads, kernels and downloads overlap on three streams.
Outputs must be byte-identical to the same plan run on device buffers, for
every slice count (including uneven slices), for row sub-ranges, for mixed
host/device pointers and for back-to-back calls with new inputs; pageable
host buffers take the unpipelined path with the same results."""
import numpy as np
import pytest

from emx_onnx_cgen_b200 import workloads as W
from emx_onnx_cgen_b200.plan import NP
from emx_onnx_cgen_b200.runtime import Session
from gpu_util import assert_bitexact, plan_for, require_gpu

pytestmark = pytest.mark.gpu

CASES = {
    # each moves more than 1 MiB across the bus per full run
    "qconv": lambda: W.qconv_stack_int8(batch=7, channels=64, height=56, width=56, wscale_range=(0.0001, 0.001)),
    "mlp": lambda: W.mlp_fp32(m=300, k=1024, hidden=512),
    "llama": lambda: W.llama_mlp_int4(m=600, hidden=512, inter=1024),
}
# overlapped runs also serve steps that move little: the full-size fp32 MLP (512 KB per run)
OVERLAP_CASES = {**CASES, "mlp_full": lambda: W.mlp_fp32()}


def _torch_dtype(torch, dt):
    return getattr(torch, np.dtype(NP[dt]).name)


def _buffers(torch, plan, inputs, pinned=True):
    hin = [torch.from_numpy(np.ascontiguousarray(inputs[n])) for n in plan.input_names]
    hout = [torch.zeros(tuple(s), dtype=_torch_dtype(torch, d)) for s, d in zip(plan.output_shapes, plan.output_dtypes)]
    if pinned:
        hin = [t.pin_memory() for t in hin]
        hout = [t.pin_memory() for t in hout]
    return hin, hout


def _device_reference(torch, s, plan, inputs):
    din = [torch.from_numpy(np.ascontiguousarray(inputs[n])).cuda() for n in plan.input_names]
    dout = [torch.zeros(tuple(sh), dtype=_torch_dtype(torch, d), device="cuda")
            for sh, d in zip(plan.output_shapes, plan.output_dtypes)]
    s.run_ptrs([t.data_ptr() for t in din], [t.data_ptr() for t in dout])
    s.sync()
    return [t.cpu().numpy() for t in dout]


@pytest.mark.parametrize("name", sorted(CASES))
@pytest.mark.parametrize("chunks", [1, 2, 3, 4, 8])
def test_pinned_host_matches_device(name, chunks):
    require_gpu()
    import torch
    wl = CASES[name]()
    plan = plan_for(wl)
    s = Session(plan)
    for seed in (1, 2):  # two calls in a row: staged rows of the first must not leak into the second
        inputs = wl.make_inputs(seed)
        ref = _device_reference(torch, s, plan, inputs)
        single = s.info().launches_per_run
        s.set_host_io_chunks(chunks)
        hin, hout = _buffers(torch, plan, inputs)
        s.run_ptrs([t.data_ptr() for t in hin], [t.data_ptr() for t in hout])
        s.sync()
        for got, exp, n in zip(hout, ref, plan.output_names):
            assert_bitexact(got.numpy(), exp, f"{name} chunks={chunks} seed={seed} {n}")
        batch = plan.batch
        expect_slices = 1 if chunks == 1 else len(range(0, batch, -(-batch // chunks)))
        assert s.info().launches_per_run == single * expect_slices
        s.set_host_io_chunks(4)


@pytest.mark.parametrize("name", sorted(CASES))
def test_row_ranges_and_mixed_pointers(name):
    require_gpu()
    import torch
    wl = CASES[name]()
    plan = plan_for(wl)
    s = Session(plan)
    inputs = wl.make_inputs(7)
    ref = _device_reference(torch, s, plan, inputs)
    batch = plan.batch
    b0, cnt = 1, batch - 2
    s.set_host_io_chunks(3)
    hin, hout = _buffers(torch, plan, inputs)
    s.run_ptrs([t.data_ptr() for t in hin], [t.data_ptr() for t in hout], batch_begin=b0, batch_count=cnt)
    s.sync()
    for got, exp, n in zip(hout, ref, plan.output_names):
        g = got.numpy()
        assert_bitexact(g[b0:b0 + cnt], exp[b0:b0 + cnt], f"{name} rows {n}")
        assert not g[:b0].any() and not g[b0 + cnt:].any(), "rows outside the range were written"
    # device inputs, page-locked host outputs
    din = [t.cuda() for t in hin]
    _, hout2 = _buffers(torch, plan, inputs)
    s.run_ptrs([t.data_ptr() for t in din], [t.data_ptr() for t in hout2])
    s.sync()
    for got, exp, n in zip(hout2, ref, plan.output_names):
        assert_bitexact(got.numpy(), exp, f"{name} mixed {n}")
    # pageable host buffers: unpipelined path
    hin3, hout3 = _buffers(torch, plan, inputs, pinned=False)
    s.run_ptrs([t.data_ptr() for t in hin3], [t.data_ptr() for t in hout3])
    s.sync()
    assert s.info().launches_per_run == _single_launches(s, plan, torch, inputs)
    for got, exp, n in zip(hout3, ref, plan.output_names):
        assert_bitexact(got.numpy(), exp, f"{name} pageable {n}")


def _single_launches(s, plan, torch, inputs):
    _device_reference(torch, s, plan, inputs)
    return s.info().launches_per_run


def test_chunk_count_is_validated():
    require_gpu()
    from emx_onnx_cgen_b200.runtime import EmxError
    s = Session(plan_for(CASES["mlp"]()))
    for bad in (0, 65, -1):
        with pytest.raises(EmxError):
            s.set_host_io_chunks(bad)


@pytest.mark.parametrize("name", sorted(OVERLAP_CASES))
def test_overlapped_runs(name):
    """Overlapped mode: five runs issued back to back on one stream, each with
    its own page-locked buffers and no synchronisation in between (uploads,
    kernels and downloads of neighbouring runs overlap through two staging
    sets); after join + sync every output equals its device-buffer run."""
    require_gpu()
    import torch
    wl = OVERLAP_CASES[name]()
    plan = plan_for(wl)
    s = Session(plan)
    inputs = [wl.make_inputs(20 + k) for k in range(5)]
    refs = [_device_reference(torch, s, plan, x) for x in inputs]
    s.set_host_io_overlap(True)
    st = torch.cuda.Stream()
    bufs = [_buffers(torch, plan, x) for x in inputs]
    for hin, hout in bufs:
        s.run_ptrs([t.data_ptr() for t in hin], [t.data_ptr() for t in hout], stream=st.cuda_stream)
    s.join(st.cuda_stream)
    st.synchronize()
    for k, ((_, hout), ref) in enumerate(zip(bufs, refs)):
        for got, exp, n in zip(hout, ref, plan.output_names):
            assert_bitexact(got.numpy(), exp, f"{name} overlapped run {k} {n}")
    s.sync()
    # a row range through the overlapped path, then back to the default mode
    b0, cnt = 1, plan.batch - 2
    hin, hout = _buffers(torch, plan, inputs[0])
    s.run_ptrs([t.data_ptr() for t in hin], [t.data_ptr() for t in hout], batch_begin=b0, batch_count=cnt)
    s.sync()
    for got, exp, n in zip(hout, refs[0], plan.output_names):
        assert_bitexact(got.numpy()[b0:b0 + cnt], exp[b0:b0 + cnt], f"{name} overlapped rows {n}")
    s.set_host_io_overlap(False)
    hin, hout = _buffers(torch, plan, inputs[1])
    s.run_ptrs([t.data_ptr() for t in hin], [t.data_ptr() for t in hout])
    s.sync()
    for got, exp, n in zip(hout, refs[1], plan.output_names):
        assert_bitexact(got.numpy(), exp, f"{name} after overlap {n}")

"""The benchmark's workload table, on CPU: every workload at every shard count
the scaling runs use (1, 2, 4, 8 GPUs) is a graph at batch/N whose
algorithmic work is 1/N of the full inference, and its plan launches the
kernel the roofline is computed for (the per-op times of that kernel are the
roofline's denominator, so a plan without it would divide by zero)."""
from __future__ import annotations

import functools

import pytest

import bench
from emx_onnx_cgen_b200 import kernel_ids as K
from emx_onnx_cgen_b200 import lowering
from emx_onnx_cgen_b200.plan import B200PlanEmitter

SHARDS = (1, 2, 4, 8)


@functools.lru_cache(maxsize=None)
def _spec(name, n):
    return bench.workload_spec(name, n)


def _shards(name):
    # the int4 MLP draws its full-size weights (seconds per draw): the full
    # inference and the smallest shard only
    return (1, 8) if name == "llama_mlp_int4" else SHARDS


@pytest.mark.parametrize("name", bench.ALL_WORKLOADS)
def test_shards_split_the_batch_and_the_work(name):
    wl1, dom1, _ = _spec(name, 1)
    for n in _shards(name):
        wl, dom, _ = _spec(name, n)
        assert dom["kernel"] == dom1["kernel"]
        assert dom["full_rows"] * n == dom1["full_rows"], (name, n)
        assert dom["ops_total"] * n == dom1["ops_total"], (name, n)
        # the graph's leading (batch) extent of every input shrinks by N
        for a, b in zip(wl.graph.inputs, wl1.graph.inputs):
            lead = 1 if name == "lstm_fp32" else 0  # LSTM X is [seq, batch, input]
            assert tuple(a.shape[:lead]) == tuple(b.shape[:lead])
            assert a.shape[lead] * n == b.shape[lead], (name, n, a.name)


@pytest.mark.parametrize("name", bench.ALL_WORKLOADS)
def test_shard_plans_launch_the_dominant_kernel(name):
    # the int4 MLP's full-size weight packing takes seconds: its smallest shard only
    shards = (8,) if name == "llama_mlp_int4" else (1, 8)
    kernels = None
    for n in shards:
        wl, dom, opts = _spec(name, n)
        plan = B200PlanEmitter(**opts).emit_plan(lowering.lower(wl.graph))
        names = [K.NAMES[op.kernel] for op in plan.ops]
        assert dom["kernel"] in names, (name, n, names)
        if kernels is not None:
            assert names == kernels, (name, n)
        kernels = names

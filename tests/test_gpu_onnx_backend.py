"""The onnx.backend-style adapter on the GPU: run_model / prepare + run give
the oracle's outputs (bit-exact for these cases) for inputs passed in graph
order or by name, and reject inputs of the wrong dtype or shape."""
import numpy as np
import pytest

from emx_onnx_cgen_b200 import onnx_backend as ob, workloads as W
from emx_onnx_cgen_b200.onnx_writer import write_onnx_bytes
from gpu_util import assert_bitexact, require_gpu
from oracle import oracle

pytestmark = pytest.mark.gpu

CASES = {
    "qconv_stack_int8": dict(batch=2, channels=64, height=10, width=12, n_convs=2),
    "mlp_fp32": dict(m=8, k=128, hidden=256),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_run_model_matches_oracle(name):
    require_gpu()
    wl = getattr(W, name)(**CASES[name])
    inputs = wl.make_inputs(11)
    ref = oracle.run_graph(wl.graph, inputs)
    outs = ob.run_model(write_onnx_bytes(wl.graph), [inputs[t.name] for t in wl.graph.inputs], device="CUDA:0")
    assert len(outs) == len(wl.graph.outputs)
    for t, got in zip(wl.graph.outputs, outs):
        assert_bitexact(got, ref[t.name], t.name)


def test_prepared_rep_reruns_and_checks_inputs():
    require_gpu()
    wl = W.qconv_stack_int8(**CASES["qconv_stack_int8"])
    rep = ob.prepare(write_onnx_bytes(wl.graph), "CUDA")
    try:
        for seed in (1, 2):
            inputs = wl.make_inputs(seed)
            ref = oracle.run_graph(wl.graph, inputs)
            (got,) = rep.run(inputs)  # by name
            assert_bitexact(got, ref[wl.graph.outputs[0].name])
        x = wl.make_inputs(3)[rep.input_names[0]]
        with pytest.raises(TypeError):
            rep.run([x.astype(np.int16)])
        with pytest.raises(ValueError):
            rep.run([x[:1]])
        with pytest.raises(ValueError):
            rep.run([])
    finally:
        rep.close()

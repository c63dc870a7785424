"""The CPU restatement (oracle/oracle.c) reproduces the reference's generated C
bit for bit on every golden fixture; the workload builders reproduce the
fixtures' weights."""
import numpy as np
import pytest

from golden_util import cases, load
from oracle import oracle


@pytest.mark.parametrize("name", sorted(cases()))
def test_port_matches_reference_c(name):
    wl, inputs, ref = load(name)
    runs = [(inputs, ref)]
    if hasattr(wl, "samples"):  # a whole model, several seeded input sets
        runs = [(wl.sample(inputs, i), wl.sample(ref, i)) for i in range(wl.samples)]
    for x, r in runs:
        got = oracle.run_graph(wl.graph, x)
        for k, v in r.items():
            assert got[k].dtype == v.dtype and got[k].shape == v.shape
            assert np.array_equal(got[k].view(np.uint8), v.view(np.uint8)), k


@pytest.mark.parametrize("name", sorted(n for n, m in cases().items() if "builder" in m))
def test_builders_reproduce_fixture_weights(name):
    from emx_onnx_cgen_b200 import workloads as W
    meta = cases()[name]
    kwargs = {k: tuple(v) if isinstance(v, list) else v for k, v in meta["kwargs"].items()}
    wl = W.BUILDERS[meta["builder"]](**kwargs)
    data = np.load(f"{__import__('golden_util').GOLDEN}/{name}.npz")
    for key in data.files:
        if key.startswith("init:"):
            assert np.array_equal(wl.graph.initializers[key[5:]], data[key]), key
        if key.startswith("in:"):
            assert np.array_equal(wl.make_inputs(meta["seed"])[key[3:]], data[key]), key

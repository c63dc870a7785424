"""Loading the golden fixtures made by tests/golden/make_golden.py."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from emx_onnx_cgen_b200 import workloads as W
from emx_onnx_cgen_b200.spec import GraphSpec, NodeSpec, TensorSpec

GOLDEN = Path(__file__).resolve().parent / "golden"


def cases() -> dict:
    return json.loads((GOLDEN / "cases.json").read_text())["cases"]


class ModelFixture:
    """A whole model stored with its fixture: ``graph`` rebuilt from the JSON
    topology and the stored initializers.  Its inputs and outputs carry a
    leading axis of ``samples`` seeded runs (``sample(arrays, i)`` picks one)."""

    def __init__(self, meta: dict, inits: dict):
        g = meta["graph"]
        ts = lambda rows: [TensorSpec(n, dt, tuple(shape)) for n, dt, shape in rows]
        self.name = g["name"]
        self.graph = GraphSpec(
            g["name"], ts(g["inputs"]), ts(g["outputs"]),
            [NodeSpec(op, nm, tuple(ins), tuple(outs), attrs, dom) for op, nm, ins, outs, attrs, dom in g["nodes"]],
            dict(inits), ts(g["values"]), tuple(tuple(o) for o in g["opset_imports"]))
        self.samples = int(meta["samples"])

    @staticmethod
    def sample(arrays: dict, i: int) -> dict:
        return {k: v[i] for k, v in arrays.items()}


def load(name: str):
    """(workload rebuilt from the recorded builder args, inputs, reference outputs).

    The stored initializers are written back into the rebuilt graph so the
    fixture stays self-contained even if a random generator's stream changed."""
    meta = cases()[name]
    if "graph" in meta:
        data = np.load(GOLDEN / f"{name}.npz")
        inits = {k[5:]: data[k] for k in data.files if k.startswith("init:")}
        inputs = {k[3:]: data[k] for k in data.files if k.startswith("in:")}
        outputs = {k[4:]: data[k] for k in data.files if k.startswith("out:")}
        return ModelFixture(meta, inits), inputs, outputs
    kwargs = {k: tuple(v) if isinstance(v, list) else v for k, v in meta["kwargs"].items()}
    wl = W.BUILDERS[meta["builder"]](**kwargs)
    data = np.load(GOLDEN / f"{name}.npz")
    for key in data.files:
        if key.startswith("init:"):
            wl.graph.initializers[key[5:]] = data[key]
    inputs = {k[3:]: data[k] for k in data.files if k.startswith("in:")}
    outputs = {k[4:]: data[k] for k in data.files if k.startswith("out:")}
    return wl, inputs, outputs

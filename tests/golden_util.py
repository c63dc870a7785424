"""Loading the golden fixtures made by tests/golden/make_golden.py."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from emx_onnx_cgen_b200 import workloads as W

GOLDEN = Path(__file__).resolve().parent / "golden"


def cases() -> dict:
    return json.loads((GOLDEN / "cases.json").read_text())["cases"]


def load(name: str):
    """(workload rebuilt from the recorded builder args, inputs, reference outputs).

    The stored initializers are written back into the rebuilt graph so the
    fixture stays self-contained even if a random generator's stream changed."""
    meta = cases()[name]
    kwargs = {k: tuple(v) if isinstance(v, list) else v for k, v in meta["kwargs"].items()}
    wl = W.BUILDERS[meta["builder"]](**kwargs)
    data = np.load(GOLDEN / f"{name}.npz")
    for key in data.files:
        if key.startswith("init:"):
            wl.graph.initializers[key[5:]] = data[key]
    inputs = {k[3:]: data[k] for k in data.files if k.startswith("in:")}
    outputs = {k[4:]: data[k] for k in data.files if k.startswith("out:")}
    return wl, inputs, outputs

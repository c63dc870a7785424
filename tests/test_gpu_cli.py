"""The command line on the GPU: ``verify`` accepts the CPU restatement's
outputs and rejects perturbed ones; ``compile`` + ``run`` from plan files
(and from a reference-format ``.bin``) give the outputs of a Session built
in memory."""
import dataclasses

import numpy as np
import pytest

from emx_onnx_cgen_b200 import cli, workloads as W
from emx_onnx_cgen_b200.lowering import lower
from emx_onnx_cgen_b200.onnx_writer import write_onnx
from emx_onnx_cgen_b200.refbin import partition_constants, weight_bin_bytes
from emx_onnx_cgen_b200.runtime import Session
from gpu_util import assert_bitexact, plan_for, require_gpu
from oracle import oracle

pytestmark = pytest.mark.gpu

CASES = {
    "qconv_stack_int8": dict(batch=2, channels=64, height=10, width=12, n_convs=2),
    "mlp_fp32": dict(m=8, k=128, hidden=256),
    "llama_mlp_int4": dict(m=16, hidden=256, inter=512),
}
# every case runs at the reference verify's default --max-ulp 100 (measured
# max ULP: 0 for all three at these sizes; the int4 MLP's full-size worst case
# is bounded per element in test_gpu_nbits.py)
MAX_ULP = {}


def _files(tmp_path, name, seed=3):
    wl = W.__dict__[name](**CASES[name])
    model = write_onnx(wl.graph, tmp_path / f"{name}.onnx")
    inputs = wl.make_inputs(seed)
    np.savez(tmp_path / "in.npz", **inputs)
    return wl, model, inputs


@pytest.mark.parametrize("name", sorted(CASES))
def test_verify_against_oracle(name, tmp_path, capsys):
    require_gpu()
    wl, model, inputs = _files(tmp_path, name)
    expected = oracle.run_graph(wl.graph, inputs)
    np.savez(tmp_path / "exp.npz", **expected)
    tol = ["--max-ulp", str(MAX_ULP.get(name, 100))]
    rc = cli.main(["verify", str(model), "--inputs", str(tmp_path / "in.npz"), "--expected",
                   str(tmp_path / "exp.npz"), *tol])
    out = capsys.readouterr().out
    with capsys.disabled():
        print(f"\n{name}: verify {out.strip()} (tolerance --max-ulp {tol[1]})")
    assert rc == 0 and out.startswith("OK (max ULP"), out
    # perturb one element of the first output far beyond any tolerance
    name0 = wl.graph.outputs[0].name
    bad = dict(expected)
    arr = bad[name0].copy().reshape(-1)
    arr[arr.size // 2] = (arr[arr.size // 2] + 100) if arr.dtype.kind in "ui" else arr[arr.size // 2] * 3 + 1
    bad[name0] = arr.astype(expected[name0].dtype).reshape(expected[name0].shape)
    np.savez(tmp_path / "bad.npz", **bad)
    assert cli.main(["verify", str(model), "--inputs", str(tmp_path / "in.npz"), "--expected",
                     str(tmp_path / "bad.npz"), *tol]) == 1


@pytest.mark.parametrize("name", sorted(CASES))
def test_compile_run_from_files(name, tmp_path):
    require_gpu()
    wl, model, inputs = _files(tmp_path, name, seed=5)
    ref = Session(plan_for(wl)).run(inputs)
    assert cli.main(["compile", str(model), "-o", str(tmp_path / "plan")]) == 0
    prefix = tmp_path / "plan" / wl.graph.name
    assert cli.main(["run", str(prefix), "--inputs", str(tmp_path / "in.npz"), "--outputs",
                     str(tmp_path / "out.npz")]) == 0
    with np.load(tmp_path / "out.npz") as z:
        for k, v in ref.items():
            assert_bitexact(z[k], v, k)
    # the same model with its large initializers taken from a reference-format .bin
    names = {c.name for c in partition_constants(lower(wl.graph).constants, 1024)[1]}
    (tmp_path / "m.bin").write_bytes(weight_bin_bytes(lower(wl.graph).constants, 1024))
    g0 = wl.graph
    gz = dataclasses.replace(g0, initializers={k: (np.zeros_like(v) if k in names else v)
                                               for k, v in g0.initializers.items()})
    write_onnx(gz, tmp_path / "z.onnx")
    assert cli.main(["run", str(tmp_path / "z.onnx"), "--weights-bin", str(tmp_path / "m.bin"),
                     "--large-weight-threshold", "1024", "--inputs", str(tmp_path / "in.npz"), "--outputs",
                     str(tmp_path / "out2.npz")]) == 0
    with np.load(tmp_path / "out2.npz") as z:
        for k, v in ref.items():
            assert_bitexact(z[k], v, k)

"""The QOperator layout and pooling kernels (Reshape, Transpose, MaxPool,
QLinearAveragePool, QLinearSoftmax) and the reference's own QOperator model,
micro_kws_m_static_qoperator.onnx, end to end on the B200 kernels.

Bar: bit-exact against the reference's generated C (golden fixtures) and the
CPU restatement, for every op and for the model's float output."""
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from emx_onnx_cgen_b200 import kernel_ids as K, workloads as W
from emx_onnx_cgen_b200.onnx_writer import write_onnx
from emx_onnx_cgen_b200.runtime import Session
from golden_util import cases, load
from gpu_util import assert_bitexact, plan_for, require_gpu
from oracle import oracle

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
OPS = ("maxpool", "qavgpool", "qsoftmax", "transpose")


@pytest.mark.parametrize("name", sorted(n for n in cases() if n.startswith(OPS)))
def test_golden(name):
    require_gpu()
    wl, inputs, ref = load(name)
    out = Session(plan_for(wl)).run(inputs)
    for k, v in ref.items():
        assert_bitexact(out[k], v, f"{name}:{k}")


@pytest.mark.parametrize("wl", [
    W.pool8(shape=(8, 64, 56, 56), kernel=(3, 3), strides=(2, 2), pads=(1, 1, 1, 1)),
    W.pool8(shape=(3, 16, 31, 29), kernel=(5, 3), strides=(2, 3), dilations=(2, 1), ceil_mode=1, dtype="u8"),
    W.pool8(shape=(8, 64, 56, 56), kind="avg", kernel=(3, 3), strides=(2, 2), pads=(1, 1, 1, 1)),
    W.pool8(shape=(4, 32, 17, 23), kind="avg", kernel=(4, 4), strides=(3, 3), pads=(2, 2, 2, 2),
            count_include_pad=1, dtype="u8", x_zero=128, y_dtype="i8", y_zero=-4, x_scale=0.01, y_scale=0.03),
    W.qlinear_softmax8(shape=(1000, 1000)),
    W.qlinear_softmax8(shape=(64, 9, 130), axis=1, dtype="i8", x_zero=3, x_scale=0.5, y_zero=-128),
    W.qlinear_softmax8(shape=(5, 7, 11), axis=1, opset=11),
    W.transpose(shape=(16, 64, 28, 28), perm=(0, 2, 3, 1), dtype="u8"),
    W.transpose(shape=(9, 33, 65), perm=(2, 0, 1), dtype="f16"),
    W.transpose(shape=(2, 3, 4, 5, 6, 7), perm=(5, 3, 1, 0, 2, 4), dtype="f32"),
], ids=lambda w: w.name + str(sorted(w.params.items()))[:70])
def test_vs_port(wl):
    require_gpu()
    x = wl.make_inputs(4)
    ref = oracle.run_graph(wl.graph, x)
    out = Session(plan_for(wl)).run(x)
    for k, v in ref.items():
        assert_bitexact(out[k], v, k)


@pytest.mark.parametrize("wl", [
    W.pool8(shape=(6, 8, 13, 11)),
    W.pool8(shape=(6, 8, 13, 11), kind="avg"),
    W.qlinear_softmax8(shape=(6, 37)),
    W.transpose(shape=(6, 3, 4, 5), perm=(0, 2, 3, 1)),
], ids=lambda w: w.name)
def test_batch_slices(wl):
    """Rows 2..4 of a batch-6 plan: the kernels take the run's batch."""
    require_gpu()
    x = wl.make_inputs(2)["X"]
    ref = oracle.run_graph(wl.graph, {"X": x})["Y"]
    plan = plan_for(wl)
    assert plan.batch == 6
    s = Session(plan)
    y = np.zeros_like(ref)
    s.run_ptrs([x.ctypes.data], [y.ctypes.data], batch_begin=2, batch_count=3)
    s.sync()
    assert_bitexact(y[2:5], ref[2:5], "rows 2..4")
    assert not y[:2].any() and not y[5:].any()


def test_kws_model_all_samples():
    """Every stored input set of micro_kws_m_static_qoperator.onnx: the B200
    output equals the reference's generated C bit for bit."""
    require_gpu()
    fx, inputs, ref = load("kws_qoperator")
    plan = plan_for(fx)
    assert K.K_QLINEAR_SOFTMAX in [o.kernel for o in plan.ops]
    sess = Session(plan)
    for i in range(fx.samples):
        out = sess.run(fx.sample(inputs, i))
        for k, v in fx.sample(ref, i).items():
            assert_bitexact(out[k], v, f"sample {i}:{k}")


def test_kws_model_cli_verify(tmp_path):
    """python -m emx_onnx_cgen_b200 verify on the model (written back to ONNX
    from the fixture), bit-exact (--max-ulp 0 --atol-eps 0); a changed expected
    value is rejected."""
    require_gpu()
    fx, inputs, ref = load("kws_qoperator")
    model = write_onnx(fx.graph, tmp_path / "micro_kws_m_static_qoperator.onnx")
    np.savez(tmp_path / "in.npz", **fx.sample(inputs, 2))
    exp = fx.sample(ref, 2)
    np.savez(tmp_path / "exp.npz", **exp)
    cmd = [sys.executable, "-m", "emx_onnx_cgen_b200", "verify", str(model), "--inputs", str(tmp_path / "in.npz"),
           "--expected", str(tmp_path / "exp.npz"), "--max-ulp", "0", "--atol-eps", "0"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    print(r.stdout, r.stderr)
    assert r.returncode == 0 and r.stdout.startswith("OK (max ULP 0)"), r.stdout + r.stderr
    bad = {k: v.copy() for k, v in exp.items()}
    k0 = next(iter(bad))
    bad[k0].reshape(-1)[int(np.argmax(bad[k0]))] *= 0.5
    np.savez(tmp_path / "bad.npz", **bad)
    cmd[cmd.index(str(tmp_path / "exp.npz"))] = str(tmp_path / "bad.npz")
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 1, r.stdout + r.stderr

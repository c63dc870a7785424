"""Command line, plan files, ONNX export and the reference's weight file (CPU).

* the ONNX writer round-trips every built-in workload through the reader;
* ``compile`` writes plan files that load back to the same plan bytes the
  in-memory emitter produces, with ``--input-dim`` in both of the
  reference's forms;
* ``weight_bin_bytes`` writes byte for byte the ``<model>.bin`` the
  reference's C emitter writes (c_emitter.py:4230-4268, :4398-4407) at
  several thresholds, and a plan built from that file equals the plan built
  from the initializers;
* the verify metric equals the reference's ``worst_ulp_diff``
  (verification.py:25-60) on random, signed-zero and NaN data.
"""
import dataclasses
from pathlib import Path

import numpy as np
import pytest

from emx_onnx_cgen_b200 import cli, lowering, workloads as W
from emx_onnx_cgen_b200.onnx_reader import infer_types, read_onnx, read_onnx_bytes
from emx_onnx_cgen_b200.onnx_writer import write_onnx, write_onnx_bytes
from emx_onnx_cgen_b200.plan import B200PlanEmitter, load_plan
from emx_onnx_cgen_b200.refbin import constants_from_bin, partition_constants, weight_bin_bytes
from emx_onnx_cgen_b200.verify import check_output, ulp_distance
from oracle import refc

SMALL = {
    "qconv_stack_int8": dict(batch=2, channels=32, height=8, width=8),
    "llama_mlp_int4": dict(m=4, hidden=128, inter=256),
    "mlp_fp32": dict(m=4, k=64, hidden=256),
    "lstm_fp32": dict(seq=3, batch=2, input_size=16, hidden=32),
    "attention_fp16": dict(batch=1, heads=2, seq=16, head_dim=16),
    "matmul_nbits_f16": dict(zero_points="block", bias=True),
    "swish_mul_f16": {}, "qlinear_matmul_u8": {}, "matmul_integer_u8": {}, "conv_f32": {},
    "softmax_f32": {}, "quant_dequant": {},
}


def _wl(name):
    return W.__dict__[name](**SMALL[name])


def _same_attr(a, b):
    if isinstance(a, float):
        return np.float32(a) == np.float32(b)
    if isinstance(a, np.ndarray):
        return np.array_equal(a, b)
    if isinstance(a, (list, tuple)):
        return list(a) == list(b)
    return a == b


@pytest.mark.parametrize("name", sorted(SMALL))
def test_writer_round_trip(name):
    g = _wl(name).graph
    g2 = read_onnx_bytes(write_onnx_bytes(g))
    assert (g2.name, g2.inputs, g2.outputs, g2.values, g2.opset_imports) == \
        (g.name, g.inputs, g.outputs, g.values, g.opset_imports)
    assert [(n.op_type, n.name, n.inputs, n.outputs, n.domain) for n in g2.nodes] == \
        [(n.op_type, n.name, n.inputs, n.outputs, n.domain) for n in g.nodes]
    for n1, n2 in zip(g.nodes, g2.nodes):
        assert set(n1.attrs) == set(n2.attrs)
        assert all(_same_attr(v, n2.attrs[k]) for k, v in n1.attrs.items()), n1.name
    for k, v in g.initializers.items():
        assert g2.initializers[k].dtype == v.dtype and np.array_equal(g2.initializers[k], v), k


@pytest.mark.parametrize("name", ["qconv_stack_int8", "mlp_fp32", "llama_mlp_int4", "lstm_fp32"])
def test_compile_writes_loadable_plan(name, tmp_path):
    wl = _wl(name)
    model = tmp_path / f"{name}.onnx"
    write_onnx(wl.graph, model)
    assert cli.main(["compile", str(model), "-o", str(tmp_path / "out")]) == 0
    plan, wpath = load_plan(tmp_path / "out" / wl.graph.name)
    ref = B200PlanEmitter().emit_plan(lowering.lower(wl.graph))
    assert plan.plan_bytes == ref.plan_bytes
    assert Path(wpath).read_bytes() == ref.weight_bytes
    assert (plan.input_names, plan.input_shapes, plan.input_dtypes) == (ref.input_names, ref.input_shapes,
                                                                        ref.input_dtypes)
    assert (plan.output_names, plan.output_shapes, plan.output_dtypes, plan.batch, plan.arena_bytes) == \
        (ref.output_names, ref.output_shapes, ref.output_dtypes, ref.batch, ref.arena_bytes)


def test_input_dim_forms(tmp_path):
    """A symbolic batch pinned by name or by input position gives the plan of
    the static model; unbound it is an error (exit 2)."""
    wl = W.qconv_stack_int8(batch=3, channels=32, height=8, width=8)
    g = wl.graph
    dp = {t.name: {0: "N"} for t in (*g.inputs, *g.outputs, *g.values)}
    model = tmp_path / "sym.onnx"
    write_onnx(g, model, dim_params=dp)
    ref = B200PlanEmitter().emit_plan(lowering.lower(g)).plan_bytes
    by_name = cli.compile_model(model, cli.parse_input_dims(["N=3"]))
    by_pos = cli.compile_model(model, cli.parse_input_dims([f"{g.inputs[0].name}:0=3"]))
    assert by_name.plan_bytes == ref and by_pos.plan_bytes == ref
    assert cli.main(["compile", str(model), "-o", str(tmp_path)]) == 2
    assert cli.main(["compile", str(model), "--input-dim", "N=0"]) == 2


def test_unsupported_model_is_a_usage_error(tmp_path):
    wl = W.softmax_f32()
    g = dataclasses.replace(wl.graph, nodes=[dataclasses.replace(n, op_type="Hardmax") for n in wl.graph.nodes])
    model = tmp_path / "bad.onnx"
    write_onnx(g, model)
    assert cli.main(["compile", str(model), "-o", str(tmp_path)]) == 2


def test_export_command(tmp_path):
    out = tmp_path / "m.onnx"
    ins = tmp_path / "in.npz"
    assert cli.main(["export", "mlp_fp32", str(out), "--param", "m=4", "--param", "k=64", "--param", "hidden=128",
                     "--inputs-out", str(ins), "--seed", "5"]) == 0
    spec = infer_types(read_onnx(out))
    wl = W.mlp_fp32(m=4, k=64, hidden=128)
    assert spec.inputs == wl.graph.inputs
    with np.load(ins) as z:
        np.testing.assert_array_equal(z["X"], wl.make_inputs(5)["X"])
    assert cli.main(["export", "matmul_nbits_f16", str(out), "--param", "zero_points='u8'"]) == 2


# ------------------------------------------------------------------ the reference's weight file
def test_partition_rule_synthetic():
    """Smallest first, ties in constant order, while the inline total fits."""
    C = lowering.ConstTensor
    f32 = lowering.ScalarType.F32
    consts = [C(f"c{i}", (n,), np.zeros(n, np.float32), f32) for i, n in enumerate([100, 10, 30, 10, 5])]
    inline, large = partition_constants(consts, threshold=4 * 55)
    assert [c.name for c in inline] == ["c1", "c2", "c3", "c4"] and [c.name for c in large] == ["c0"]
    inline, large = partition_constants(consts, threshold=4 * 24)  # c4 + c1 fit, c3 (tied with c1) does not
    assert [c.name for c in inline] == ["c1", "c4"] and [c.name for c in large] == ["c0", "c2", "c3"]
    inline, large = partition_constants(consts, threshold=0)
    assert len(inline) == 5 and not large


@pytest.mark.skipif(not refc.reference_available(), reason="reference compiler source not present")
@pytest.mark.parametrize("name", ["qconv_stack_int8", "mlp_fp32", "llama_mlp_int4", "lstm_fp32",
                                  "matmul_nbits_f16", "qlinear_matmul_u8", "conv_f32"])
@pytest.mark.parametrize("threshold", [64, 1024, 100 * 1024])
def test_weight_bin_matches_reference_emitter(name, threshold, tmp_path):
    g = _wl(name).graph
    _, bin_path = refc.emit_c(g, tmp_path, "m", large_weight_threshold=threshold)
    ref = bin_path.read_bytes() if bin_path else b""
    assert weight_bin_bytes(lowering.lower(g).constants, threshold) == ref


@pytest.mark.parametrize("name", ["qconv_stack_int8", "mlp_fp32", "llama_mlp_int4", "lstm_fp32"])
def test_plan_from_weight_bin(name, tmp_path):
    """Large constants blanked in the model and read back from the .bin give
    the plan of the original model; the CLI does the same with --weights-bin."""
    g = _wl(name).graph
    model = lowering.lower(g)
    data = weight_bin_bytes(model.constants, 1024)
    _, large = partition_constants(model.constants, 1024)
    assert large, "the case must have constants above the threshold"
    names = {c.name for c in large}
    blank = dataclasses.replace(model, constants=tuple(
        dataclasses.replace(c, data=np.zeros_like(c.data)) if c.name in names else c for c in model.constants))
    ref = B200PlanEmitter().emit_plan(model)
    got = B200PlanEmitter().emit_plan(constants_from_bin(blank, data, 1024))
    assert (got.plan_bytes, got.weight_bytes) == (ref.plan_bytes, ref.weight_bytes)
    with pytest.raises(ValueError):
        constants_from_bin(blank, data[:-1], 1024)
    # through the CLI: a model file whose large initializers are zero + the .bin
    gz = dataclasses.replace(g, initializers={k: (np.zeros_like(v) if k in names else v)
                                              for k, v in g.initializers.items()})
    write_onnx(gz, tmp_path / "z.onnx")
    (tmp_path / "z.bin").write_bytes(data)
    assert cli.main(["compile", str(tmp_path / "z.onnx"), "-o", str(tmp_path / "out"), "--weights-bin",
                     str(tmp_path / "z.bin"), "--large-weight-threshold", "1024"]) == 0
    plan, wpath = load_plan(tmp_path / "out" / g.name)
    assert plan.plan_bytes == ref.plan_bytes and Path(wpath).read_bytes() == ref.weight_bytes
    # a file written for another threshold (here: none, everything inline) is refused
    assert cli.main(["compile", str(tmp_path / "z.onnx"), "--weights-bin", str(tmp_path / "z.bin"),
                     "--large-weight-threshold", "0"]) == 2


# ------------------------------------------------------------------ verify metric
def _cases():
    rng = np.random.default_rng(3)
    for dt in (np.float16, np.float32, np.float64):
        b = rng.standard_normal(400).astype(dt)
        a = (b + rng.standard_normal(400) * np.finfo(dt).eps * rng.choice([0.1, 3, 300], 400)).astype(dt)
        a[:5] = [-0.0, 0.0, np.nan, 1.0, -b[4]]
        b[:5] = [0.0, -0.0, np.nan, np.nan, b[4]]
        yield a, b


@pytest.mark.skipif(not refc.reference_available(), reason="reference source not present")
@pytest.mark.parametrize("atol_eps", [0.0, 1.0, 8.0])
def test_ulp_metric_matches_reference(atol_eps):
    refc._import_reference()
    from emx_onnx_cgen.verification import worst_ulp_diff
    for a, b in _cases():
        ref_max, _ = worst_ulp_diff(a, b, atol_eps=atol_eps)
        assert int(ulp_distance(a, b, atol_eps).max()) == ref_max, a.dtype
        c = check_output("y", a, b, max_ulp=ref_max, atol_eps=atol_eps)
        assert c.ok and c.max_ulp == ref_max
        if ref_max:
            assert not check_output("y", a, b, max_ulp=ref_max - 1, atol_eps=atol_eps).ok


def test_integer_outputs_compare_exactly():
    a = np.arange(10, dtype=np.uint8)
    assert check_output("y", a, a.copy()).ok
    b = a.copy()
    b[7] = 0
    c = check_output("y", a, b)
    assert not c.ok and c.mismatches == 1 and c.worst[0] == (7,)


def test_target_flag(tmp_path, capsys):
    """``compile --target b200`` is the B200 emit target; other targets are the reference CLI's."""
    wl = W.mlp_fp32(m=4, k=64, hidden=128)
    model = write_onnx(wl.graph, tmp_path / "m.onnx")
    assert cli.main(["compile", str(model), "--target", "b200", "-o", str(tmp_path / "out")]) == 0
    assert (tmp_path / "out" / f"{wl.graph.name}.plan").exists()
    with pytest.raises(SystemExit):
        cli.main(["compile", str(model), "--target", "c"])

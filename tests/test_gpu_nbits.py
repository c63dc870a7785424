"""com.microsoft MatMulNBits (int4 weights x fp16 activations, tcgen05) and
the fp16 Swish / Mul kernels, against the reference's generated C (golden
fixtures) and the CPU restatement.

Tolerances.  The MatMulNBits kernel multiplies exact dequantised weights
(hi + lo fp16 split) in the tensor cores' fp32 accumulators, while the
reference sums (float)a * deq sequentially in float; only the summation order
differs.  One MatMulNBits output therefore agrees within a stated fp16 ULP
bound, measured with the reference's own metric (shared/ulp.py:26-50, pairs
closer than 1 fp16 eps skipped; the defaults of the reference's verify,
--max-ulp 100, --atol-eps 1):
  * NBITS_MAX_ULP = 100 for every output element,
  * and at least NBITS_FRAC_WITHIN_2 of the elements within 2 ULP.
Through the whole MLP the intermediate P = Swish(G) * U is rounded to fp16 on
both sides; where the two sums straddle an fp16 rounding boundary of G, U or
P, P differs by one fp16 ULP and the down projection carries that difference
into Y.  The MLP output is checked against that propagation bound, element
by element: |Y - Y_ref| <= sum_k ulp(P_ref[m,k]) * |deq_down[n,k]|
+ 2^-20 * sum_k |P_ref[m,k] * deq_down[n,k]| + ulp(Y_ref[m,n]).
Swish and Mul are bit-exact (double exp / division and one rounding to fp16,
as the reference evaluates them; the Swish check covers all 65536 fp16 inputs).
"""
import numpy as np
import pytest

from emx_onnx_cgen_b200 import workloads as W
from emx_onnx_cgen_b200.runtime import Session
from emx_onnx_cgen_b200.spec import GraphSpec, NodeSpec, TensorSpec
from golden_util import cases, load
from gpu_util import assert_bitexact, plan_for, require_gpu, ulp_diff_f16
from oracle import oracle

pytestmark = pytest.mark.gpu

NBITS_MAX_ULP = 100
NBITS_FRAC_WITHIN_2 = 0.99


def _check_ulp(got, ref, what):
    d = ulp_diff_f16(got, ref)
    frac2 = float(np.mean(d <= 2)) if d.size else 1.0
    assert int(d.max(initial=0)) <= NBITS_MAX_ULP, f"{what}: max ULP {int(d.max())}"
    assert frac2 >= NBITS_FRAC_WITHIN_2, f"{what}: only {frac2:.4f} of elements within 2 ULP"
    return int(d.max(initial=0)), frac2


def _dequant_f64(graph, prefix):
    """Reference dequantised weights [N][K] (float64) of MatMulNBits `prefix`."""
    from emx_onnx_cgen_b200.plan import unpack_nbits
    node = next(n for n in graph.nodes if n.name == prefix)
    k, n, bs = int(node.attrs["K"]), int(node.attrs["N"]), int(node.attrs["block_size"])
    q = unpack_nbits(graph.initializers[node.inputs[1]], n, bs)[:, :k].astype(np.float64)
    sc = graph.initializers[node.inputs[2]].astype(np.float64).reshape(n, -1)
    blk = np.arange(k) // bs
    return (q - 8.0) * sc[:, blk]


def _check_mlp(wl, a_rows, y_rows, what):
    """Propagation bound of the docstring for llama_mlp_int4 outputs."""
    g = wl.graph
    gate = oracle.run_graph(_single(g, "gate", "A", "G", len(a_rows)), {"A": a_rows})["G"]
    up = oracle.run_graph(_single(g, "up", "A", "U", len(a_rows)), {"A": a_rows})["U"]
    p_ref = oracle.mul_f16(oracle.swish_f16(gate, 1.0), up)
    y_ref = oracle.matmul_nbits_f16(p_ref, g.initializers["down_B"], g.initializers["down_s"],
                                    p_ref.shape[1], y_rows.shape[1], int(wl.params["block"]))
    deq = np.abs(_dequant_f64(g, "down"))
    pf = p_ref.astype(np.float64)
    bound = (np.spacing(np.abs(p_ref)).astype(np.float64) @ deq.T + 2.0 ** -20 * (np.abs(pf) @ deq.T)
             + np.spacing(np.abs(y_ref)).astype(np.float64))
    err = np.abs(y_rows.astype(np.float64) - y_ref.astype(np.float64))
    worst = float(np.max(err / bound))
    assert worst <= 1.0, f"{what}: error reaches {worst:.3f} x the propagation bound"
    return int(ulp_diff_f16(y_rows, y_ref).max(initial=0)), worst


def _single(g, node_name, a, out, rows):
    node = next(n for n in g.nodes if n.name == node_name)
    k, n = int(node.attrs["K"]), int(node.attrs["N"])
    return GraphSpec(node_name, [TensorSpec(a, "f16", (rows, k))], [TensorSpec(out, "f16", (rows, n))],
                     [NodeSpec("MatMulNBits", node.name, (a, *node.inputs[1:]), (out,), node.attrs, node.domain)],
                     {k2: v for k2, v in g.initializers.items() if k2 in node.inputs}, opset_imports=g.opset_imports)


@pytest.mark.parametrize("name", sorted(n for n in cases() if n.startswith("nbits")))
def test_golden(name):
    require_gpu()
    wl, inputs, ref = load(name)
    out = Session(plan_for(wl)).run(inputs)
    for k, v in ref.items():
        _check_ulp(out[k], v, f"{name}:{k}")


@pytest.mark.parametrize("name", sorted(n for n in cases() if n.startswith("swishmul")))
def test_golden_swish_mul_bitexact(name):
    require_gpu()
    wl, inputs, ref = load(name)
    out = Session(plan_for(wl)).run(inputs)
    for k, v in ref.items():
        assert_bitexact(out[k], v, k)


def test_swish_all_fp16_values():
    require_gpu()
    x = np.arange(65536, dtype=np.uint16).view(np.float16)
    g = GraphSpec("swish_all", [TensorSpec("X", "f16", (65536,))], [TensorSpec("Y", "f16", (65536,))],
                  [NodeSpec("Swish", "s", ("X",), ("Y",), {"alpha": 1.0})], {}, opset_imports=(("", 24),))
    wl = W.Workload("swish_all", g, lambda seed=0: {"X": x}, {"X": 0, "Y": 0}, {})
    ref = oracle.run_graph(g, {"X": x})["Y"]
    out = Session(plan_for(wl)).run({"X": x})["Y"]
    assert_bitexact(out, ref, "swish over all fp16")


# (123, 77): the one-value-per-thread Mul; (64, 96): eight fp16 values per thread
@pytest.mark.parametrize("alpha,shape", [(1.0, (123, 77)), (0.5, (123, 77)), (1.702, (123, 77)), (1.0, (64, 96))])
def test_swish_mul_vs_port(alpha, shape):
    require_gpu()
    wl = W.swish_mul_f16(shape, alpha)
    x = wl.make_inputs(3)
    x["Z"][0, :5] = [np.inf, -np.inf, np.nan, -0.0, 65504]
    ref = oracle.run_graph(wl.graph, x)
    out = Session(plan_for(wl)).run(x)
    for k in ("S", "P"):
        assert_bitexact(out[k], ref[k], k)


@pytest.mark.parametrize("kw", [
    dict(m=64, k=256, n=192),
    dict(m=300, k=512, n=136, zero_points="block", bias=True),
    dict(m=257, k=200, n=40, block=16, zero_points="column"),
    dict(m=1, k=64, n=8, block=64),
    dict(m=33, k=1024, n=264, block=128, bias=True),
])
def test_single_vs_port(kw):
    require_gpu()
    wl = W.matmul_nbits_f16(**kw)
    x = wl.make_inputs(4)
    ref = oracle.run_graph(wl.graph, x)["Y"]
    out = Session(plan_for(wl)).run(x)["Y"]
    _check_ulp(out, ref, str(kw))


@pytest.mark.parametrize("kw", [dict(m=300, hidden=512, inter=704), dict(m=513, hidden=256, inter=200)])
def test_fused_mlp_vs_port(kw):
    require_gpu()
    wl = W.llama_mlp_int4(**kw)
    plan = plan_for(wl)
    assert any("fused" in op.label for op in plan.ops)
    x = wl.make_inputs(6)
    out = Session(plan).run(x)["Y"]
    _check_mlp(wl, x["A"], out, str(kw))


def test_full_size_rows():
    """The 2048 x 4096 -> 11008 -> 4096 workload; the CPU restatement (bit-
    identical to the reference's generated C) checks 64 rows spread over the
    batch (rows are independent: Y[m] depends on A[m] only)."""
    require_gpu()
    wl = W.llama_mlp_int4()
    x = wl.make_inputs(0)
    out = Session(plan_for(wl)).run(x)["Y"]
    rows = np.unique(np.concatenate([[0, 1, 2047], np.linspace(2, 2046, 61).astype(int)]))
    assert rows.size >= 64
    worst_ulp, worst_bound = _check_mlp(wl, x["A"][rows], out[rows], "full-size sample rows")
    print(f"llama MLP, {rows.size} full-size rows: worst ULP of Y {worst_ulp}, "
          f"worst error / propagation bound {worst_bound:.3f}")
    assert np.all(np.isfinite(out))


def test_row_slices():
    require_gpu()
    wl = W.llama_mlp_int4(m=40, hidden=128, inter=192)
    x = wl.make_inputs(9)["A"]
    full = Session(plan_for(wl)).run({"A": x})["Y"]
    s = Session(plan_for(wl))
    y = np.zeros_like(full)
    s.run_ptrs([x.ctypes.data], [y.ctypes.data], batch_begin=7, batch_count=20)
    s.sync()
    assert_bitexact(y[7:27], full[7:27], "rows 7..26 of a slice run vs the full run")

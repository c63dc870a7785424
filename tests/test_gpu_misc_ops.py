"""QLinearMatMul, MatMulInteger, fp32 Conv, fp32 Softmax and
Quantize/DequantizeLinear on the B200 kernels, against the reference's
generated C (golden fixtures) and the CPU restatement.

Bars: bit-exact for every op except Softmax, whose reference calls glibc's
expf (CUDA's differs by at most 2 ulp, glibc's by up to 0.502 ulp from the
exact value); Softmax outputs must agree within SOFTMAX_MAX_ULP fp32 ULP
(reference metric, shared/ulp.py:26-50, atol 1 eps)."""
import numpy as np
import pytest

from emx_onnx_cgen_b200 import workloads as W
from emx_onnx_cgen_b200.runtime import Session
from emx_onnx_cgen_b200.spec import GraphSpec, NodeSpec, TensorSpec
from golden_util import cases, load
from gpu_util import assert_bitexact, plan_for, require_gpu, ulp_diff_f32
from oracle import oracle

pytestmark = pytest.mark.gpu

SOFTMAX_MAX_ULP = 8
EXACT = ("qmm", "mmi", "conv", "qdq")


@pytest.mark.parametrize("name", sorted(n for n in cases() if n.startswith(EXACT + ("softmax",))))
def test_golden(name):
    require_gpu()
    wl, inputs, ref = load(name)
    out = Session(plan_for(wl)).run(inputs)
    for k, v in ref.items():
        if name.startswith("softmax"):
            assert int(ulp_diff_f32(out[k], v).max(initial=0)) <= SOFTMAX_MAX_ULP, name
        else:
            assert_bitexact(out[k], v, f"{name}:{k}")


@pytest.mark.parametrize("wl", [
    W.qlinear_matmul_u8(m=300, k=513, n=130),
    W.qlinear_matmul_u8(m=7, k=64, n=33, a_zero=3, b_dtype="u8", b_zero=200, scales=(0.25, 0.125, 0.5)),
    W.matmul_integer_u8(m=129, k=1000, n=65, a_zero=0, b_zero=-5),
    W.conv_f32(batch=3, cin=16, cout=24, h=20, w=17, kernel=3, stride=2, pad=1),
    W.conv_f32(batch=1, cin=6, cout=6, h=11, w=11, kernel=5, pad=4, dilation=2, group=3),
    W.quant_dequant((33, 70), out_dtype="i8", zero=5, scale=0.01),
], ids=lambda w: w.name + str(sorted(w.params.items()))[:60])
def test_exact_vs_port(wl):
    require_gpu()
    x = wl.make_inputs(4)
    ref = oracle.run_graph(wl.graph, x)
    out = Session(plan_for(wl)).run(x)
    for k, v in ref.items():
        assert_bitexact(out[k], v, k)


# K a multiple of 16 (<= 32768): tcgen05 kind::i8 with the zero points restored in the epilogue.
# Partial row / column tiles, each zero-point combination (row sums, column sums, both, none),
# both requantisations, scalar and vector stores, signed and unsigned B.
@pytest.mark.parametrize("wl", [
    W.qlinear_matmul_u8(m=300, k=512, n=200),
    W.qlinear_matmul_u8(m=257, k=1024, n=513, a_zero=0, b_dtype="u8", b_zero=77),
    W.qlinear_matmul_u8(m=129, k=272, n=96, a_zero=9, b_dtype="u8", b_zero=250, scales=(0.25, 0.125, 2.0)),
    W.matmul_integer_u8(m=384, k=2048, n=256, a_zero=128, b_zero=3),
    W.matmul_integer_u8(m=100, k=32, n=20, a_zero=0, b_zero=0),
    W.matmul_integer_u8(m=1, k=16, n=1, a_zero=255, b_zero=-128),
], ids=lambda w: w.name + str(sorted(w.params.items()))[:60])
def test_qmatmul_tensor_cores_vs_port(wl):
    require_gpu()
    plan = plan_for(wl)
    assert "[tensor cores]" in plan.ops[0].label
    x = wl.make_inputs(5)
    ref = oracle.run_graph(wl.graph, x)
    out = Session(plan).run(x)
    for k, v in ref.items():
        assert_bitexact(out[k], v, k)


@pytest.mark.parametrize("quantized", [False, True])
def test_qmatmul_tensor_cores_runtime_b(quantized):
    """B a graph input rather than an initializer: B^T and its column sums are
    written by a preparation launch every run."""
    require_gpu()
    m, k, n = 200, 320, 72
    if quantized:
        inits = {"a_s": np.asarray(0.02, np.float32).reshape(()), "a_z": np.asarray(17, np.uint8).reshape(()),
                 "b_s": np.asarray(0.01, np.float32).reshape(()), "b_z": np.asarray(-9, np.int8).reshape(()),
                 "y_s": np.asarray(0.7, np.float32).reshape(()), "y_z": np.asarray(3, np.uint8).reshape(())}
        node = NodeSpec("QLinearMatMul", "qmm", ("A", "a_s", "a_z", "B", "b_s", "b_z", "y_s", "y_z"), ("Y",))
        out = TensorSpec("Y", "u8", (m, n))
    else:
        inits = {"a_z": np.asarray(200, np.uint8).reshape(()), "b_z": np.asarray(5, np.int8).reshape(())}
        node = NodeSpec("MatMulInteger", "mmi", ("A", "B", "a_z", "b_z"), ("Y",))
        out = TensorSpec("Y", "i32", (m, n))
    g = GraphSpec("qmm_runtime_b", [TensorSpec("A", "u8", (m, k)), TensorSpec("B", "i8", (k, n))], [out], [node],
                  initializers=inits, opset_imports=(("", 10),))
    wl = W.Workload("qmm_runtime_b", g, None, {"A": 0, "Y": 0}, {})
    plan = plan_for(wl)
    assert "[tensor cores]" in plan.ops[0].label
    rng = np.random.default_rng(11)
    x = {"A": rng.integers(0, 256, (m, k)).astype(np.uint8), "B": rng.integers(-128, 128, (k, n)).astype(np.int8)}
    ref = oracle.run_graph(g, x)
    sess = Session(plan)
    for _ in range(2):  # the second run recomputes B^T and the column sums from zero
        got = sess.run(x)
        assert_bitexact(got["Y"], ref["Y"], "Y")


def test_qmatmul_tensor_cores_largest_k():
    """K = 32768 with every A byte 255: the largest raw sums the path admits."""
    require_gpu()
    wl = W.matmul_integer_u8(m=130, k=32768, n=40, a_zero=0, b_zero=0)
    plan = plan_for(wl)
    assert "[tensor cores]" in plan.ops[0].label
    x = {"A": np.full((130, 32768), 255, np.uint8)}
    ref = oracle.run_graph(wl.graph, x)
    out = Session(plan).run(x)
    assert_bitexact(out["Y"], ref["Y"], "Y")


# rows staged in shared memory: (64, 1000), (300, 4096) and (10, 4) four-float copies, (5, 4097) and
# (2, 3, 4, 50) scalar, (2, 20001) one row per block; rows too long for twelve per SM stream through
# L2: (7, 20000) and (3, 60000), both ending in a partial chunk; (2, 60001) and (8, 300, 5) take the
# strided kernel
@pytest.mark.parametrize("shape,axis", [((64, 1000), -1), ((300, 4096), 1), ((7, 20000), 1), ((3, 60000), 1),
                                        ((10, 4), 1), ((5, 4097), -1), ((2, 20001), 1), ((2, 60001), 1),
                                        ((8, 300, 5), 1), ((2, 3, 4, 50), 3), ((1, 1), 0)])
def test_softmax_vs_port(shape, axis):
    require_gpu()
    wl = W.softmax_f32(shape, axis)
    x = wl.make_inputs(2)
    flat = x["X"].reshape(-1)
    flat[:3] = np.array([30.0, -50.0, 0.0], np.float32)[:flat.size]
    ref = oracle.run_graph(wl.graph, x)["Y"]
    out = Session(plan_for(wl)).run(x)["Y"]
    assert int(ulp_diff_f32(out, ref).max(initial=0)) <= SOFTMAX_MAX_ULP


@pytest.mark.parametrize("wl", [
    W.conv_f32(batch=2, cin=40, cout=70, h=23, w=19, kernel=3, pad=1),         # partial channel / pixel tiles
    W.conv_f32(batch=1, cin=8, cout=8, h=9, w=9, kernel=7, pad=3),              # 49 taps: untiled kernel
    W.conv_f32(batch=2, cin=12, cout=36, h=15, w=13, kernel=5, stride=3, pad=2, dilation=2, group=4),
], ids=lambda w: w.name + str(sorted(w.params.items()))[:60])
def test_conv_f32_tiled_vs_port(wl):
    require_gpu()
    x = wl.make_inputs(6)
    ref = oracle.run_graph(wl.graph, x)
    out = Session(plan_for(wl)).run(x)
    assert_bitexact(out["Y"], ref["Y"], "Y")


def test_conv_f32_skipped_taps():
    """Taps outside the image are skipped, not added as zero: an output whose
    taps all fall outside keeps a -0.0 bias, and an infinite weight over an
    in-image zero gives NaN only where the reference multiplies."""
    require_gpu()
    wl = W.conv_f32(batch=1, cin=3, cout=5, h=6, w=6, kernel=3, pad=3)
    wl.graph.initializers["bias"] = np.full(5, -0.0, np.float32)
    w = wl.graph.initializers["W"].copy()
    w[1, 2, 0, 0] = np.inf
    w[3, 0, 2, 1] = -np.inf
    wl.graph.initializers["W"] = w
    x = wl.make_inputs(7)
    x["X"][0, :, ::2, ::3] = 0.0
    ref = oracle.run_graph(wl.graph, x)
    out = Session(plan_for(wl)).run(x)
    assert np.signbit(ref["Y"][0, :, 0, 0]).all()  # the corner output sees no tap
    assert_bitexact(out["Y"], ref["Y"], "Y")


@pytest.mark.parametrize("out_dtype,zero,scale", [("u8", 128, 0.02), ("i8", -7, 0.05)])
def test_quant_dequant_per_tensor_x4(out_dtype, zero, scale):
    """Per-tensor scale, element count a multiple of 4: four values per thread,
    with ties, out-of-range values, infinities and NaN among them."""
    require_gpu()
    wl = W.quant_dequant((64, 100), out_dtype=out_dtype, zero=zero, scale=scale)
    x = wl.make_inputs(8)
    flat = x["X"].reshape(-1)
    flat[:8] = np.array([0.5, 1.5, -2.5, 1e6, -1e6, np.inf, -np.inf, np.nan], np.float32) * np.float32(scale)
    flat[-3:] = [np.nan, -0.0, 2.5 * scale]
    ref = oracle.run_graph(wl.graph, x)
    out = Session(plan_for(wl)).run(x)
    for k, v in ref.items():
        assert_bitexact(out[k], v, k)


def test_quantize_per_axis_and_specials():
    require_gpu()
    shape = (3, 4, 10)
    g = GraphSpec("qax", [TensorSpec("X", "f32", shape)], [TensorSpec("Q", "u8", shape), TensorSpec("D", "f32", shape)],
                  [NodeSpec("QuantizeLinear", "q", ("X", "s", "z"), ("Q",), {"axis": 1}),
                   NodeSpec("DequantizeLinear", "dq", ("Q", "s", "z"), ("D",), {"axis": 1})],
                  {"s": np.array([0.1, 0.02, 0.5, 3.0], np.float32), "z": np.array([0, 100, 128, 255], np.uint8)},
                  opset_imports=(("", 13),))
    wl = W.Workload("qax", g, lambda seed=0: {}, {"X": 0, "Q": 0, "D": 0}, {})
    x = (np.random.default_rng(0).standard_normal(shape) * 20).astype(np.float32)
    x[0, 0, :6] = [np.inf, -np.inf, np.nan, 0.05, 0.15, -0.25]   # ties at .5 round to even
    ref = oracle.run_graph(g, {"X": x})
    out = Session(plan_for(wl)).run({"X": x})
    for k in ("Q", "D"):
        assert_bitexact(out[k], ref[k], k)

"""Host-side plan emission (no GPU): plan format, kernel-id mirror, boundary
parity with the reference's own LoweredModel, unsupported-op behaviour."""
import struct

import numpy as np
import pytest

from emx_onnx_cgen_b200 import kernel_ids as K, lowering, workloads as W
from emx_onnx_cgen_b200.plan import B200PlanEmitter, _HDR, PLAN_MAGIC
from emx_onnx_cgen_b200.spec import GraphSpec, NodeSpec, TensorSpec
from oracle import refc

SMALL = {
    "qconv": lambda: W.qconv_stack_int8(batch=2, height=12, width=12),
    "qconv_c16": lambda: W.qconv_stack_int8(batch=1, channels=16, height=5, width=5, n_convs=3),
    "mlp": lambda: W.mlp_fp32(m=4, k=32, hidden=64),
    "llama_int4": lambda: W.llama_mlp_int4(m=4, hidden=64, inter=96),
    "nbits_zp_bias": lambda: W.matmul_nbits_f16(m=5, k=96, n=40, zero_points="block", bias=True),
    "nbits_zpcol_b16": lambda: W.matmul_nbits_f16(m=3, k=64, n=24, block=16, zero_points="column"),
    "swish_mul": lambda: W.swish_mul_f16((8, 24)),
    "lstm": lambda: W.lstm_fp32(seq=3, batch=2, input_size=8, hidden=16),
    "attention": lambda: W.attention_fp16(batch=1, heads=2, seq=16, head_dim=8),
    "maxpool": lambda: W.pool8(),
    "maxpool_same": lambda: W.pool8(shape=(2, 3, 10, 7), kernel=(4, 3), strides=(3, 2), auto_pad="SAME_LOWER"),
    "qavgpool": lambda: W.pool8(kind="avg", count_include_pad=1, ceil_mode=1),
    "qsoftmax": lambda: W.qlinear_softmax8(),
    "qsoftmax_opset11": lambda: W.qlinear_softmax8(shape=(3, 4, 6), axis=1, opset=11),
    "transpose": lambda: W.transpose(),
    "kws_qoperator_model": lambda: __import__("golden_util").load("kws_qoperator")[0],
}


def test_kernel_ids_parsed_from_header():
    assert K.K_QCONV_TC == 2 and K.K_PAD_NHWC == 1
    assert K.QC_ADD_SIGNED > K.QC_N
    assert K.NAMES[K.K_QCONV_TC] == "qconv_tc"


@pytest.mark.parametrize("key", sorted(SMALL))
def test_plan_matches_reference_lowering(key):
    if not refc.reference_available():
        pytest.skip("reference source tree not present")
    wl = SMALL[key]()
    mine = B200PlanEmitter().emit_plan(lowering.lower(wl.graph))
    _, ref_lowered = refc.lower(wl.graph)
    theirs = B200PlanEmitter().emit_plan(ref_lowered)
    assert mine.plan_bytes == theirs.plan_bytes
    assert mine.weight_bytes == theirs.weight_bytes


def test_qconv_stack_plan_shape():
    plan = B200PlanEmitter().emit_plan(lowering.lower(W.qconv_stack_int8().graph))
    kinds = [K.NAMES[o.kernel] for o in plan.ops]
    assert kinds == ["pad_nhwc", "qconv_tc", "qconv_tc", "qconv_tc", "qconv_tc"]
    hdr = _HDR.unpack_from(plan.plan_bytes)
    assert hdr[0] == PLAN_MAGIC and hdr[6] == 32
    assert len(plan.plan_bytes) == 56 + 96 * len(plan.tensors) + 2 * 8 + 440 * len(plan.ops)


def test_llama_mlp_plan_fuses_gate_up_swish_mul():
    plan = B200PlanEmitter().emit_plan(lowering.lower(W.llama_mlp_int4(m=8, hidden=128, inter=192).graph))
    kinds = [K.NAMES[o.kernel] for o in plan.ops]
    assert kinds == ["nbits_gemm", "nbits_gemm"]
    assert plan.ops[0].ip[K.NB_FUSED] == 1 and plan.ops[1].ip[K.NB_FUSED] == 0
    assert plan.ops[0].ip[K.NB_NTILES] == 3 and plan.ops[1].ip[K.NB_NTILES] == 1


def test_nbits_rejections():
    wl = W.matmul_nbits_f16(m=4, k=60, n=24)
    with pytest.raises(lowering.UnsupportedOpError, match="multiples of 8"):
        B200PlanEmitter().emit_plan(lowering.lower(wl.graph))


def test_unsupported_op_raises():
    g = GraphSpec("bad", [TensorSpec("X", "f32", (2, 2))], [TensorSpec("Y", "f32", (2, 2))],
                  [NodeSpec("Cos", "c", ("X",), ("Y",))], {})
    with pytest.raises(lowering.UnsupportedOpError):
        B200PlanEmitter().emit_plan(lowering.lower(g))


EMPTY_EXTENT_CASES = {
    "qconv_batch0": lambda: W.qconv_stack_int8(batch=0, height=8, width=8),
    "mlp_rows0": lambda: W.mlp_fp32(m=0, k=8, hidden=16),
    "attention_batch0": lambda: W.attention_fp16(batch=0, heads=1, seq=8, head_dim=16),
    "attention_seq0": lambda: W.attention_fp16(batch=1, heads=1, seq=0, head_dim=16),
    "lstm_batch0": lambda: W.lstm_fp32(seq=3, batch=0, input_size=4, hidden=4),
    "int4_mlp_rows0": lambda: W.llama_mlp_int4(m=0, hidden=64, inter=64),
}


@pytest.mark.parametrize("name", sorted(EMPTY_EXTENT_CASES))
def test_ops_with_only_empty_outputs_launch_nothing(name):
    """A zero extent (the reference accepts zero dimensions) empties every
    output: the reference's loops run zero times, and the plan has no op."""
    wl = EMPTY_EXTENT_CASES[name]()
    plan = B200PlanEmitter().emit_plan(lowering.lower(wl.graph))
    assert plan.ops == []
    assert all(0 in shp for shp in plan.output_shapes)


def test_empty_input_with_non_empty_outputs_is_rejected():
    # an LSTM over zero steps still has Y_h / Y_c; a Gemm with K = 0 still has Y
    with np.errstate(divide="ignore"):
        cases = [W.lstm_fp32(seq=0, batch=2, input_size=4, hidden=4), W.mlp_fp32(m=2, k=0, hidden=16)]
    for wl in cases:
        with pytest.raises(lowering.UnsupportedOpError, match="empty input"):
            B200PlanEmitter().emit_plan(lowering.lower(wl.graph))


def test_weight_image_layout():
    """Tensor-core weight image: [tap][oc][cin] with each row's 16-byte chunks
    at their swizzled positions (chunk j of row r at j ^ ((r*cin >> 7) & (cin/16-1)))."""
    from emx_onnx_cgen_b200.plan import qconv_weight_image
    for cin in (32, 64, 128):
        w = np.random.default_rng(cin).integers(-127, 128, (64, cin, 3, 3)).astype(np.int8)
        img = qconv_weight_image(w)
        assert img.shape == (9, 64, cin)
        for tap in (0, 4, 8):
            kh, kw = divmod(tap, 3)
            for oc in (0, 1, 2, 5, 63):
                phase = ((oc * cin) >> 7) & (cin // 16 - 1)
                for j in range(cin // 16):
                    pos = j ^ phase
                    assert np.array_equal(img[tap, oc, 16 * pos:16 * pos + 16], w[oc, 16 * j:16 * j + 16, kh, kw])


def _chain_marks(plan):
    return [(K.NAMES[o.kernel], o.ip.get(K.QC_CHAIN, 0)) for o in plan.ops]


def test_conv_stack_is_one_chain():
    """Consecutive same-geometry convolutions, each reading the previous
    one's output, form one chain: the first op carries the length and a
    zero-initialised state tensor (epoch, finished CTAs, one progress word per
    128-row tile), the others are marked as members."""
    plan = B200PlanEmitter().emit_plan(lowering.lower(W.qconv_stack_int8().graph))
    assert _chain_marks(plan) == [("pad_nhwc", 0), ("qconv_tc", 4), ("qconv_tc", -1), ("qconv_tc", -1),
                                  ("qconv_tc", -1)]
    head = plan.ops[1]
    state = plan.tensors[head.tensors[6]]
    n, hp, wp, oh, ow = (head.ip[k] for k in (K.QC_N, K.QC_HP, K.QC_WP, K.QC_OH, K.QC_OW))
    q_end = (n - 1) * hp * wp + (oh - 1) * wp + ow
    assert state.nbytes == 8 * (2 + -(-q_end // 128))
    # every member reads the previous member's output
    for a, b in zip(plan.ops[1:], plan.ops[2:]):
        assert b.tensors[0] == a.tensors[4]


@pytest.mark.parametrize("n_convs", [1, 2, 3, 9])
def test_chain_lengths_and_opt_out(n_convs):
    wl = W.qconv_stack_int8(batch=2, channels=32, height=8, width=8, n_convs=n_convs)
    plan = B200PlanEmitter().emit_plan(lowering.lower(wl.graph))
    marks = [m for _, m in _chain_marks(plan)[1:]]
    if n_convs == 1:
        assert marks == [0]
    else:  # chains hold at most 8 convolutions; a lone remainder runs on its own (0)
        heads = [m for m in marks if m > 0]
        assert sum(heads) + marks.count(0) == n_convs and all(1 < h <= 8 for h in heads)
        assert marks.count(-1) == sum(heads) - len(heads)
        assert heads[0] == min(n_convs, 8)
    plain = B200PlanEmitter(chain_convs=False).emit_plan(lowering.lower(wl.graph))
    assert all(m == 0 for _, m in _chain_marks(plain))


def test_conv_f32_zero_taps_flag():
    """Out-of-image taps may be staged as zeros only when that cannot change a
    result: finite weights and no -0.0 bias entry."""
    def flag(bias=None, w_patch=None):
        wl = W.conv_f32(batch=1, cin=2, cout=3, h=5, w=5, kernel=3, pad=1)
        if bias is not None:
            wl.graph.initializers["bias"] = np.asarray(bias, np.float32)
        if w_patch is not None:
            w = wl.graph.initializers["W"].copy()
            w[0, 0, 0, 0] = w_patch
            wl.graph.initializers["W"] = w
        return B200PlanEmitter().emit_plan(lowering.lower(wl.graph)).ops[0].ip[K.CF_ZERO_TAPS_OK]

    assert flag() == 1
    assert flag(bias=[0.0, 1.0, -2.0]) == 1
    assert flag(bias=[0.5, -0.0, 1.0]) == 0
    assert flag(w_patch=np.inf) == 0
    assert flag(w_patch=np.nan) == 0


def _weight(plan, tid, dtype):
    t = plan.tensors[tid]
    return np.frombuffer(plan.weight_bytes[t.offset:t.offset + t.nbytes], dtype=dtype).reshape(t.shape)


@pytest.mark.parametrize("b_dtype", ["i8", "u8"])
def test_qmatmul_tensor_core_plan_packs_constant_b(b_dtype):
    """K a multiple of 16 with B an initializer: B^T [N][K] and B's column sums
    (signed per B's type) are packed into the weights; A's row sums are scratch."""
    from emx_onnx_cgen_b200.plan import T_TEMP, T_WEIGHT
    wl = W.qlinear_matmul_u8(m=40, k=96, n=24, b_dtype=b_dtype, b_zero=3)
    plan = B200PlanEmitter().emit_plan(lowering.lower(wl.graph))
    op = plan.ops[0]
    assert "[tensor cores]" in op.label and op.ip[K.QM_B_PACKED] == 1
    b = wl.graph.initializers["B"]
    bt = _weight(plan, op.tensors[3], np.uint8)
    assert plan.tensors[op.tensors[3]].kind == T_WEIGHT and bt.shape == (24, 96)
    assert np.array_equal(bt, np.ascontiguousarray(b.T).view(np.uint8))
    assert np.array_equal(_weight(plan, op.tensors[4], np.int32), b.astype(np.int64).sum(axis=0))
    assert plan.tensors[op.tensors[5]].kind == T_TEMP and plan.tensors[op.tensors[5]].shape == (40,)


def test_qmatmul_tensor_core_plan_runtime_b_and_ineligible_k():
    from emx_onnx_cgen_b200.plan import T_TEMP
    m, k, n = 8, 64, 16
    g = GraphSpec("mmi_rt", [TensorSpec("A", "u8", (m, k)), TensorSpec("B", "i8", (k, n))],
                  [TensorSpec("Y", "i32", (m, n))], [NodeSpec("MatMulInteger", "mmi", ("A", "B"), ("Y",))],
                  initializers={}, opset_imports=(("", 10),))
    plan = B200PlanEmitter().emit_plan(lowering.lower(g))
    op = plan.ops[0]
    assert op.ip.get(K.QM_B_PACKED, 0) == 0 and len(op.tensors) == 6
    assert all(plan.tensors[t].kind == T_TEMP for t in plan.ops[0].tensors[3:])
    # K not a multiple of 16, or the tensor cores switched off: the CUDA-core kernel
    for wl, kw in ((W.matmul_integer_u8(m=8, k=40, n=16), {}), (W.matmul_integer_u8(m=8, k=64, n=16),
                                                                 {"use_tensor_cores": False})):
        op = B200PlanEmitter(**kw).emit_plan(lowering.lower(wl.graph)).ops[0]
        assert len(op.tensors) == 3 and "[tensor cores]" not in op.label


def test_swish_plan_reserves_a_table():
    wl = W.swish_mul_f16((8, 24))
    plan = B200PlanEmitter().emit_plan(lowering.lower(wl.graph))
    (sw,) = [o for o in plan.ops if o.kernel == K.K_SWISH_F16]  # standalone: no MatMulNBits to fuse into
    assert plan.tensors[sw.tensors[2]].nbytes == 2 * 65536


def test_kws_qoperator_model_plan():
    """The reference's micro_kws_m_static_qoperator.onnx (stored with its golden
    fixture): both Reshapes alias their source, every op has a kernel."""
    from golden_util import load
    fx = load("kws_qoperator")[0]
    plan = B200PlanEmitter().emit_plan(lowering.lower(fx.graph))
    kinds = [K.NAMES[o.kernel] for o in plan.ops]
    assert kinds == ["quantize_linear", "qconv_generic", "maxpool", "qconv_generic", "qlinear_avgpool",
                     "qconv_generic", "qlinear_avgpool", "dequantize_linear", "transpose", "quantize_linear",
                     "qlinear_matmul", "qlinear_add", "qlinear_matmul", "qlinear_add", "qlinear_matmul",
                     "qlinear_add", "qlinear_softmax", "dequantize_linear"]


def test_reshape_to_graph_output_copies():
    g = GraphSpec("r", [TensorSpec("X", "f32", (2, 3, 4))], [TensorSpec("Y", "f32", (2, 12))],
                  [NodeSpec("Reshape", "r", ("X", "s"), ("Y",))], {"s": np.array([2, -1], np.int64)})
    plan = B200PlanEmitter().emit_plan(lowering.lower(g))
    assert [K.NAMES[o.kernel] for o in plan.ops] == ["copy"]
    assert plan.ops[0].ip[K.CP_BYTES] == 96 and plan.ops[0].ip[K.CP_BATCH] == 2


def test_qsoftmax_exp_table_is_libm_expf():
    """The planner's exp table holds the C library's expf of v(b) - v(bm)."""
    import ctypes
    import ctypes.util
    from emx_onnx_cgen_b200.plan import qsoftmax_exp_table
    libm = ctypes.CDLL(ctypes.util.find_library("m"))
    libm.expf.restype, libm.expf.argtypes = ctypes.c_float, [ctypes.c_float]
    t = qsoftmax_exp_table(True, -5, np.float32(0.11))
    v = lambda b: np.float32(np.float32(np.int8(np.uint8(b)).astype(np.int32) + 5) * np.float32(0.11))
    for b, bm in [(0, 0), (3, 200), (127, 128), (128, 127), (255, 1)]:
        assert t[b, bm] == np.float32(libm.expf(float(np.float32(v(b) - v(bm))))), (b, bm)

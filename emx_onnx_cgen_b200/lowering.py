"""Lowering of a ``GraphSpec`` into ``LoweredModel`` objects for the hot-path ops.

The drop-in boundary of this backend is the reference compiler's
``LoweredModel`` (src/emx_onnx_cgen/codegen/c_emitter.py:333-350), produced by
``Compiler._lower_model`` (compiler.py:514-606).  ``B200PlanEmitter`` reads
lowered ops by class name and field name only, so it accepts the reference's
own objects unchanged.  Where the reference compiler is not installed (the GPU
hosts that run the tests and the benchmark), this module produces objects with
the same class names and the same fields for the ops this backend runs:

  QLinearConvOp   ir/ops/nn.py:4734     QLinearAddOp  ir/ops/elementwise.py:1114
  GemmOp          ir/ops/nn.py:1624     UnaryOp       ir/ops/elementwise.py:538
  BinaryOp        ir/ops/elementwise.py:23
  MatMulNBitsOp   ir/ops/nn.py:1035     AttentionOp   ir/ops/nn.py:2478
  LstmOp          ir/ops/nn.py:8449     ReshapeOp     ir/ops/misc.py:1995
  TransposeOp     ir/ops/misc.py:1927   MaxPoolOp     ir/ops/nn.py:9614
  QLinearAveragePoolOp ir/ops/nn.py:5454 QLinearSoftmaxOp ir/ops/nn.py:5997

Attribute defaults follow the reference's lowerings (lowering/qlinear_conv.py:40,
qlinear_add.py:31, gemm.py:9, matmul_nbits.py:120, attention.py:363 (scale
default 1/sqrt(head_size), attention.py:313), lstm.py:335).  The test suite
checks, wherever the reference is importable, that both lowerings yield
byte-identical plans.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from enum import Enum

import numpy as np

from .spec import GraphSpec


class ScalarType(str, Enum):
    """Mirror of the reference's ScalarType values used on the hot path."""
    F32 = "f32"
    F16 = "f16"
    F64 = "f64"
    U8 = "u8"
    I8 = "i8"
    I32 = "i32"
    I64 = "i64"
    BOOL = "bool"


class ScalarFunction(str, Enum):
    RELU = "relu"
    SWISH = "swish"
    SIGMOID = "sigmoid"
    TANH = "tanh"
    MUL = "mul"
    ADD = "add"


class UnsupportedOpError(Exception):
    """Same role as the reference's errors.UnsupportedOpError (errors.py:5)."""


@dataclass(frozen=True)
class ConstTensor:
    name: str
    shape: tuple[int, ...]
    data: np.ndarray
    dtype: ScalarType


@dataclass
class OpContext:
    shapes: dict[str, tuple[int, ...]]
    dtypes: dict[str, ScalarType]

    def shape(self, name: str) -> tuple[int, ...]:
        return self.shapes[name]

    def dtype(self, name: str) -> ScalarType:
        return self.dtypes[name]


@dataclass(frozen=True)
class LoweredModel:
    name: str
    input_names: tuple[str, ...]
    input_shapes: tuple[tuple[int, ...], ...]
    input_dtypes: tuple[ScalarType, ...]
    output_names: tuple[str, ...]
    output_shapes: tuple[tuple[int, ...], ...]
    output_dtypes: tuple[ScalarType, ...]
    constants: tuple[ConstTensor, ...]
    ops: tuple[object, ...]
    op_context: OpContext


# ------------------------------------------------------------------ op dataclasses
@dataclass(frozen=True)
class QLinearConvOp:
    input0: str
    input_scale: str
    input_zero_point: str
    weights: str
    weight_scale: str
    weight_zero_point: str
    output_scale: str
    output_zero_point: str
    bias: str | None
    output: str
    batch: int
    in_channels: int
    out_channels: int
    spatial_rank: int
    in_spatial: tuple[int, ...]
    out_spatial: tuple[int, ...]
    kernel_shape: tuple[int, ...]
    strides: tuple[int, ...]
    pads: tuple[int, ...]
    dilations: tuple[int, ...]
    group: int
    input_dtype: ScalarType
    weight_dtype: ScalarType
    dtype: ScalarType
    weight_scale_per_channel: bool
    weight_zero_per_channel: bool


@dataclass(frozen=True)
class QLinearAddOp:
    input0: str
    input0_scale: str
    input0_zero_point: str
    input1: str
    input1_scale: str
    input1_zero_point: str
    output_scale: str
    output_zero_point: str
    output: str
    input0_shape: tuple[int, ...]
    input1_shape: tuple[int, ...]
    output_shape: tuple[int, ...]
    input0_dtype: ScalarType
    input1_dtype: ScalarType
    dtype: ScalarType


@dataclass(frozen=True)
class GemmOp:
    input_a: str
    input_b: str
    input_c: str | None
    output: str
    trans_a: int
    trans_b: int
    alpha: float | int
    beta: float | int


@dataclass(frozen=True)
class UnaryOp:
    input0: str
    output: str
    function: ScalarFunction
    params: tuple[float, ...] = ()


@dataclass(frozen=True)
class BinaryOp:
    input0: str
    input1: str
    output: str
    function: ScalarFunction


@dataclass(frozen=True)
class MatMulNBitsOp:
    input0: str
    input1: str
    scales: str
    zero_points: str | None
    bias: str | None
    output: str
    bits: int
    block_size: int
    k: int
    n: int
    accuracy_level: int
    n_blocks_per_col: int
    blob_size: int
    input0_shape: tuple[int, ...]
    output_shape: tuple[int, ...]
    m: int
    input0_dtype: ScalarType
    output_dtype: ScalarType
    scales_dtype: ScalarType


@dataclass(frozen=True)
class AttentionOp:
    input_q: str
    input_k: str
    input_v: str
    input_attn_mask: str | None
    input_past_key: str | None
    input_past_value: str | None
    output: str
    output_present_key: str | None
    output_present_value: str | None
    output_qk_matmul: str | None
    batch: int
    q_heads: int
    kv_heads: int
    q_seq: int
    kv_seq: int
    total_seq: int
    past_seq: int
    qk_head_size: int
    v_head_size: int
    scale: float
    is_causal: bool
    softcap: float
    q_rank: int
    head_group_size: int
    dtype: ScalarType


@dataclass(frozen=True)
class LstmOp:
    input_x: str
    input_w: str
    input_r: str
    input_b: str | None
    input_sequence_lens: str | None
    input_initial_h: str | None
    input_initial_c: str | None
    input_p: str | None
    output_y: str | None
    output_y_h: str | None
    output_y_c: str | None
    seq_length: int
    batch_size: int
    input_size: int
    hidden_size: int
    num_directions: int
    direction: str
    layout: int
    input_forget: int
    clip: float | None
    activation_kinds: tuple[int, ...]
    dtype: ScalarType


@dataclass(frozen=True)
class QLinearMatMulOp:
    input0: str
    input0_scale: str
    input0_zero_point: str
    input1: str
    input1_scale: str
    input1_zero_point: str
    output_scale: str
    output_zero_point: str
    output: str
    input0_shape: tuple[int, ...]
    input1_shape: tuple[int, ...]
    output_shape: tuple[int, ...]
    m: int
    n: int
    k: int
    input0_dtype: ScalarType
    input1_dtype: ScalarType
    dtype: ScalarType
    input0_scale_dtype: ScalarType
    input1_scale_dtype: ScalarType
    output_scale_dtype: ScalarType


@dataclass(frozen=True)
class MatMulIntegerOp:
    input0: str
    input1: str
    input0_zero_point: str | None
    input1_zero_point: str | None
    output: str
    input0_shape: tuple[int, ...]
    input1_shape: tuple[int, ...]
    output_shape: tuple[int, ...]
    m: int
    n: int
    k: int
    input0_dtype: ScalarType
    input1_dtype: ScalarType
    dtype: ScalarType


@dataclass(frozen=True)
class ConvOp:
    input0: str
    weights: str
    bias: str | None
    output: str
    batch: int
    in_channels: int
    out_channels: int
    spatial_rank: int
    in_spatial: tuple[int, ...]
    out_spatial: tuple[int, ...]
    kernel_shape: tuple[int, ...]
    strides: tuple[int, ...]
    pads: tuple[int, ...]
    dilations: tuple[int, ...]
    group: int
    dtype: ScalarType


@dataclass(frozen=True)
class SoftmaxOp:
    input0: str
    output: str
    axis: int | None
    use_legacy_axis_semantics: bool = False


@dataclass(frozen=True)
class QuantizeLinearOp:
    input0: str
    scale: str
    zero_point: str | None
    output: str
    axis: int | None
    block_size: int | None


@dataclass(frozen=True)
class DequantizeLinearOp:
    input0: str
    scale: str
    zero_point: str | None
    output: str
    axis: int | None
    block_size: int | None


@dataclass(frozen=True)
class ReshapeOp:
    input0: str
    output: str


@dataclass(frozen=True)
class TransposeOp:
    input0: str
    output: str
    perm: tuple[int, ...]


@dataclass(frozen=True)
class MaxPoolOp:
    input0: str
    output: str
    indices: str | None
    batch: int
    channels: int
    spatial_rank: int
    in_spatial: tuple[int, ...]
    out_spatial: tuple[int, ...]
    kernel_shape: tuple[int, ...]
    strides: tuple[int, ...]
    pads: tuple[int, ...]
    dilations: tuple[int, ...]
    ceil_mode: bool
    storage_order: int
    dtype: ScalarType
    indices_dtype: ScalarType | None


@dataclass(frozen=True)
class QLinearAveragePoolOp:
    input0: str
    input_scale: str
    input_zero_point: str
    output_scale: str
    output_zero_point: str
    output: str
    batch: int
    channels: int
    in_h: int
    in_w: int
    out_h: int
    out_w: int
    kernel_h: int
    kernel_w: int
    dilation_h: int
    dilation_w: int
    stride_h: int
    stride_w: int
    pad_top: int
    pad_left: int
    pad_bottom: int
    pad_right: int
    count_include_pad: bool
    input_dtype: ScalarType
    dtype: ScalarType
    input_scale_dtype: ScalarType
    output_scale_dtype: ScalarType
    input_scale_shape: tuple[int, ...]
    output_scale_shape: tuple[int, ...]
    input_zero_shape: tuple[int, ...]
    output_zero_shape: tuple[int, ...]
    spatial_rank: int = 2
    channels_last: bool = False


@dataclass(frozen=True)
class QLinearSoftmaxOp:
    input0: str
    input_scale: str
    input_zero_point: str
    output_scale: str
    output_zero_point: str
    output: str
    input_shape: tuple[int, ...]
    output_shape: tuple[int, ...]
    axis: int
    outer: int
    axis_size: int
    inner: int
    dtype: ScalarType
    input_dtype: ScalarType
    input_scale_dtype: ScalarType
    output_scale_dtype: ScalarType


def _auto_pads(a, in_spatial, ks, strides, dil) -> tuple[int, ...]:
    """(begin..., end...) pads of a pooling node: explicit, or from auto_pad
    (VALID: none; SAME_UPPER / SAME_LOWER: out = ceil(in / stride), the odd
    pad at the end / the start), as lowering/maxpool.py:78-103 resolves them."""
    rank = len(in_spatial)
    mode = a.get("auto_pad", "NOTSET")
    mode = mode.decode() if isinstance(mode, bytes) else str(mode)
    if mode in ("", "NOTSET"):
        return tuple(int(v) for v in a.get("pads", [0] * (2 * rank)))
    if mode == "VALID":
        return (0,) * (2 * rank)
    if mode not in ("SAME_UPPER", "SAME_LOWER"):
        raise UnsupportedOpError(f"auto_pad {mode} is not supported")
    begin, end = [], []
    for size, k, s, d in zip(in_spatial, ks, strides, dil):
        need = max(0, (-(-size // s) - 1) * s + d * (k - 1) + 1 - size)
        first = need // 2 if mode == "SAME_UPPER" else (need + 1) // 2
        begin.append(first)
        end.append(need - first)
    return (*begin, *end)


def _pool_out(size: int, k: int, s: int, d: int, p0: int, p1: int, ceil_mode: bool) -> int:
    """Output extent of a pooling window (ONNX; with ceil_mode the last window
    must start inside the input or its leading pad)."""
    span = size + p0 + p1 - ((k - 1) * d + 1)
    out = (-(-span // s) if ceil_mode else span // s) + 1
    if ceil_mode and (out - 1) * s >= size + p0:
        out -= 1
    return out


# ------------------------------------------------------------------ lowering
def _st(suffix: str) -> ScalarType:
    return ScalarType(suffix)


def lower(spec: GraphSpec) -> LoweredModel:
    shapes: dict[str, tuple[int, ...]] = {}
    dtypes: dict[str, ScalarType] = {}
    for t in (*spec.inputs, *spec.outputs, *spec.values):
        shapes[t.name] = tuple(t.shape)
        dtypes[t.name] = _st(t.dtype)
    consts = []
    for name, arr in spec.initializers.items():
        t = spec.tensor(name)
        shapes[name] = tuple(arr.shape)
        dtypes[name] = _st(t.dtype)
        consts.append(ConstTensor(name, tuple(arr.shape), arr, _st(t.dtype)))
    ops = []
    _INITS.clear()
    _INITS.update(spec.initializers)
    _INITS["__opset__"] = np.int64(dict(spec.opset_imports).get("", 17))
    try:
        for node in spec.nodes:
            ops.append(_lower_node(node, shapes, dtypes))
    finally:
        _INITS.clear()
    return LoweredModel(
        name=spec.name,
        input_names=tuple(t.name for t in spec.inputs),
        input_shapes=tuple(tuple(t.shape) for t in spec.inputs),
        input_dtypes=tuple(_st(t.dtype) for t in spec.inputs),
        output_names=tuple(t.name for t in spec.outputs),
        output_shapes=tuple(tuple(t.shape) for t in spec.outputs),
        output_dtypes=tuple(_st(t.dtype) for t in spec.outputs),
        constants=tuple(consts),
        ops=tuple(ops),
        op_context=OpContext(shapes, dtypes),
    )


_INITS: dict[str, np.ndarray] = {}  # the graph's initializers while lower() runs (Reshape reads its shape)


def _initializer(name: str) -> np.ndarray:
    if name not in _INITS:
        raise UnsupportedOpError(f"'{name}' must be an initializer")
    return _INITS[name]


def _lower_node(node, shapes, dtypes):
    a = dict(node.attrs)
    ins = list(node.inputs)
    op = node.op_type
    if op == "QLinearConv":
        x, w = ins[0], ins[3]
        n, c, *sp = shapes[x]
        oc, _, *ks = shapes[w]
        rank = len(sp)
        ks = tuple(a.get("kernel_shape", ks))
        strides = tuple(a.get("strides", [1] * rank))
        dil = tuple(a.get("dilations", [1] * rank))
        pads = tuple(a.get("pads", [0] * (2 * rank)))
        out_sp = tuple((sp[i] + pads[i] + pads[i + rank] - ((ks[i] - 1) * dil[i] + 1)) // strides[i] + 1
                       for i in range(rank))
        y = node.outputs[0]
        shapes[y] = (n, oc, *out_sp)
        dtypes[y] = dtypes[ins[7]]
        ws_shape, wz_shape = shapes[ins[4]], shapes[ins[5]]
        return QLinearConvOp(
            input0=x, input_scale=ins[1], input_zero_point=ins[2], weights=w, weight_scale=ins[4],
            weight_zero_point=ins[5], output_scale=ins[6], output_zero_point=ins[7],
            bias=ins[8] if len(ins) > 8 and ins[8] else None, output=y, batch=n, in_channels=c,
            out_channels=oc, spatial_rank=rank, in_spatial=tuple(sp), out_spatial=out_sp, kernel_shape=ks,
            strides=strides, pads=pads, dilations=dil, group=int(a.get("group", 1)),
            input_dtype=dtypes[x], weight_dtype=dtypes[w], dtype=dtypes[ins[7]],
            weight_scale_per_channel=int(np.prod(ws_shape)) > 1,
            weight_zero_per_channel=int(np.prod(wz_shape)) > 1)
    if op == "QLinearAdd":
        y = node.outputs[0]
        shapes[y] = tuple(np.broadcast_shapes(shapes[ins[0]], shapes[ins[3]]))
        dtypes[y] = dtypes[ins[7]]
        return QLinearAddOp(
            input0=ins[0], input0_scale=ins[1], input0_zero_point=ins[2], input1=ins[3], input1_scale=ins[4],
            input1_zero_point=ins[5], output_scale=ins[6], output_zero_point=ins[7], output=y,
            input0_shape=shapes[ins[0]], input1_shape=shapes[ins[3]], output_shape=shapes[y],
            input0_dtype=dtypes[ins[0]], input1_dtype=dtypes[ins[3]], dtype=dtypes[y])
    if op == "Gemm":
        ta, tb = int(a.get("transA", 0)), int(a.get("transB", 0))
        sa, sb = shapes[ins[0]], shapes[ins[1]]
        m = sa[1] if ta else sa[0]
        nn_ = sb[0] if tb else sb[1]
        y = node.outputs[0]
        shapes[y] = (m, nn_)
        dtypes[y] = dtypes[ins[0]]
        return GemmOp(input_a=ins[0], input_b=ins[1], input_c=ins[2] if len(ins) > 2 and ins[2] else None,
                      output=y, trans_a=ta, trans_b=tb, alpha=float(a.get("alpha", 1.0)),
                      beta=float(a.get("beta", 1.0)))
    if op in ("Relu", "Swish", "Sigmoid", "Tanh"):
        y = node.outputs[0]
        shapes[y] = shapes[ins[0]]
        dtypes[y] = dtypes[ins[0]]
        fn = {"Relu": ScalarFunction.RELU, "Swish": ScalarFunction.SWISH, "Sigmoid": ScalarFunction.SIGMOID,
              "Tanh": ScalarFunction.TANH}[op]
        params = (float(a.get("alpha", 1.0)),) if op == "Swish" else ()
        return UnaryOp(input0=ins[0], output=y, function=fn, params=params)
    if op in ("Mul", "Add"):
        y = node.outputs[0]
        shapes[y] = tuple(np.broadcast_shapes(shapes[ins[0]], shapes[ins[1]]))
        dtypes[y] = dtypes[ins[0]]
        return BinaryOp(input0=ins[0], input1=ins[1], output=y,
                        function=ScalarFunction.MUL if op == "Mul" else ScalarFunction.ADD)
    if op == "MatMulNBits":
        k, n = int(a["K"]), int(a["N"])
        bits, block = int(a.get("bits", 4)), int(a.get("block_size", 32))
        nb = (k + block - 1) // block
        xs = shapes[ins[0]]
        y = node.outputs[0]
        shapes[y] = (*xs[:-1], n)
        dtypes[y] = dtypes[ins[0]]
        return MatMulNBitsOp(
            input0=ins[0], input1=ins[1], scales=ins[2],
            zero_points=ins[3] if len(ins) > 3 and ins[3] else None,
            bias=ins[5] if len(ins) > 5 and ins[5] else None, output=y, bits=bits, block_size=block, k=k, n=n,
            accuracy_level=int(a.get("accuracy_level", 0)), n_blocks_per_col=nb, blob_size=block * bits // 8,
            input0_shape=xs, output_shape=shapes[y], m=int(np.prod(xs[:-1])), input0_dtype=dtypes[ins[0]],
            output_dtype=dtypes[ins[0]], scales_dtype=dtypes[ins[2]])
    if op in ("QLinearMatMul", "MatMulInteger"):
        a_name, b_name = ins[0], ins[3] if op == "QLinearMatMul" else ins[1]
        xs, ws = shapes[a_name], shapes[b_name]
        if len(ws) != 2:
            raise UnsupportedOpError(f"{op}: only 2-D B has a B200 kernel")
        m, k, n = int(np.prod(xs[:-1])) if len(xs) > 1 else 1, xs[-1], ws[1]
        y = node.outputs[0]
        shapes[y] = (*xs[:-1], n)
        if op == "QLinearMatMul":
            dtypes[y] = dtypes[ins[7]]
            return QLinearMatMulOp(
                input0=ins[0], input0_scale=ins[1], input0_zero_point=ins[2], input1=ins[3], input1_scale=ins[4],
                input1_zero_point=ins[5], output_scale=ins[6], output_zero_point=ins[7], output=y,
                input0_shape=xs, input1_shape=ws, output_shape=shapes[y], m=m, n=n, k=k,
                input0_dtype=dtypes[ins[0]], input1_dtype=dtypes[ins[3]], dtype=dtypes[y],
                input0_scale_dtype=dtypes[ins[1]], input1_scale_dtype=dtypes[ins[4]],
                output_scale_dtype=dtypes[ins[6]])
        dtypes[y] = ScalarType.I32
        return MatMulIntegerOp(
            input0=ins[0], input1=ins[1], input0_zero_point=ins[2] if len(ins) > 2 and ins[2] else None,
            input1_zero_point=ins[3] if len(ins) > 3 and ins[3] else None, output=y, input0_shape=xs,
            input1_shape=ws, output_shape=shapes[y], m=m, n=n, k=k, input0_dtype=dtypes[ins[0]],
            input1_dtype=dtypes[ins[1]], dtype=ScalarType.I32)
    if op == "Conv":
        x, w = ins[0], ins[1]
        n, c, *sp = shapes[x]
        oc, _, *ks = shapes[w]
        rank = len(sp)
        ks = tuple(a.get("kernel_shape", ks))
        strides = tuple(a.get("strides", [1] * rank))
        dil = tuple(a.get("dilations", [1] * rank))
        pads = tuple(a.get("pads", [0] * (2 * rank)))
        out_sp = tuple((sp[i] + pads[i] + pads[i + rank] - ((ks[i] - 1) * dil[i] + 1)) // strides[i] + 1
                       for i in range(rank))
        y = node.outputs[0]
        shapes[y] = (n, oc, *out_sp)
        dtypes[y] = dtypes[x]
        return ConvOp(input0=x, weights=w, bias=ins[2] if len(ins) > 2 and ins[2] else None, output=y, batch=n,
                      in_channels=c, out_channels=oc, spatial_rank=rank, in_spatial=tuple(sp),
                      out_spatial=out_sp, kernel_shape=ks, strides=strides, pads=pads, dilations=dil,
                      group=int(a.get("group", 1)), dtype=dtypes[x])
    if op == "Softmax":
        y = node.outputs[0]
        shapes[y] = shapes[ins[0]]
        dtypes[y] = dtypes[ins[0]]
        return SoftmaxOp(input0=ins[0], output=y, axis=int(a.get("axis", -1)))
    if op in ("QuantizeLinear", "DequantizeLinear"):
        y = node.outputs[0]
        shapes[y] = shapes[ins[0]]
        if op == "QuantizeLinear":
            dtypes[y] = dtypes[ins[2]] if len(ins) > 2 and ins[2] else ScalarType.U8
            cls = QuantizeLinearOp
        else:
            dtypes[y] = dtypes[ins[1]]
            cls = DequantizeLinearOp
        return cls(input0=ins[0], scale=ins[1], zero_point=ins[2] if len(ins) > 2 and ins[2] else None, output=y,
                   axis=int(a["axis"]) if "axis" in a else None,
                   block_size=int(a["block_size"]) if "block_size" in a else None)
    if op == "Attention":
        b, hq, tq, d = shapes[ins[0]]
        _, hkv, tkv, _ = shapes[ins[1]]
        dv = shapes[ins[2]][3]
        y = node.outputs[0]
        shapes[y] = (b, hq, tq, dv)
        dtypes[y] = dtypes[ins[0]]
        scale = float(a["scale"]) if "scale" in a else 1.0 / math.sqrt(d)
        return AttentionOp(
            input_q=ins[0], input_k=ins[1], input_v=ins[2], input_attn_mask=None, input_past_key=None,
            input_past_value=None, output=y, output_present_key=None, output_present_value=None,
            output_qk_matmul=None, batch=b, q_heads=hq, kv_heads=hkv, q_seq=tq, kv_seq=tkv, total_seq=tkv,
            past_seq=0, qk_head_size=d, v_head_size=dv, scale=scale, is_causal=bool(a.get("is_causal", 0)),
            softcap=float(a.get("softcap", 0.0)), q_rank=4, head_group_size=hq // hkv, dtype=dtypes[ins[0]])
    if op == "LSTM":
        t, b, i = shapes[ins[0]]
        h = int(a["hidden_size"])
        outs = list(node.outputs) + [""] * (3 - len(node.outputs))
        for name, shp in zip(outs, [(t, 1, b, h), (1, b, h), (1, b, h)]):
            if name:
                shapes[name] = shp
                dtypes[name] = dtypes[ins[0]]
        return LstmOp(
            input_x=ins[0], input_w=ins[1], input_r=ins[2], input_b=ins[3] if len(ins) > 3 and ins[3] else None,
            input_sequence_lens=None, input_initial_h=None, input_initial_c=None, input_p=None,
            output_y=outs[0] or None, output_y_h=outs[1] or None, output_y_c=outs[2] or None, seq_length=t,
            batch_size=b, input_size=i, hidden_size=h, num_directions=1,
            direction=str(a.get("direction", "forward")), layout=int(a.get("layout", 0)),
            input_forget=int(a.get("input_forget", 0)), clip=a.get("clip"), activation_kinds=(2, 1, 1),
            dtype=dtypes[ins[0]])
    if op == "Reshape":
        shape_name = ins[1]
        target = list(int(v) for v in np.asarray(_initializer(shape_name)).reshape(-1))
        src = shapes[ins[0]]
        out = [src[i] if v == 0 and not int(a.get("allowzero", 0)) else v for i, v in enumerate(target)]
        if -1 in out:
            known = int(np.prod([v for v in out if v != -1]))
            out[out.index(-1)] = int(np.prod(src)) // max(known, 1)
        y = node.outputs[0]
        shapes[y] = tuple(out)
        dtypes[y] = dtypes[ins[0]]
        return ReshapeOp(input0=ins[0], output=y)
    if op == "Transpose":
        src = shapes[ins[0]]
        perm = tuple(int(v) for v in a.get("perm", list(range(len(src)))[::-1]))
        y = node.outputs[0]
        shapes[y] = tuple(src[p_] for p_ in perm)
        dtypes[y] = dtypes[ins[0]]
        return TransposeOp(input0=ins[0], output=y, perm=perm)
    if op in ("MaxPool", "QLinearAveragePool"):
        x = ins[0]
        n, c, *sp = shapes[x]
        rank = len(sp)
        ks = tuple(int(v) for v in a["kernel_shape"])
        strides = tuple(int(v) for v in a.get("strides", [1] * rank))
        dil = tuple(int(v) for v in a.get("dilations", [1] * rank))
        pads = _auto_pads(a, tuple(sp), ks, strides, dil)
        ceil_mode = bool(int(a.get("ceil_mode", 0)))
        out_sp = tuple(_pool_out(sp[i], ks[i], strides[i], dil[i], pads[i], pads[i + rank], ceil_mode)
                       for i in range(rank))
        y = node.outputs[0]
        shapes[y] = (n, c, *out_sp)
        if op == "MaxPool":
            dtypes[y] = dtypes[x]
            return MaxPoolOp(input0=x, output=y, indices=node.outputs[1] if len(node.outputs) > 1 else None,
                             batch=n, channels=c, spatial_rank=rank, in_spatial=tuple(sp), out_spatial=out_sp,
                             kernel_shape=ks, strides=strides, pads=pads, dilations=dil, ceil_mode=ceil_mode,
                             storage_order=int(a.get("storage_order", 0)), dtype=dtypes[x], indices_dtype=None)
        if rank != 2:
            raise UnsupportedOpError("QLinearAveragePool: only 2-D pooling has a B200 kernel")
        dtypes[y] = dtypes[ins[4]]
        return QLinearAveragePoolOp(
            input0=x, input_scale=ins[1], input_zero_point=ins[2], output_scale=ins[3], output_zero_point=ins[4],
            output=y, batch=n, channels=c, in_h=sp[0], in_w=sp[1], out_h=out_sp[0], out_w=out_sp[1],
            kernel_h=ks[0], kernel_w=ks[1], dilation_h=dil[0], dilation_w=dil[1], stride_h=strides[0],
            stride_w=strides[1], pad_top=pads[0], pad_left=pads[1], pad_bottom=pads[2], pad_right=pads[3],
            count_include_pad=bool(int(a.get("count_include_pad", 0))), input_dtype=dtypes[x], dtype=dtypes[y],
            input_scale_dtype=dtypes[ins[1]], output_scale_dtype=dtypes[ins[3]],
            input_scale_shape=shapes[ins[1]], output_scale_shape=shapes[ins[3]],
            input_zero_shape=shapes[ins[2]], output_zero_shape=shapes[ins[4]],
            channels_last=bool(int(a.get("channels_last", 0))))
    if op == "QLinearSoftmax":
        src = shapes[ins[0]]
        opset = int(a["opset"]) if "opset" in a else int(_INITS["__opset__"])
        legacy = opset < 13
        axis = int(a["axis"]) if "axis" in a else (1 if legacy else -1)
        if axis < 0:
            axis += len(src)
        outer = int(np.prod(src[:axis], dtype=np.int64))
        if legacy:
            axis_size, inner = int(np.prod(src[axis:], dtype=np.int64)), 1
        else:
            axis_size, inner = src[axis], int(np.prod(src[axis + 1:], dtype=np.int64))
        y = node.outputs[0]
        shapes[y] = src
        dtypes[y] = dtypes[ins[4]]
        return QLinearSoftmaxOp(
            input0=ins[0], input_scale=ins[1], input_zero_point=ins[2], output_scale=ins[3],
            output_zero_point=ins[4], output=y, input_shape=src, output_shape=src, axis=axis, outer=outer,
            axis_size=axis_size, inner=inner, dtype=dtypes[y], input_dtype=dtypes[ins[0]],
            input_scale_dtype=dtypes[ins[1]], output_scale_dtype=dtypes[ins[3]])
    raise UnsupportedOpError(f"{op} has no B200 kernel")

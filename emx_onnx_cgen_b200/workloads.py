"""The five graphs this backend is measured on, as seeded synthetic ONNX graphs.

Each builder returns a ``GraphSpec`` whose weights are drawn from
``numpy.random.default_rng(weight_seed)`` and an ``inputs(seed)`` function
that draws the graph inputs from ``default_rng(seed)``.  Sizes are parameters
so the same graph runs at full size (benchmark) and at slices the CPU oracle
finishes in seconds (parity tests).  Distributions follow the workload
definitions:

* ``mlp_fp32``           Gemm(transB) -> Relu -> Gemm(transB), fp32, opset 17
* ``qconv_stack_int8``   4 x QLinearConv 3x3 (64->64) with a com.microsoft
                         QLinearAdd residual after every second conv
* ``llama_mlp_int4``     com.microsoft MatMulNBits gate/up -> Swish(gate)*up ->
                         MatMulNBits down, fp16 activations, int4 weights
* ``attention_fp16``     opset-23 Attention, causal, fp16
* ``lstm_fp32``          ONNX LSTM, forward, fp32

No public dataset is involved; all inputs are synthetic.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import numpy as np

from .spec import GraphSpec, NodeSpec, TensorSpec


@dataclass
class Workload:
    name: str
    graph: GraphSpec
    make_inputs: Callable[[int], dict[str, np.ndarray]]
    batch_axis: dict[str, int]          # graph input/output name -> axis of independent rows
    params: dict[str, object]


def _scalar(value, dtype) -> np.ndarray:
    return np.asarray(value, dtype=dtype).reshape(())


# --------------------------------------------------------------------------- cfg 1
def mlp_fp32(m: int = 64, k: int = 1024, hidden: int = 4096, weight_seed: int = 1) -> Workload:
    rng = np.random.default_rng(weight_seed)
    w1 = rng.normal(0.0, 1.0 / np.sqrt(k), (hidden, k)).astype(np.float32)
    b1 = rng.uniform(-0.1, 0.1, hidden).astype(np.float32)
    w2 = rng.normal(0.0, 1.0 / np.sqrt(hidden), (k, hidden)).astype(np.float32)
    b2 = rng.uniform(-0.1, 0.1, k).astype(np.float32)
    g = GraphSpec(
        name="mlp_fp32",
        inputs=[TensorSpec("X", "f32", (m, k))],
        outputs=[TensorSpec("Y", "f32", (m, k))],
        nodes=[
            NodeSpec("Gemm", "gemm1", ("X", "W1", "b1"), ("H",), {"transB": 1}),
            NodeSpec("Relu", "relu", ("H",), ("R",)),
            NodeSpec("Gemm", "gemm2", ("R", "W2", "b2"), ("Y",), {"transB": 1}),
        ],
        initializers={"W1": w1, "b1": b1, "W2": w2, "b2": b2},
        values=[TensorSpec("H", "f32", (m, hidden)), TensorSpec("R", "f32", (m, hidden))],
        opset_imports=(("", 17),),
    )

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        r = np.random.default_rng(seed)
        return {"X": r.uniform(-1.0, 1.0, (m, k)).astype(np.float32)}

    return Workload("mlp_fp32", g, make_inputs, {"X": 0, "Y": 0},
                    dict(m=m, k=k, hidden=hidden))


# --------------------------------------------------------------------------- cfg 2
def qconv_stack_int8(batch: int = 32, channels: int = 64, height: int = 56, width: int = 56,
                     n_convs: int = 4, wscale_range: tuple[float, float] = (0.001, 0.01),
                     weight_seed: int = 1) -> Workload:
    """uint8 NCHW activations, per-tensor scale 0.02 / zero point 128 at the input.

    Every QLinearConv has int8 OIHW weights ~U(-127,127), per-output-channel
    fp32 scales ~U(wscale_range), weight zero point 0, int32 bias
    ~U(-1000,1000) and output scale 0.02 / zero point 0 (the ReLU folded into
    the output zero point and the uint8 clamp).  After every second conv a
    com.microsoft QLinearAdd adds the block input back in (output scale 0.04,
    zero point 128); the last add is the graph output.
    """
    rng = np.random.default_rng(weight_seed)
    c = channels
    inits: dict[str, np.ndarray] = {
        "x_scale": _scalar(0.02, np.float32),
        "x_zero": _scalar(128, np.uint8),
        "h_scale": _scalar(0.02, np.float32),
        "h_zero": _scalar(0, np.uint8),
        "a_scale": _scalar(0.04, np.float32),
        "a_zero": _scalar(128, np.uint8),
    }
    nodes: list[NodeSpec] = []
    values: list[TensorSpec] = []
    shape = (batch, c, height, width)
    cur, cur_scale, cur_zero = "X", "x_scale", "x_zero"
    block_in, block_scale, block_zero = cur, cur_scale, cur_zero
    for i in range(n_convs):
        inits[f"w{i}"] = rng.integers(-127, 128, (c, c, 3, 3)).astype(np.int8)
        inits[f"ws{i}"] = rng.uniform(wscale_range[0], wscale_range[1], c).astype(np.float32)
        inits[f"wz{i}"] = np.zeros(c, np.int8)
        inits[f"b{i}"] = rng.integers(-1000, 1001, c).astype(np.int32)
        out = f"H{i}"
        nodes.append(NodeSpec(
            "QLinearConv", f"conv{i}",
            (cur, cur_scale, cur_zero, f"w{i}", f"ws{i}", f"wz{i}", "h_scale", "h_zero", f"b{i}"),
            (out,), {"kernel_shape": [3, 3], "pads": [1, 1, 1, 1], "strides": [1, 1]}))
        values.append(TensorSpec(out, "u8", shape))
        cur, cur_scale, cur_zero = out, "h_scale", "h_zero"
        if i % 2 == 1:
            last = i == n_convs - 1
            aout = "Y" if last else f"A{i}"
            nodes.append(NodeSpec(
                "QLinearAdd", f"add{i}",
                (cur, cur_scale, cur_zero, block_in, block_scale, block_zero, "a_scale", "a_zero"),
                (aout,), {}, "com.microsoft"))
            if not last:
                values.append(TensorSpec(aout, "u8", shape))
            cur, cur_scale, cur_zero = aout, "a_scale", "a_zero"
            block_in, block_scale, block_zero = cur, cur_scale, cur_zero
    if n_convs % 2 == 1:   # odd stack: the last conv is the output
        nodes[-1] = NodeSpec(nodes[-1].op_type, nodes[-1].name, nodes[-1].inputs, ("Y",),
                             nodes[-1].attrs)
        values = [v for v in values if v.name != cur]
    g = GraphSpec(
        name="qconv_stack_int8",
        inputs=[TensorSpec("X", "u8", shape)],
        outputs=[TensorSpec("Y", "u8", shape)],
        nodes=nodes, initializers=inits, values=values,
        opset_imports=(("", 17), ("com.microsoft", 1)),
    )

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        r = np.random.default_rng(seed)
        return {"X": r.integers(0, 256, shape).astype(np.uint8)}

    return Workload("qconv_stack_int8", g, make_inputs, {"X": 0, "Y": 0},
                    dict(batch=batch, channels=c, height=height, width=width, n_convs=n_convs,
                         wscale_range=tuple(wscale_range)))


# --------------------------------------------------------------------------- cfg 3
def llama_mlp_int4(m: int = 2048, hidden: int = 4096, inter: int = 11008, block: int = 32,
                   weight_seed: int = 1) -> Workload:
    """fp16 activations ~N(0,1); uint4 weights ~U(0,15) in blocks of 32 along K.

    Scales fp16 ~U(0.005, 0.02); no zero-point input (the default zero point
    8 of MatMulNBits applies); accuracy_level 0.  SiLU(gate)*up is expressed
    as Swish(alpha=1) followed by Mul.
    """
    rng = np.random.default_rng(weight_seed)

    def nbits(prefix: str, k: int, n: int) -> dict[str, np.ndarray]:
        nb = -(-k // block)  # n_blocks_per_col = ceil(K / block_size)
        return {
            f"{prefix}_B": rng.integers(0, 256, (n, nb, block // 2)).astype(np.uint8),
            f"{prefix}_s": rng.uniform(0.005, 0.02, (n, nb)).astype(np.float16),
        }

    inits = {**nbits("gate", hidden, inter), **nbits("up", hidden, inter), **nbits("down", inter, hidden)}

    def mm(name, a, out, k, n):
        return NodeSpec("MatMulNBits", name, (a, f"{name}_B", f"{name}_s"), (out,),
                        {"bits": 4, "block_size": block, "K": k, "N": n, "accuracy_level": 0},
                        "com.microsoft")

    nodes = [
        mm("gate", "A", "G", hidden, inter),
        mm("up", "A", "U", hidden, inter),
        NodeSpec("Swish", "silu", ("G",), ("S",), {"alpha": 1.0}),
        NodeSpec("Mul", "mul", ("S", "U"), ("P",)),
        mm("down", "P", "Y", inter, hidden),
    ]
    values = [TensorSpec(n, "f16", (m, inter)) for n in ("G", "U", "S", "P")]
    g = GraphSpec(
        name="llama_mlp_int4",
        inputs=[TensorSpec("A", "f16", (m, hidden))],
        outputs=[TensorSpec("Y", "f16", (m, hidden))],
        nodes=nodes, initializers=inits, values=values,
        opset_imports=(("", 24), ("com.microsoft", 1)),
    )

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        r = np.random.default_rng(seed)
        return {"A": r.standard_normal((m, hidden)).astype(np.float16)}

    return Workload("llama_mlp_int4", g, make_inputs, {"A": 0, "Y": 0},
                    dict(m=m, hidden=hidden, inter=inter, block=block))


# --------------------------------------------------------------------------- cfg 4
def attention_fp16(batch: int = 8, heads: int = 32, seq: int = 2048, head_dim: int = 128,
                   causal: bool = True) -> Workload:
    shape = (batch, heads, seq, head_dim)
    g = GraphSpec(
        name="attention_fp16",
        inputs=[TensorSpec(n, "f16", shape) for n in ("Q", "K", "V")],
        outputs=[TensorSpec("Y", "f16", shape)],
        nodes=[NodeSpec("Attention", "attn", ("Q", "K", "V"), ("Y",),
                        {"is_causal": 1 if causal else 0})],
        initializers={},
        opset_imports=(("", 23),),
    )

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        r = np.random.default_rng(seed)
        return {n: r.standard_normal(shape).astype(np.float16) for n in ("Q", "K", "V")}

    return Workload("attention_fp16", g, make_inputs, {"Q": 0, "K": 0, "V": 0, "Y": 0},
                    dict(batch=batch, heads=heads, seq=seq, head_dim=head_dim, causal=causal))


# --------------------------------------------------------------------------- cfg 5
def lstm_fp32(seq: int = 512, batch: int = 256, input_size: int = 512, hidden: int = 1024,
              weight_seed: int = 1) -> Workload:
    rng = np.random.default_rng(weight_seed)
    w = rng.uniform(-1 / 32, 1 / 32, (1, 4 * hidden, input_size)).astype(np.float32)
    r = rng.uniform(-1 / 32, 1 / 32, (1, 4 * hidden, hidden)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, (1, 8 * hidden)).astype(np.float32)
    g = GraphSpec(
        name="lstm_fp32",
        inputs=[TensorSpec("X", "f32", (seq, batch, input_size))],
        outputs=[TensorSpec("Y", "f32", (seq, 1, batch, hidden)),
                 TensorSpec("Y_h", "f32", (1, batch, hidden)),
                 TensorSpec("Y_c", "f32", (1, batch, hidden))],
        nodes=[NodeSpec("LSTM", "lstm", ("X", "W", "R", "B"), ("Y", "Y_h", "Y_c"),
                        {"hidden_size": hidden})],
        initializers={"W": w, "R": r, "B": b},
        opset_imports=(("", 22),),
    )

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        rr = np.random.default_rng(seed)
        return {"X": rr.uniform(-1.0, 1.0, (seq, batch, input_size)).astype(np.float32)}

    return Workload("lstm_fp32", g, make_inputs, {"X": 1, "Y": 2, "Y_h": 1, "Y_c": 1},
                    dict(seq=seq, batch=batch, input_size=input_size, hidden=hidden))


# --------------------------------------------------------------------------- single ops
def matmul_nbits_f16(m: int = 64, k: int = 256, n: int = 192, block: int = 32, zero_points: str = "none",
                     bias: bool = False, weight_seed: int = 1, accuracy_level: int = 0) -> Workload:
    """One com.microsoft MatMulNBits (bits 4) on fp16 activations ~N(0,1).

    accuracy_level 4 selects the int8 activation path (activations quantised
    per row and K block, exact int32 block sums).

    zero_points: "none" (default zero point 8), "block" (uint8 [N][ceil(n_blocks/2)],
    4-bit packed per block) or "column" (uint8 [N], one per column).  Optional
    fp16 bias [N] ~U(-1, 1); scales fp16 [N][n_blocks] ~U(0.005, 0.02).
    """
    if zero_points not in ("none", "block", "column"):
        raise ValueError(f"zero_points must be 'none', 'block' or 'column', not {zero_points!r}")
    rng = np.random.default_rng(weight_seed)
    nb = -(-k // block)
    inits = {"B": rng.integers(0, 256, (n, nb, block // 2)).astype(np.uint8),
             "scales": rng.uniform(0.005, 0.02, (n, nb)).astype(np.float16)}
    ins = ["A", "B", "scales"]
    if zero_points == "block":
        inits["zp"] = rng.integers(0, 256, (n, (nb + 1) // 2)).astype(np.uint8)
    elif zero_points == "column":
        inits["zp"] = rng.integers(0, 16, (n,)).astype(np.uint8)
    if zero_points != "none":
        ins.append("zp")
    if bias:
        inits["bias"] = rng.uniform(-1.0, 1.0, (n,)).astype(np.float16)
        ins += [""] * (5 - len(ins)) + ["bias"]
    g = GraphSpec(
        name="matmul_nbits_f16",
        inputs=[TensorSpec("A", "f16", (m, k))],
        outputs=[TensorSpec("Y", "f16", (m, n))],
        nodes=[NodeSpec("MatMulNBits", "mm", tuple(ins), ("Y",),
                        {"bits": 4, "block_size": block, "K": k, "N": n, "accuracy_level": accuracy_level},
                        "com.microsoft")],
        initializers=inits,
        opset_imports=(("", 21), ("com.microsoft", 1)),
    )

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        return {"A": np.random.default_rng(seed).standard_normal((m, k)).astype(np.float16)}

    return Workload("matmul_nbits_f16", g, make_inputs, {"A": 0, "Y": 0},
                    dict(m=m, k=k, n=n, block=block, zero_points=zero_points, bias=bias,
                         accuracy_level=accuracy_level))


def swish_mul_f16(shape: tuple[int, ...] = (256, 512), alpha: float = 1.0) -> Workload:
    """Swish(X, alpha) * Z on fp16 tensors (the unfused element-wise kernels)."""
    g = GraphSpec(
        name="swish_mul_f16",
        inputs=[TensorSpec("X", "f16", tuple(shape)), TensorSpec("Z", "f16", tuple(shape))],
        outputs=[TensorSpec("S", "f16", tuple(shape)), TensorSpec("P", "f16", tuple(shape))],
        nodes=[NodeSpec("Swish", "silu", ("X",), ("S",), {"alpha": alpha}),
               NodeSpec("Mul", "mul", ("S", "Z"), ("P",))],
        initializers={},
        opset_imports=(("", 24),),
    )

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        r = np.random.default_rng(seed)
        return {"X": (4 * r.standard_normal(shape)).astype(np.float16),
                "Z": r.standard_normal(shape).astype(np.float16)}

    return Workload("swish_mul_f16", g, make_inputs, {"X": 0, "Z": 0, "S": 0, "P": 0},
                    dict(shape=tuple(shape), alpha=alpha))


def qlinear_matmul_u8(m: int = 64, k: int = 256, n: int = 128, a_zero: int = 128, b_dtype: str = "i8",
                      b_zero: int = 0, scales: tuple[float, float, float] = (0.02, 0.005, 0.5),
                      weight_seed: int = 1) -> Workload:
    """QLinearMatMul: uint8 A [m,k], int8/uint8 B [k,n] initializer, uint8 output (zero point
    10); scales (a, b, y) per tensor -- powers of two make the multiplier exact, which selects
    the reference's integer requantisation."""
    rng = np.random.default_rng(weight_seed)
    npt = np.int8 if b_dtype == "i8" else np.uint8
    lo, hi = (-127, 128) if b_dtype == "i8" else (0, 256)
    inits = {"B": rng.integers(lo, hi, (k, n)).astype(npt),
             "a_s": _scalar(scales[0], np.float32), "a_z": _scalar(a_zero, np.uint8),
             "b_s": _scalar(scales[1], np.float32), "b_z": _scalar(b_zero, npt),
             "y_s": _scalar(scales[2], np.float32), "y_z": _scalar(10, np.uint8)}
    g = GraphSpec(
        name="qlinear_matmul_u8",
        inputs=[TensorSpec("A", "u8", (m, k))],
        outputs=[TensorSpec("Y", "u8", (m, n))],
        nodes=[NodeSpec("QLinearMatMul", "qmm", ("A", "a_s", "a_z", "B", "b_s", "b_z", "y_s", "y_z"), ("Y",))],
        initializers=inits, opset_imports=(("", 10),),
    )

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        return {"A": np.random.default_rng(seed).integers(0, 256, (m, k)).astype(np.uint8)}

    return Workload("qlinear_matmul_u8", g, make_inputs, {"A": 0, "Y": 0},
                    dict(m=m, k=k, n=n, a_zero=a_zero, b_dtype=b_dtype, b_zero=b_zero, scales=tuple(scales)))


def matmul_integer_u8(m: int = 64, k: int = 256, n: int = 128, a_zero: int = 128, b_zero: int = 3,
                      weight_seed: int = 1) -> Workload:
    """MatMulInteger: uint8 A [m,k], int8 B [k,n] initializer, scalar zero points, int32 output."""
    rng = np.random.default_rng(weight_seed)
    inits = {"B": rng.integers(-127, 128, (k, n)).astype(np.int8),
             "a_z": _scalar(a_zero, np.uint8), "b_z": _scalar(b_zero, np.int8)}
    g = GraphSpec(
        name="matmul_integer_u8",
        inputs=[TensorSpec("A", "u8", (m, k))],
        outputs=[TensorSpec("Y", "i32", (m, n))],
        nodes=[NodeSpec("MatMulInteger", "mmi", ("A", "B", "a_z", "b_z"), ("Y",))],
        initializers=inits, opset_imports=(("", 10),),
    )

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        return {"A": np.random.default_rng(seed).integers(0, 256, (m, k)).astype(np.uint8)}

    return Workload("matmul_integer_u8", g, make_inputs, {"A": 0, "Y": 0}, dict(m=m, k=k, n=n))


def conv_f32(batch: int = 2, cin: int = 8, cout: int = 16, h: int = 12, w: int = 12, kernel: int = 3,
             stride: int = 1, pad: int = 1, dilation: int = 1, group: int = 1, weight_seed: int = 1) -> Workload:
    """fp32 Conv 2-D with bias."""
    rng = np.random.default_rng(weight_seed)
    inits = {"W": rng.standard_normal((cout, cin // group, kernel, kernel)).astype(np.float32) * np.float32(0.1),
             "bias": rng.uniform(-0.1, 0.1, cout).astype(np.float32)}
    oh = (h + 2 * pad - dilation * (kernel - 1) - 1) // stride + 1
    ow = (w + 2 * pad - dilation * (kernel - 1) - 1) // stride + 1
    g = GraphSpec(
        name="conv_f32",
        inputs=[TensorSpec("X", "f32", (batch, cin, h, w))],
        outputs=[TensorSpec("Y", "f32", (batch, cout, oh, ow))],
        nodes=[NodeSpec("Conv", "conv", ("X", "W", "bias"), ("Y",),
                        {"kernel_shape": [kernel, kernel], "pads": [pad] * 4, "strides": [stride] * 2,
                         "dilations": [dilation] * 2, "group": group})],
        initializers=inits, opset_imports=(("", 17),),
    )

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        return {"X": np.random.default_rng(seed).standard_normal((batch, cin, h, w)).astype(np.float32)}

    return Workload("conv_f32", g, make_inputs, {"X": 0, "Y": 0},
                    dict(batch=batch, cin=cin, cout=cout, h=h, w=w, kernel=kernel, stride=stride, pad=pad,
                         dilation=dilation, group=group))


def softmax_f32(shape: tuple[int, ...] = (32, 1000), axis: int = -1) -> Workload:
    """Softmax over one axis, fp32 inputs ~N(0, 4)."""
    g = GraphSpec(
        name="softmax_f32",
        inputs=[TensorSpec("X", "f32", tuple(shape))],
        outputs=[TensorSpec("Y", "f32", tuple(shape))],
        nodes=[NodeSpec("Softmax", "sm", ("X",), ("Y",), {"axis": axis})],
        initializers={}, opset_imports=(("", 13),),
    )

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        return {"X": (2 * np.random.default_rng(seed).standard_normal(shape)).astype(np.float32)}

    return Workload("softmax_f32", g, make_inputs, {"X": 0, "Y": 0}, dict(shape=tuple(shape), axis=axis))


def quant_dequant(shape: tuple[int, ...] = (16, 64), out_dtype: str = "u8", zero: int = 7,
                  scale: float = 0.03) -> Workload:
    """QuantizeLinear (fp32 -> u8/i8, per-tensor scale and zero point) followed by
    DequantizeLinear back to fp32; both results are graph outputs."""
    npt = np.uint8 if out_dtype == "u8" else np.int8
    inits = {"s": _scalar(scale, np.float32), "z": _scalar(zero, npt)}
    g = GraphSpec(
        name="quant_dequant",
        inputs=[TensorSpec("X", "f32", tuple(shape))],
        outputs=[TensorSpec("Q", out_dtype, tuple(shape)), TensorSpec("D", "f32", tuple(shape))],
        nodes=[NodeSpec("QuantizeLinear", "q", ("X", "s", "z"), ("Q",)),
               NodeSpec("DequantizeLinear", "dq", ("Q", "s", "z"), ("D",))],
        initializers=inits, opset_imports=(("", 13),),
    )

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        return {"X": (3 * np.random.default_rng(seed).standard_normal(shape)).astype(np.float32)}

    return Workload("quant_dequant", g, make_inputs, {"X": 0, "Q": 0, "D": 0},
                    dict(shape=tuple(shape), out_dtype=out_dtype, zero=zero, scale=scale))


def _bytes(rng, shape, dtype: str) -> np.ndarray:
    """8-bit tensor uniform over its whole range."""
    lo, hi = (-128, 128) if dtype == "i8" else (0, 256)
    return rng.integers(lo, hi, size=shape).astype(np.int8 if dtype == "i8" else np.uint8)


def pool8(shape: tuple[int, ...] = (2, 8, 13, 11), kind: str = "max", kernel: tuple[int, int] = (3, 2),
          strides: tuple[int, int] = (2, 1), pads: tuple[int, ...] = (1, 0, 1, 1), dilations: tuple[int, int] = (1, 1),
          ceil_mode: int = 0, count_include_pad: int = 0, auto_pad: str | None = None, dtype: str = "i8",
          y_dtype: str | None = None, x_scale: float = 0.05, x_zero: int = -3, y_scale: float = 0.04,
          y_zero: int = 5) -> Workload:
    """One 2-D pooling node on an 8-bit NCHW tensor: MaxPool (kind "max") or
    com.microsoft QLinearAveragePool (kind "avg", per-tensor scales and zero
    points)."""
    from .lowering import _auto_pads, _pool_out
    y_dtype = y_dtype or dtype
    attrs = {"kernel_shape": list(kernel), "strides": list(strides)}
    if auto_pad:
        attrs["auto_pad"] = auto_pad
    else:
        attrs["pads"] = list(pads)
    if tuple(dilations) != (1, 1):
        attrs["dilations"] = list(dilations)
    if ceil_mode:
        attrs["ceil_mode"] = 1
    pd = _auto_pads(attrs, shape[2:], kernel, strides, dilations)
    out = (shape[0], shape[1], *(_pool_out(shape[2 + i], kernel[i], strides[i], dilations[i], pd[i], pd[i + 2],
                                           bool(ceil_mode)) for i in range(2)))
    npt = lambda d: np.int8 if d == "i8" else np.uint8
    if kind == "max":
        node = NodeSpec("MaxPool", "pool", ("X",), ("Y",), attrs)
        inits, y_dtype = {}, dtype
    else:
        if count_include_pad:
            attrs["count_include_pad"] = 1
        inits = {"xs": _scalar(x_scale, np.float32), "xz": _scalar(x_zero, npt(dtype)),
                 "ys": _scalar(y_scale, np.float32), "yz": _scalar(y_zero, npt(y_dtype))}
        node = NodeSpec("QLinearAveragePool", "pool", ("X", "xs", "xz", "ys", "yz"), ("Y",), attrs, "com.microsoft")
    g = GraphSpec(name=f"{kind}pool8", inputs=[TensorSpec("X", dtype, tuple(shape))],
                  outputs=[TensorSpec("Y", y_dtype, out)], nodes=[node], initializers=inits,
                  opset_imports=(("", 13), ("com.microsoft", 1)))

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        return {"X": _bytes(np.random.default_rng(seed), shape, dtype)}

    return Workload(f"{kind}pool8", g, make_inputs, {"X": 0, "Y": 0}, dict(shape=tuple(shape), kind=kind))


def qlinear_softmax8(shape: tuple[int, ...] = (6, 37), axis: int = -1, dtype: str = "u8", x_scale: float = 0.08,
                     x_zero: int = 128, y_scale: float = 1.0 / 256, y_zero: int = 0, opset: int = 13) -> Workload:
    """com.microsoft QLinearSoftmax on an 8-bit tensor (opset < 13: the
    flattened [outer, rest] semantics)."""
    npt = np.int8 if dtype == "i8" else np.uint8
    inits = {"xs": _scalar(x_scale, np.float32), "xz": _scalar(x_zero, npt), "ys": _scalar(y_scale, np.float32),
             "yz": _scalar(y_zero, npt)}
    g = GraphSpec(name="qlinear_softmax8", inputs=[TensorSpec("X", dtype, tuple(shape))],
                  outputs=[TensorSpec("Y", dtype, tuple(shape))],
                  nodes=[NodeSpec("QLinearSoftmax", "sm", ("X", "xs", "xz", "ys", "yz"), ("Y",),
                                  {"axis": axis, "opset": opset}, "com.microsoft")],
                  initializers=inits, opset_imports=(("", 13), ("com.microsoft", 1)))

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        return {"X": _bytes(np.random.default_rng(seed), shape, dtype)}

    return Workload("qlinear_softmax8", g, make_inputs, {"X": 0, "Y": 0}, dict(shape=tuple(shape), axis=axis))


def transpose(shape: tuple[int, ...] = (2, 3, 4, 5), perm: tuple[int, ...] = (0, 2, 3, 1),
              dtype: str = "f32") -> Workload:
    """Transpose of one tensor (Y = X.transpose(perm)), any element type."""
    out = tuple(shape[p] for p in perm)
    g = GraphSpec(name="transpose", inputs=[TensorSpec("X", dtype, tuple(shape))],
                  outputs=[TensorSpec("Y", dtype, out)],
                  nodes=[NodeSpec("Transpose", "t", ("X",), ("Y",), {"perm": list(perm)})],
                  initializers={}, opset_imports=(("", 13),))

    def make_inputs(seed: int = 0) -> dict[str, np.ndarray]:
        rng = np.random.default_rng(seed)
        if dtype in ("u8", "i8"):
            return {"X": _bytes(rng, shape, dtype)}
        return {"X": rng.standard_normal(shape).astype(np.float16 if dtype == "f16" else np.float32)}

    return Workload("transpose", g, make_inputs, {"X": 0, "Y": 0} if perm[0] == 0 else {},
                    dict(shape=tuple(shape), perm=tuple(perm)))


BUILDERS = {
    "mlp_fp32": mlp_fp32,
    "qconv_stack_int8": qconv_stack_int8,
    "llama_mlp_int4": llama_mlp_int4,
    "attention_fp16": attention_fp16,
    "lstm_fp32": lstm_fp32,
    "matmul_nbits_f16": matmul_nbits_f16,
    "swish_mul_f16": swish_mul_f16,
    "qlinear_matmul_u8": qlinear_matmul_u8,
    "matmul_integer_u8": matmul_integer_u8,
    "conv_f32": conv_f32,
    "softmax_f32": softmax_f32,
    "quant_dequant": quant_dequant,
    "pool8": pool8,
    "qlinear_softmax8": qlinear_softmax8,
    "transpose": transpose,
}

"""TEST INFRASTRUCTURE ONLY: Python driver for the CPU restatement in oracle.c.

``run_graph(spec, inputs)`` executes a ``GraphSpec`` node by node through the
restated reference loop nests (liboracle.so), the way the reference's
generated ``<model>()`` calls one ``nodeN_*`` function per lowered op in graph
order (codegen/c_emitter.py:2297, :2791-2853).  The product never imports
this module.
"""
from __future__ import annotations

import ctypes
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
from emx_onnx_cgen_b200.spec import GraphSpec  # noqa: E402

_LIB: ctypes.CDLL | None = None


def build() -> Path:
    so = HERE / "liboracle.so"
    if not so.exists() or so.stat().st_mtime < (HERE / "oracle.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
    return so


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = ctypes.CDLL(str(build()))
    return _LIB


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


_i, _f, _sz = ctypes.c_int, ctypes.c_float, ctypes.c_size_t


# ------------------------------------------------------------------ op wrappers
def qlinear_conv2d(x, xs, xz, w, ws, wz, ys, yz, bias, strides=(1, 1), pads=(0, 0, 0, 0),
                   dilations=(1, 1), group=1, y_dtype=np.uint8):
    x = np.ascontiguousarray(x); w = np.ascontiguousarray(w)
    n, c, h, wd = x.shape
    oc, _, kh, kw = w.shape
    oh = (h + pads[0] + pads[2] - ((kh - 1) * dilations[0] + 1)) // strides[0] + 1
    ow = (wd + pads[1] + pads[3] - ((kw - 1) * dilations[1] + 1)) // strides[1] + 1
    y = np.zeros((n, oc, oh, ow), dtype=y_dtype)
    ws = np.ascontiguousarray(np.asarray(ws, np.float32).reshape(-1))
    wz32 = None if wz is None else np.ascontiguousarray(np.asarray(wz).astype(np.int32).reshape(-1))
    b = None if bias is None else np.ascontiguousarray(np.asarray(bias, np.int32))
    lib().orc_qlinear_conv2d(
        _p(x), _i(x.dtype == np.int8), _i(n), _i(c), _i(h), _i(wd), _f(float(np.float32(xs))), _i(int(xz)),
        _p(w), _i(w.dtype == np.int8), _i(oc), _i(kh), _i(kw), _p(ws), _i(ws.size > 1),
        _p(wz32), _i(wz32 is not None and wz32.size > 1), _f(float(np.float32(ys))), _i(int(yz)), _p(b),
        _i(strides[0]), _i(strides[1]), _i(pads[0]), _i(pads[1]), _i(dilations[0]), _i(dilations[1]),
        _i(group), _p(y), _i(y.dtype == np.int8), _i(oh), _i(ow))
    return y


def qlinear_add(a, a_s, a_z, b, b_s, b_z, y_s, y_z, y_dtype=np.uint8):
    """Multidirectional broadcast as the reference's loop nest indexes it
    (templates/qlinear_add_op.c.j2): both operands at the output shape."""
    shape = np.broadcast_shapes(a.shape, b.shape)
    a = np.ascontiguousarray(np.broadcast_to(a, shape)); b = np.ascontiguousarray(np.broadcast_to(b, shape))
    y = np.zeros(a.shape, dtype=y_dtype)
    lib().orc_qlinear_add(_p(a), _i(a.dtype == np.int8), _f(float(np.float32(a_s))), _i(int(a_z)),
                          _p(b), _i(b.dtype == np.int8), _f(float(np.float32(b_s))), _i(int(b_z)),
                          _f(float(np.float32(y_s))), _i(int(y_z)), _p(y), _i(y.dtype == np.int8),
                          _sz(a.size))
    return y


def _pool_geometry(x, a):
    """(kernel, strides, dilations, pads, out) of a 2-D pooling node, ONNX rules."""
    ks = [int(v) for v in a["kernel_shape"]]
    st = [int(v) for v in a.get("strides", [1, 1])]
    dl = [int(v) for v in a.get("dilations", [1, 1])]
    mode = a.get("auto_pad", "NOTSET")
    mode = mode.decode() if isinstance(mode, bytes) else str(mode)
    if mode in ("SAME_UPPER", "SAME_LOWER"):
        pd = [0, 0, 0, 0]
        for i in range(2):
            need = max(0, (-(-x.shape[2 + i] // st[i]) - 1) * st[i] + dl[i] * (ks[i] - 1) + 1 - x.shape[2 + i])
            pd[i] = need // 2 if mode == "SAME_UPPER" else (need + 1) // 2
            pd[i + 2] = need - pd[i]
    elif mode == "VALID":
        pd = [0, 0, 0, 0]
    else:
        pd = [int(v) for v in a.get("pads", [0, 0, 0, 0])]
    ceil_mode = bool(int(a.get("ceil_mode", 0)))
    out = []
    for i in range(2):
        span = x.shape[2 + i] + pd[i] + pd[i + 2] - ((ks[i] - 1) * dl[i] + 1)
        o = (-(-span // st[i]) if ceil_mode else span // st[i]) + 1
        if ceil_mode and (o - 1) * st[i] >= x.shape[2 + i] + pd[i]:
            o -= 1
        out.append(o)
    return ks, st, dl, pd, out


def maxpool8(x, a):
    ks, st, dl, pd, (oh, ow) = _pool_geometry(x, a)
    x = np.ascontiguousarray(x)
    n, c, h, w = x.shape
    y = np.zeros((n, c, oh, ow), dtype=x.dtype)
    lib().orc_maxpool8(_p(x), _p(y), _i(x.dtype == np.int8), *(ctypes.c_long(v) for v in
                       (n, c, h, w, oh, ow, ks[0], ks[1], st[0], st[1], dl[0], dl[1], pd[0], pd[1])))
    return y


def qlinear_avgpool8(x, xs, xz, ys, yz, a):
    ks, st, dl, pd, (oh, ow) = _pool_geometry(x, a)
    x = np.ascontiguousarray(x)
    n, c, h, w = x.shape
    y = np.zeros((n, c, oh, ow), dtype=np.asarray(yz).dtype)
    lib().orc_qavgpool8(_p(x), _p(y), _i(x.dtype == np.int8), _i(y.dtype == np.int8),
                        *(ctypes.c_long(v) for v in (n, c, h, w, oh, ow, ks[0], ks[1], st[0], st[1], dl[0], dl[1],
                                                     pd[0], pd[1])),
                        _i(int(a.get("count_include_pad", 0))), _f(float(np.float32(np.asarray(xs).reshape(-1)[0]))),
                        _i(int(np.asarray(xz).reshape(-1)[0])), _f(float(np.float32(np.asarray(ys).reshape(-1)[0]))),
                        _i(int(np.asarray(yz).reshape(-1)[0])))
    return y


def qlinear_softmax8(x, xs, xz, ys, yz, axis, legacy):
    x = np.ascontiguousarray(x)
    ax = axis % x.ndim
    outer = int(np.prod(x.shape[:ax]))
    if legacy:
        n_axis, inner = int(np.prod(x.shape[ax:])), 1
    else:
        n_axis, inner = x.shape[ax], int(np.prod(x.shape[ax + 1:]))
    y = np.zeros(x.shape, dtype=np.asarray(yz).dtype)
    lib().orc_qsoftmax8(_p(x), _p(y), _i(x.dtype == np.int8), _i(y.dtype == np.int8), ctypes.c_long(outer),
                        ctypes.c_long(n_axis), ctypes.c_long(inner),
                        _f(float(np.float32(np.asarray(xs).reshape(-1)[0]))), _i(int(np.asarray(xz).reshape(-1)[0])),
                        _f(float(np.float32(np.asarray(ys).reshape(-1)[0]))), _i(int(np.asarray(yz).reshape(-1)[0])))
    return y


def reshape(x, shape, allowzero=0):
    """templates/reshape_op.c.j2: the same elements in row-major order."""
    tgt = [int(v) for v in np.asarray(shape).reshape(-1)]
    tgt = [x.shape[i] if v == 0 and not allowzero else v for i, v in enumerate(tgt)]
    return np.ascontiguousarray(x).reshape(tgt)


def gemm_f32(a, b, c=None, trans_a=0, trans_b=0, alpha=1.0, beta=1.0):
    a = np.ascontiguousarray(a, np.float32); b = np.ascontiguousarray(b, np.float32)
    m, k = (a.shape[1], a.shape[0]) if trans_a else a.shape
    n = b.shape[0] if trans_b else b.shape[1]
    mode = 0
    if c is not None:
        c = np.ascontiguousarray(c, np.float32)
        if c.size == 1:
            mode = 1
        elif c.ndim == 1 and c.shape[0] == n:
            mode = 2
        elif c.ndim == 2 and c.shape == (1, n):
            mode = 2
        elif c.ndim == 2 and c.shape == (m, 1):
            mode = 3
        else:
            mode = 4
    y = np.zeros((m, n), np.float32)
    lib().orc_gemm_f32(_p(a), _p(b), _p(c), _i(mode), _i(m), _i(n), _i(k), _i(trans_a), _i(trans_b),
                       _f(alpha), _f(beta), _p(y))
    return y


def _unary(fn, x, dtype, *extra):
    x = np.ascontiguousarray(x, dtype)
    y = np.zeros_like(x)
    getattr(lib(), fn)(_p(x), _p(y), _sz(x.size), *extra)
    return y


def _binary(fn, a, b, dtype):
    a = np.ascontiguousarray(a, dtype); b = np.ascontiguousarray(b, dtype)
    assert a.shape == b.shape
    y = np.zeros_like(a)
    getattr(lib(), fn)(_p(a), _p(b), _p(y), _sz(a.size))
    return y


def relu_f32(x): return _unary("orc_relu_f32", x, np.float32)
def sigmoid_f32(x): return _unary("orc_sigmoid_f32", x, np.float32)
def tanh_f32(x): return _unary("orc_tanh_f32", x, np.float32)
def swish_f16(x, alpha=1.0):
    # the generated C declares `const _Float16 alpha = <double literal>;`
    # (shared/scalar_functions.py:880-896): alpha is rounded once to fp16
    return _unary("orc_swish_f16", x, np.float16, _f(float(np.float16(alpha))))
def sigmoid_f16(x): return _unary("orc_sigmoid_f16", x, np.float16)
def mul_f16(a, b): return _binary("orc_mul_f16", a, b, np.float16)
def mul_f32(a, b): return _binary("orc_mul_f32", a, b, np.float32)
def add_f32(a, b): return _binary("orc_add_f32", a, b, np.float32)


def matmul_nbits_f16(a, b_packed, scales, k, n, block=32, zero_points=None, bias=None, accuracy_level=0):
    """accuracy_level 4 selects the reference's int8 activation path."""
    a = np.ascontiguousarray(a, np.float16)
    m = int(np.prod(a.shape[:-1]))
    y = np.zeros((*a.shape[:-1], n), np.float16)
    b_packed = np.ascontiguousarray(b_packed, np.uint8)
    scales_pb = int(np.ndim(scales) >= 2)
    scales = np.ascontiguousarray(scales, np.float16)
    zp_pb = int(zero_points is not None and np.ndim(zero_points) >= 2)
    zp = None if zero_points is None else np.ascontiguousarray(zero_points, np.uint8)
    bias = None if bias is None else np.ascontiguousarray(bias, np.float16)
    fn = lib().orc_matmul_nbits_i8_f16 if int(accuracy_level) == 4 else lib().orc_matmul_nbits_f16
    fn(_p(a), _p(b_packed), _p(scales), _i(scales_pb), _p(zp), _i(zp_pb), _p(bias), _i(m), _i(n), _i(k), _i(block),
       _p(y))
    return y


def attention_f16(q, k, v, scale=None, is_causal=True):
    q = np.ascontiguousarray(q, np.float16); k = np.ascontiguousarray(k, np.float16)
    v = np.ascontiguousarray(v, np.float16)
    b, hq, tq, d = q.shape
    _, hkv, tkv, _ = k.shape
    dv = v.shape[3]
    if scale is None:
        scale = 1.0 / np.sqrt(d)
    out = np.zeros((b, hq, tq, dv), np.float16)
    lib().orc_attention_f16(_p(q), _p(k), _p(v), _p(out), _i(b), _i(hq), _i(hkv), _i(tq), _i(tkv),
                            _i(d), _i(dv), _f(float(scale)), _i(int(bool(is_causal))))
    return out


def lstm_f32(x, w, r, bias):
    x = np.ascontiguousarray(x, np.float32)
    t, b, i = x.shape
    hidden = r.shape[-1]
    y = np.zeros((t, 1, b, hidden), np.float32)
    yh = np.zeros((1, b, hidden), np.float32)
    yc = np.zeros((1, b, hidden), np.float32)
    bias_p = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().orc_lstm_f32(_p(x), _p(np.ascontiguousarray(w, np.float32)), _p(np.ascontiguousarray(r, np.float32)),
                       _p(bias_p), _i(t), _i(b), _i(i), _i(hidden), _p(y), _p(yh), _p(yc))
    return y, yh, yc


# ------------------------------------------------------------------ graph runner
def _u8(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint8), int(a.dtype == np.int8)


def qlinear_matmul(a, sa, za, b, sb, zb, sy, zy):
    a8, a_s = _u8(a)
    b8, b_s = _u8(b)
    m = int(np.prod(a.shape[:-1])) if a.ndim > 1 else 1
    k, n = a.shape[-1], b.shape[1]
    y_signed = int(np.asarray(zy).dtype == np.int8)
    y = np.zeros((*a.shape[:-1], n), np.int8 if y_signed else np.uint8)
    f = lambda v: float(np.asarray(v, np.float32).reshape(-1)[0])
    i = lambda v: int(np.asarray(v).reshape(-1)[0])
    lib().orc_qlinear_matmul(_p(a8), _i(a_s), _p(b8), _i(b_s), _f(f(sa)), _i(i(za)), _f(f(sb)), _i(i(zb)),
                             _f(f(sy)), _i(i(zy)), _i(y_signed), _i(m), _i(k), _i(n), _p(y.view(np.uint8)))
    return y


def matmul_integer(a, b, za=None, zb=None):
    a8, a_s = _u8(a)
    b8, b_s = _u8(b)
    m = int(np.prod(a.shape[:-1])) if a.ndim > 1 else 1
    k, n = a.shape[-1], b.shape[1]
    y = np.zeros((*a.shape[:-1], n), np.int32)
    i = lambda v: 0 if v is None else int(np.asarray(v).reshape(-1)[0])
    lib().orc_matmul_integer(_p(a8), _i(a_s), _p(b8), _i(b_s), _i(i(za)), _i(i(zb)), _i(m), _i(k), _i(n), _p(y))
    return y


def conv2d_f32(x, w, bias, strides, pads, dilations, group):
    x = np.ascontiguousarray(x, np.float32); w = np.ascontiguousarray(w, np.float32)
    n, c, h, wd = x.shape
    oc, _, kh, kw = w.shape
    oh = (h + pads[0] + pads[2] - ((kh - 1) * dilations[0] + 1)) // strides[0] + 1
    ow = (wd + pads[1] + pads[3] - ((kw - 1) * dilations[1] + 1)) // strides[1] + 1
    y = np.zeros((n, oc, oh, ow), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().orc_conv2d_f32(_p(x), _p(w), _p(b), _i(n), _i(c), _i(h), _i(wd), _i(oc), _i(kh), _i(kw),
                         _i(strides[0]), _i(strides[1]), _i(pads[0]), _i(pads[1]), _i(dilations[0]),
                         _i(dilations[1]), _i(group), _i(oh), _i(ow), _p(y))
    return y


def softmax_f32(x, axis=-1):
    x = np.ascontiguousarray(x, np.float32)
    ax = axis % x.ndim
    outer = int(np.prod(x.shape[:ax])); inner = int(np.prod(x.shape[ax + 1:]))
    y = np.zeros_like(x)
    lib().orc_softmax_f32(_p(x), _p(y), ctypes.c_long(outer), ctypes.c_long(x.shape[ax]), ctypes.c_long(inner))
    return y


def _axis_split(shape, scale, axis):
    if np.asarray(scale).size == 1:
        return int(np.prod(shape)), 1, 1
    ax = (1 if axis is None else axis) % len(shape)
    return int(np.prod(shape[:ax])), shape[ax], int(np.prod(shape[ax + 1:]))


def quantize_linear(x, scale, zp=None, axis=None):
    x = np.ascontiguousarray(x, np.float32)
    sc = np.ascontiguousarray(np.asarray(scale, np.float32).reshape(-1))
    outer, alen, inner = _axis_split(x.shape, sc, axis)
    zdt = np.uint8 if zp is None else np.asarray(zp).dtype
    z8 = None if zp is None else np.ascontiguousarray(np.asarray(zp).reshape(-1)).view(np.uint8)
    y = np.zeros(x.shape, zdt)
    lib().orc_quantize_linear(_p(x), _p(sc), _p(z8), _i(zdt == np.int8), _i(zdt == np.int8), ctypes.c_long(outer),
                              ctypes.c_long(alen), ctypes.c_long(inner), _p(y.view(np.uint8)))
    return y


def dequantize_linear(x, scale, zp=None, axis=None):
    x8, xs = _u8(x)
    sc = np.ascontiguousarray(np.asarray(scale, np.float32).reshape(-1))
    outer, alen, inner = _axis_split(x.shape, sc, axis)
    z8 = None if zp is None else np.ascontiguousarray(np.asarray(zp).reshape(-1)).view(np.uint8)
    y = np.zeros(x.shape, np.float32)
    lib().orc_dequantize_linear(_p(x8), _i(xs), _p(sc), _p(z8), ctypes.c_long(outer), ctypes.c_long(alen),
                                ctypes.c_long(inner), _p(y))
    return y


def run_graph(spec: GraphSpec, inputs: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    env: dict[str, np.ndarray] = dict(spec.initializers)
    env.update(inputs)
    for node in spec.nodes:
        a = node.attrs
        ins = [env[n] if n else None for n in node.inputs]
        op = node.op_type
        if op == "QLinearConv":
            ks = list(a.get("kernel_shape", ins[3].shape[2:]))
            pads = list(a.get("pads", [0, 0, 0, 0]))
            out = qlinear_conv2d(ins[0], ins[1], ins[2], ins[3], ins[4],
                                 ins[5], ins[6], ins[7], ins[8] if len(ins) > 8 else None,
                                 strides=tuple(a.get("strides", [1, 1])), pads=tuple(pads),
                                 dilations=tuple(a.get("dilations", [1, 1])), group=int(a.get("group", 1)),
                                 y_dtype=ins[7].dtype)
            del ks
            res = [out]
        elif op == "QLinearAdd":
            res = [qlinear_add(ins[0], ins[1], ins[2], ins[3], ins[4], ins[5], ins[6], ins[7],
                               y_dtype=ins[7].dtype)]
        elif op == "Gemm":
            res = [gemm_f32(ins[0], ins[1], ins[2] if len(ins) > 2 else None,
                            int(a.get("transA", 0)), int(a.get("transB", 0)),
                            float(a.get("alpha", 1.0)), float(a.get("beta", 1.0)))]
        elif op == "Relu":
            res = [relu_f32(ins[0])]
        elif op == "MatMulNBits":
            res = [matmul_nbits_f16(ins[0], ins[1], ins[2], int(a["K"]), int(a["N"]),
                                    int(a.get("block_size", 32)),
                                    ins[3] if len(ins) > 3 else None,
                                    ins[5] if len(ins) > 5 else None,
                                    int(a.get("accuracy_level", 0)))]
        elif op == "Swish":
            res = [swish_f16(ins[0], float(a.get("alpha", 1.0)))]
        elif op == "Sigmoid":
            res = [sigmoid_f16(ins[0]) if ins[0].dtype == np.float16 else sigmoid_f32(ins[0])]
        elif op == "Mul":
            res = [mul_f16(ins[0], ins[1]) if ins[0].dtype == np.float16 else mul_f32(ins[0], ins[1])]
        elif op == "QLinearMatMul":
            res = [qlinear_matmul(*ins[:8])]
        elif op == "MatMulInteger":
            res = [matmul_integer(ins[0], ins[1], ins[2] if len(ins) > 2 else None,
                                  ins[3] if len(ins) > 3 else None)]
        elif op == "Conv":
            rank = ins[0].ndim - 2
            res = [conv2d_f32(ins[0], ins[1], ins[2] if len(ins) > 2 else None,
                              tuple(a.get("strides", [1] * rank)), tuple(a.get("pads", [0] * 2 * rank)),
                              tuple(a.get("dilations", [1] * rank)), int(a.get("group", 1)))]
        elif op == "Softmax":
            res = [softmax_f32(ins[0], int(a.get("axis", -1)))]
        elif op == "QuantizeLinear":
            res = [quantize_linear(ins[0], ins[1], ins[2] if len(ins) > 2 else None, a.get("axis"))]
        elif op == "DequantizeLinear":
            res = [dequantize_linear(ins[0], ins[1], ins[2] if len(ins) > 2 else None, a.get("axis"))]
        elif op == "Attention":
            res = [attention_f16(ins[0], ins[1], ins[2], a.get("scale"), bool(a.get("is_causal", 0)))]
        elif op == "Reshape":
            res = [reshape(ins[0], ins[1], int(a.get("allowzero", 0)))]
        elif op == "Transpose":
            res = [np.ascontiguousarray(np.transpose(ins[0], a.get("perm")))]
        elif op == "MaxPool":
            res = [maxpool8(ins[0], a)]
        elif op == "QLinearAveragePool":
            res = [qlinear_avgpool8(ins[0], ins[1], ins[2], ins[3], ins[4], a)]
        elif op == "QLinearSoftmax":
            opset = int(a["opset"]) if "opset" in a else dict(spec.opset_imports).get("", 17)
            legacy = opset < 13
            res = [qlinear_softmax8(ins[0], ins[1], ins[2], ins[3], ins[4],
                                    int(a["axis"]) if "axis" in a else (1 if legacy else -1), legacy)]
        elif op == "LSTM":
            res = list(lstm_f32(ins[0], ins[1][0], ins[2][0], ins[3][0] if len(ins) > 3 else None))
        else:
            raise NotImplementedError(op)
        for name, val in zip(node.outputs, res):
            if name:
                env[name] = val
    return {t.name: env[t.name] for t in spec.outputs}

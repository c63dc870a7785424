"""Minimal ONNX model reader without the ``onnx`` package.

Decodes the protobuf wire format of the messages a model file uses --
ModelProto, GraphProto, NodeProto, AttributeProto, TensorProto,
ValueInfoProto/TypeProto/TensorShapeProto, OperatorSetIdProto -- by their
field numbers in the public ``onnx.proto`` (ONNX IR version 10 numbering),
and returns a ``GraphSpec``: typed graph inputs/outputs, intermediate value
types from ``value_info``, initializers as numpy arrays, nodes with decoded
attributes and domains.  ONNX shape inference is not available;
``infer_types`` fills the dtype and static shape of every node output that
``value_info`` leaves untyped, for the operators of the reference's quantised
model fixtures (the role ONNX shape inference plays in the reference's
importer, onnx_import.py:2146-2185).  Symbolic dimensions must be bound by the
caller (``dim_values``): by parameter name (``{"batch": 1}`` fixes every
axis carrying that name) or by position (``{"images:0": 1}`` fixes axis 0 of
value ``images``), the two forms of the reference's ``--input-dim``
(cli.py:992-1001, input_dim_overrides.py).

    spec = infer_types(read_onnx("model.onnx", dim_values={"batch": 32}))
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

from .spec import GraphSpec, NodeSpec, TensorSpec

# TensorProto.DataType -> spec dtype suffix
_DTYPES = {1: "f32", 2: "u8", 3: "i8", 4: "u16", 5: "i16", 6: "i32", 7: "i64", 9: "bool", 10: "f16", 11: "f64",
           12: "u32", 13: "u64"}
_NP = {"f32": np.float32, "u8": np.uint8, "i8": np.int8, "u16": np.uint16, "i16": np.int16, "i32": np.int32,
       "i64": np.int64, "bool": np.bool_, "f16": np.float16, "f64": np.float64, "u32": np.uint32, "u64": np.uint64}


class OnnxFormatError(ValueError):
    pass


# ------------------------------------------------------------------ wire format
def _varint(buf: bytes, pos: int) -> tuple[int, int]:
    result = shift = 0
    while True:
        if pos >= len(buf):
            raise OnnxFormatError("truncated varint")
        b = buf[pos]
        pos += 1
        result |= (b & 0x7F) << shift
        if not b & 0x80:
            return result, pos
        shift += 7
        if shift > 70:
            raise OnnxFormatError("varint too long")


def _fields(buf: bytes):
    """Yield (field number, wire type, value) of one message; value is an int
    for varint/fixed fields and bytes for length-delimited ones."""
    pos = 0
    while pos < len(buf):
        key, pos = _varint(buf, pos)
        num, wt = key >> 3, key & 7
        if wt == 0:
            val, pos = _varint(buf, pos)
        elif wt == 1:
            val = struct.unpack_from("<Q", buf, pos)[0]
            pos += 8
        elif wt == 2:
            ln, pos = _varint(buf, pos)
            val = buf[pos:pos + ln]
            if len(val) != ln:
                raise OnnxFormatError("truncated field")
            pos += ln
        elif wt == 5:
            val = struct.unpack_from("<I", buf, pos)[0]
            pos += 4
        else:
            raise OnnxFormatError(f"unsupported wire type {wt}")
        yield num, wt, val


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= 1 << 63 else v


def _packed_varints(val, wt) -> list[int]:
    if wt == 0:
        return [_signed(val)]
    out, pos = [], 0
    while pos < len(val):
        v, pos = _varint(val, pos)
        out.append(_signed(v))
    return out


def _packed_fixed(val, wt, fmt: str) -> list:
    if wt in (1, 5):
        raw = struct.pack("<Q" if wt == 1 else "<I", val)
        return list(struct.unpack("<" + fmt, raw))
    n = len(val) // struct.calcsize(fmt)
    return list(struct.unpack(f"<{n}{fmt}", val))


# ------------------------------------------------------------------ messages
def _tensor(buf: bytes) -> tuple[str, np.ndarray]:
    dims, dtype, name, raw = [], 0, "", None
    floats, i32s, i64s, doubles, u64s, ext = [], [], [], [], [], False
    for num, wt, val in _fields(buf):
        if num == 1:
            dims += _packed_varints(val, wt)
        elif num == 2:
            dtype = val
        elif num == 4:
            floats += _packed_fixed(val, wt, "f")
        elif num == 5:
            i32s += _packed_varints(val, wt)
        elif num == 7:
            i64s += _packed_varints(val, wt)
        elif num == 8:
            name = val.decode()
        elif num == 9:
            raw = bytes(val)
        elif num == 10:
            doubles += _packed_fixed(val, wt, "d")
        elif num == 11:
            u64s += _packed_varints(val, wt)
        elif num == 14:
            ext = val == 1
    if ext:
        raise OnnxFormatError(f"tensor {name}: external data is not supported")
    if dtype not in _DTYPES:
        raise OnnxFormatError(f"tensor {name}: unsupported data type {dtype}")
    sfx = _DTYPES[dtype]
    npt = _NP[sfx]
    count = int(np.prod(dims)) if dims else 1
    if raw is not None:
        arr = np.frombuffer(raw, dtype=np.dtype(npt).newbyteorder("<")).astype(npt)
    elif sfx == "f32":
        arr = np.array(floats, np.float32)
    elif sfx == "f64":
        arr = np.array(doubles, np.float64)
    elif sfx == "i64":
        arr = np.array(i64s, np.int64)
    elif sfx in ("u64", "u32"):
        arr = np.array(u64s, npt)
    elif sfx == "f16":  # int32_data holds the 16-bit patterns
        arr = np.array(i32s, np.uint16).view(np.float16)
    else:  # int32_data holds 8/16/32-bit integers and bools
        arr = np.array(i32s, np.int64).astype(npt)
    if arr.size != count:
        raise OnnxFormatError(f"tensor {name}: {arr.size} values for shape {dims}")
    return name, arr.reshape(dims)


def _value_info(buf: bytes, dim_values: dict[str, int]) -> TensorSpec | None:
    name, elem, dims, has_shape = "", 0, [], False
    for num, _, val in _fields(buf):
        if num == 1:
            name = val.decode()
        elif num == 2:  # TypeProto
            for tn, _, tv in _fields(val):
                if tn != 1:  # only tensor_type
                    continue
                for n2, _, v2 in _fields(tv):
                    if n2 == 1:
                        elem = v2
                    elif n2 == 2:  # TensorShapeProto
                        has_shape = True
                        for n3, _, v3 in _fields(v2):
                            if n3 != 1:
                                continue
                            dv, dp = None, None
                            for n4, _, v4 in _fields(v3):
                                if n4 == 1:
                                    dv = _signed(v4)
                                elif n4 == 2:
                                    dp = v4.decode()
                            pos = f"{name}:{len(dims)}"
                            if pos in dim_values:
                                dv = dim_values[pos]
                                if dp is not None:  # a named axis pinned by position pins the name too
                                    dim_values.setdefault(dp, dv)
                            elif dv is None:
                                if dp not in dim_values:
                                    raise OnnxFormatError(f"value {name}: symbolic dimension {len(dims)} ({dp!r}) needs a "
                                                          f"value (dim_values[{dp!r}] or [{pos!r}])")
                                dv = dim_values[dp]
                            dims.append(dv)
    if not name or elem not in _DTYPES or not has_shape:
        return None
    return TensorSpec(name, _DTYPES[elem], tuple(dims))


def _attribute(buf: bytes):
    name, kind = "", 0
    f = i = s = t = None
    floats, ints, strings = [], [], []
    for num, wt, val in _fields(buf):
        if num == 1:
            name = val.decode()
        elif num == 2:
            f = _packed_fixed(val, wt, "f")[0]
        elif num == 3:
            i = _signed(val)
        elif num == 4:
            s = bytes(val)
        elif num == 5:
            t = _tensor(val)[1]
        elif num == 7:
            floats += _packed_fixed(val, wt, "f")
        elif num == 8:
            ints += _packed_varints(val, wt)
        elif num == 9:
            strings.append(bytes(val))
        elif num == 20:
            kind = val
    value = {1: f, 2: i, 3: s.decode() if s is not None else None, 4: t, 6: floats, 7: ints,
             8: [x.decode() for x in strings]}.get(kind)
    if kind == 0:  # older writers omit the type: infer from the populated field
        value = next((v for v in (f, i, s.decode() if s is not None else None, t) if v is not None),
                     floats or ints or strings)
    if kind == 5:
        raise OnnxFormatError(f"attribute {name}: graph attributes are not supported")
    return name, value


def _node(buf: bytes) -> NodeSpec:
    ins, outs, name, op, domain, attrs = [], [], "", "", None, {}
    for num, _, val in _fields(buf):
        if num == 1:
            ins.append(val.decode())
        elif num == 2:
            outs.append(val.decode())
        elif num == 3:
            name = val.decode()
        elif num == 4:
            op = val.decode()
        elif num == 5:
            k, v = _attribute(val)
            attrs[k] = v
        elif num == 7:
            domain = val.decode() or None
    return NodeSpec(op, name or f"{op}_{id(buf)}", tuple(ins), tuple(outs), attrs, domain)


def read_onnx_bytes(data: bytes, dim_values: dict[str, int] | None = None) -> GraphSpec:
    dim_values = dict(dim_values or {})
    graph_buf, opsets = None, []
    for num, _, val in _fields(data):
        if num == 7:
            graph_buf = val
        elif num == 8:
            dom, ver = "", 0
            for n2, _, v2 in _fields(val):
                if n2 == 1:
                    dom = v2.decode()
                elif n2 == 2:
                    ver = v2
            opsets.append((dom, ver))
    if graph_buf is None:
        raise OnnxFormatError("model has no graph")
    name, nodes, inits, inputs, outputs, values = "model", [], {}, [], [], []
    for num, _, val in _fields(graph_buf):
        if num == 1:
            nodes.append(_node(val))
        elif num == 2:
            name = val.decode()
        elif num == 5:
            k, arr = _tensor(val)
            inits[k] = arr
        elif num == 11:
            vi = _value_info(val, dim_values)
            if vi is not None:
                inputs.append(vi)
        elif num == 12:
            vi = _value_info(val, dim_values)
            if vi is None:
                raise OnnxFormatError("graph output without a typed shape")
            outputs.append(vi)
        elif num == 13:
            vi = _value_info(val, dim_values)
            if vi is not None:
                values.append(vi)
    inputs = [t for t in inputs if t.name not in inits]
    return GraphSpec(name=name, inputs=inputs, outputs=outputs, nodes=nodes, initializers=inits, values=values,
                     opset_imports=tuple(opsets) or (("", 17),))


def read_onnx(path: str | Path, dim_values: dict[str, int] | None = None) -> GraphSpec:
    return read_onnx_bytes(Path(path).read_bytes(), dim_values)


# ------------------------------------------------------------------ type / shape propagation
def _pool_out(shape, a):
    rank = len(shape) - 2
    ks = list(a.get("kernel_shape"))
    st = list(a.get("strides", [1] * rank))
    dil = list(a.get("dilations", [1] * rank))
    pads = list(a.get("pads", [0] * (2 * rank)))
    if str(a.get("auto_pad", "NOTSET")) not in ("NOTSET", ""):
        raise OnnxFormatError("auto_pad is not supported by the type propagation")
    ceil = int(a.get("ceil_mode", 0))
    out = []
    for i in range(rank):
        span = shape[2 + i] + pads[i] + pads[i + rank] - ((ks[i] - 1) * dil[i] + 1)
        out.append((-(-span // st[i]) if ceil else span // st[i]) + 1)
    return out


def _broadcast(a, b):
    return tuple(np.broadcast_shapes(tuple(a), tuple(b)))


def _matmul_shape(a, b):
    a1, b1 = len(a) == 1, len(b) == 1
    a2 = (1, *a) if a1 else tuple(a)
    b2 = (*b, 1) if b1 else tuple(b)
    batch = _broadcast(a2[:-2], b2[:-2])
    out = (*batch, a2[-2], b2[-1])
    if a1:
        out = out[:-2] + out[-1:]
    if b1:
        out = out[:-1]
    return out


def infer_types(spec: GraphSpec) -> GraphSpec:
    """Give every node output that ``value_info`` left untyped a dtype and a
    static shape, following the ONNX operator definitions of the ops the
    reference's quantised model fixtures use (the role ONNX shape inference
    plays in the reference's importer).  Raises OnnxFormatError for an op it
    has no rule for."""
    known: dict[str, TensorSpec] = {t.name: t for t in (*spec.inputs, *spec.outputs, *spec.values)}
    for k, arr in spec.initializers.items():
        known.setdefault(k, TensorSpec(k, next(s for s, t in _NP.items() if np.dtype(t) == arr.dtype),
                                       tuple(arr.shape)))
    added: list[TensorSpec] = []

    def t(name):
        if name not in known:
            raise OnnxFormatError(f"value {name} has no type")
        return known[name]

    for node in spec.nodes:
        op, ins, a = node.op_type, node.inputs, node.attrs
        if all(o in known or not o for o in node.outputs):
            continue
        x = t(ins[0])
        if op in ("QuantizeLinear",):
            res = [(t(ins[2]).dtype if len(ins) > 2 and ins[2] else "u8", x.shape)]
        elif op == "DequantizeLinear":
            res = [("f32", x.shape)]
        elif op in ("QLinearConv", "Conv"):
            w = t(ins[3] if op == "QLinearConv" else ins[1])
            aa = dict(a)
            aa.setdefault("kernel_shape", list(w.shape[2:]))
            sp = _pool_out(x.shape, aa)
            res = [(t(ins[7]).dtype if op == "QLinearConv" else x.dtype, (x.shape[0], w.shape[0], *sp))]
        elif op in ("MaxPool", "AveragePool"):
            res = [(x.dtype, (*x.shape[:2], *_pool_out(x.shape, a)))]
        elif op == "QLinearAveragePool":
            res = [(t(ins[4]).dtype, (*x.shape[:2], *_pool_out(x.shape, a)))]
        elif op == "Reshape":
            target = [int(v) for v in np.asarray(spec.initializers[ins[1]]).reshape(-1)]
            dims = [x.shape[i] if v == 0 and not int(a.get("allowzero", 0)) else v for i, v in enumerate(target)]
            if -1 in dims:
                rest = int(np.prod([d for d in dims if d != -1]))
                dims[dims.index(-1)] = int(np.prod(x.shape)) // rest
            res = [(x.dtype, tuple(dims))]
        elif op == "Flatten":
            ax = int(a.get("axis", 1)) % max(len(x.shape), 1)
            res = [(x.dtype, (int(np.prod(x.shape[:ax])), int(np.prod(x.shape[ax:]))))]
        elif op == "Transpose":
            perm = list(a.get("perm", list(range(len(x.shape)))[::-1]))
            res = [(x.dtype, tuple(x.shape[p] for p in perm))]
        elif op == "QLinearMatMul":
            res = [(t(ins[7]).dtype, _matmul_shape(x.shape, t(ins[3]).shape))]
        elif op in ("MatMul", "MatMulInteger"):
            res = [("i32" if op == "MatMulInteger" else x.dtype, _matmul_shape(x.shape, t(ins[1]).shape))]
        elif op == "QLinearAdd":
            res = [(t(ins[7]).dtype, _broadcast(x.shape, t(ins[3]).shape))]
        elif op in ("Add", "Sub", "Mul", "Div"):
            res = [(x.dtype, _broadcast(x.shape, t(ins[1]).shape))]
        elif op in ("Relu", "Sigmoid", "Tanh", "Softmax", "Swish", "Identity"):
            res = [(x.dtype, x.shape)]
        elif op == "QLinearSoftmax":
            res = [(t(ins[4]).dtype, x.shape)]
        elif op == "Gemm":
            b = t(ins[1])
            m = x.shape[1] if int(a.get("transA", 0)) else x.shape[0]
            n = b.shape[0] if int(a.get("transB", 0)) else b.shape[1]
            res = [(x.dtype, (m, n))]
        else:
            raise OnnxFormatError(f"no type rule for {op} (output {node.outputs[0]})")
        for name, (dt, shp) in zip(node.outputs, res):
            if name and name not in known:
                ts = TensorSpec(name, dt, tuple(int(d) for d in shp))
                known[name] = ts
                added.append(ts)
    return GraphSpec(spec.name, spec.inputs, spec.outputs, spec.nodes, spec.initializers,
                     list(spec.values) + added, spec.opset_imports)

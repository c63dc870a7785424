"""Minimal ONNX model writer without the ``onnx`` package: the inverse of
``onnx_reader`` for the messages it decodes (same ``onnx.proto`` field
numbers).  Used to export the built-in workload graphs as ``.onnx`` files
for the command line (``python -m emx_onnx_cgen_b200 export``) and for any
ONNX consumer, the reference compiler included.

Tensors are written with ``raw_data`` (little-endian), graph inputs and
outputs and intermediate ``value_info`` with static shapes (or chosen axes
as symbolic ``dim_param``), attributes with their ``AttributeProto.type``.
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

from .spec import GraphSpec, NodeSpec, TensorSpec

_ELEM = {"f32": 1, "u8": 2, "i8": 3, "u16": 4, "i16": 5, "i32": 6, "i64": 7, "bool": 9, "f16": 10, "f64": 11,
         "u32": 12, "u64": 13}
_ELEM_OF_NP = {np.dtype(np.float32): 1, np.dtype(np.uint8): 2, np.dtype(np.int8): 3, np.dtype(np.uint16): 4,
               np.dtype(np.int16): 5, np.dtype(np.int32): 6, np.dtype(np.int64): 7, np.dtype(np.bool_): 9,
               np.dtype(np.float16): 10, np.dtype(np.float64): 11, np.dtype(np.uint32): 12,
               np.dtype(np.uint64): 13}
IR_VERSION = 10


def _varint(v: int) -> bytes:
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(num: int, wt: int) -> bytes:
    return _varint((num << 3) | wt)


def _vfield(num: int, v: int) -> bytes:
    return _key(num, 0) + _varint(int(v))


def _lfield(num: int, payload: bytes) -> bytes:
    return _key(num, 2) + _varint(len(payload)) + payload


def _sfield(num: int, s: str) -> bytes:
    return _lfield(num, s.encode())


def tensor_proto(name: str, arr: np.ndarray) -> bytes:
    arr = np.asarray(arr)
    if arr.dtype not in _ELEM_OF_NP:
        raise ValueError(f"tensor {name}: unsupported dtype {arr.dtype}")
    out = b"".join(_vfield(1, d) for d in arr.shape)
    out += _vfield(2, _ELEM_OF_NP[arr.dtype]) + _sfield(8, name)
    out += _lfield(9, np.ascontiguousarray(arr).astype(arr.dtype.newbyteorder("<")).tobytes())
    return out


def _value_info(t: TensorSpec, params: dict[int, str] | None = None) -> bytes:
    params = params or {}
    shape = b"".join(_lfield(1, _sfield(2, params[i]) if i in params else _vfield(1, d))
                     for i, d in enumerate(t.shape))
    tensor_type = _vfield(1, _ELEM[t.dtype]) + _lfield(2, shape)
    return _sfield(1, t.name) + _lfield(2, _lfield(1, tensor_type))


def _attribute(name: str, value) -> bytes:
    out = _sfield(1, name)
    if isinstance(value, (bool, int, np.integer)):
        return out + _vfield(3, int(value)) + _vfield(20, 2)
    if isinstance(value, (float, np.floating)):
        return out + _key(2, 5) + struct.pack("<f", float(value)) + _vfield(20, 1)
    if isinstance(value, str):
        return out + _sfield(4, value) + _vfield(20, 3)
    if isinstance(value, np.ndarray):
        return out + _lfield(5, tensor_proto(name, value)) + _vfield(20, 4)
    if isinstance(value, (list, tuple)):
        vals = list(value)
        if all(isinstance(v, (int, np.integer, bool)) for v in vals):
            return out + _lfield(8, b"".join(_varint(int(v)) for v in vals)) + _vfield(20, 7)
        if all(isinstance(v, (int, float, np.integer, np.floating)) for v in vals):
            return out + _lfield(7, struct.pack(f"<{len(vals)}f", *map(float, vals))) + _vfield(20, 6)
        if all(isinstance(v, str) for v in vals):
            return out + b"".join(_sfield(9, v) for v in vals) + _vfield(20, 8)
    raise ValueError(f"attribute {name}: cannot encode {type(value).__name__}")


def _node(n: NodeSpec) -> bytes:
    out = b"".join(_sfield(1, i) for i in n.inputs) + b"".join(_sfield(2, o) for o in n.outputs)
    out += _sfield(3, n.name) + _sfield(4, n.op_type)
    out += b"".join(_lfield(5, _attribute(k, v)) for k, v in n.attrs.items())
    if n.domain:
        out += _sfield(7, n.domain)
    return out


def write_onnx_bytes(spec: GraphSpec, producer: str = "emx_onnx_cgen_b200",
                     dim_params: dict[str, dict[int, str]] | None = None) -> bytes:
    """``dim_params`` writes chosen axes symbolically: {value name: {axis: dim_param}}."""
    dp = dim_params or {}
    graph = b"".join(_lfield(1, _node(n)) for n in spec.nodes) + _sfield(2, spec.name)
    graph += b"".join(_lfield(5, tensor_proto(k, v)) for k, v in spec.initializers.items())
    graph += b"".join(_lfield(11, _value_info(t, dp.get(t.name))) for t in spec.inputs)
    graph += b"".join(_lfield(12, _value_info(t, dp.get(t.name))) for t in spec.outputs)
    graph += b"".join(_lfield(13, _value_info(t, dp.get(t.name))) for t in spec.values)
    model = _vfield(1, IR_VERSION) + _sfield(2, producer)
    model += _lfield(7, graph)
    for dom, ver in spec.opset_imports:
        model += _lfield(8, (_sfield(1, dom) if dom else b"") + _vfield(2, ver))
    return model


def write_onnx(spec: GraphSpec, path: str | Path, dim_params: dict[str, dict[int, str]] | None = None) -> Path:
    p = Path(path)
    p.write_bytes(write_onnx_bytes(spec, dim_params=dim_params))
    return p

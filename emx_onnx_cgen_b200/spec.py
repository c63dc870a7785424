"""ONNX-shaped graph description used to build the workloads this backend runs.

A ``GraphSpec`` carries what an ONNX ``ModelProto`` carries for the hot path:
typed graph inputs/outputs, intermediate value types, initializers and nodes
with attributes and domains.  It is deliberately the same information the
reference compiler's IR holds (``ir/model.py:12-68``: ``TensorType``,
``Value``, ``Node``, ``Initializer``, ``Graph``), so the same spec can be fed
to the reference's lowering (by the test oracle) and to this package's own
lowering (``emx_onnx_cgen_b200.lowering``) and the two results compared.

Dtypes are the reference's ``ScalarType`` suffix strings ("f32", "f16",
"u8", "i8", "i32", "i64", ...; ``shared/scalar_types.py:76``).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Mapping

import numpy as np

NP_DTYPE: dict[str, np.dtype] = {
    "f32": np.dtype(np.float32),
    "f16": np.dtype(np.float16),
    "f64": np.dtype(np.float64),
    "u8": np.dtype(np.uint8),
    "i8": np.dtype(np.int8),
    "i16": np.dtype(np.int16),
    "u16": np.dtype(np.uint16),
    "i32": np.dtype(np.int32),
    "u32": np.dtype(np.uint32),
    "i64": np.dtype(np.int64),
    "u64": np.dtype(np.uint64),
    "bool": np.dtype(np.bool_),
}


def dtype_of_array(arr: np.ndarray) -> str:
    for suffix, dt in NP_DTYPE.items():
        if arr.dtype == dt:
            return suffix
    raise ValueError(f"unsupported numpy dtype {arr.dtype}")


@dataclass(frozen=True)
class TensorSpec:
    name: str
    dtype: str
    shape: tuple[int, ...]

    @property
    def nbytes(self) -> int:
        return int(np.prod(self.shape, dtype=np.int64)) * NP_DTYPE[self.dtype].itemsize


@dataclass(frozen=True)
class NodeSpec:
    op_type: str
    name: str
    inputs: tuple[str, ...]
    outputs: tuple[str, ...]
    attrs: Mapping[str, object] = field(default_factory=dict)
    domain: str | None = None


@dataclass
class GraphSpec:
    name: str
    inputs: list[TensorSpec]
    outputs: list[TensorSpec]
    nodes: list[NodeSpec]
    initializers: dict[str, np.ndarray]
    values: list[TensorSpec] = field(default_factory=list)
    opset_imports: tuple[tuple[str, int], ...] = (("", 17),)

    def tensor(self, name: str) -> TensorSpec:
        for t in (*self.inputs, *self.outputs, *self.values):
            if t.name == name:
                return t
        if name in self.initializers:
            arr = self.initializers[name]
            return TensorSpec(name, dtype_of_array(arr), tuple(arr.shape))
        raise KeyError(name)

"""TEST INFRASTRUCTURE ONLY -- never imported by the product package.

A permissive stand-in for the ``onnx`` Python package, installed into the
current process only, so the reference compiler's IR, lowering and C emitter
modules import in a container where ``onnx`` is not installed.  The reference
uses ``onnx`` on the path exercised here only for module-level imports and the
``TensorProto`` data-type enum (``dtypes.py:3-34``,
``codegen/c_emitter.py:19``, ``compiler.py:12``); model parsing and ONNX
shape inference are never reached because graphs are handed to
``Compiler._lower_model`` directly as reference IR objects.

The enum values are the public ONNX ``TensorProto.DataType`` numbers.
"""
from __future__ import annotations

import importlib.abc
import importlib.machinery
import sys
import types

_TENSOR_PROTO = dict(
    UNDEFINED=0, FLOAT=1, UINT8=2, INT8=3, UINT16=4, INT16=5, INT32=6, INT64=7,
    STRING=8, BOOL=9, FLOAT16=10, DOUBLE=11, UINT32=12, UINT64=13, COMPLEX64=14,
    COMPLEX128=15, BFLOAT16=16, FLOAT8E4M3FN=17, FLOAT8E4M3FNUZ=18, FLOAT8E5M2=19,
    FLOAT8E5M2FNUZ=20, UINT4=21, INT4=22, FLOAT4E2M1=23, FLOAT8E8M0=24, UINT2=25, INT2=26,
)


class _PlaceholderModule(types.ModuleType):
    """Any attribute resolves to a fresh empty class (usable in annotations and
    ``isinstance`` checks, which then simply fail)."""

    def __getattr__(self, key: str):
        if key.startswith("__"):
            raise AttributeError(key)
        if key == "TensorProto":
            value = type("TensorProto", (), dict(_TENSOR_PROTO))
        else:
            value = type(key, (), {})
        setattr(self, key, value)
        return value


class _OnnxFinder(importlib.abc.MetaPathFinder, importlib.abc.Loader):
    def find_spec(self, name, path, target=None):
        if name == "onnx" or name.startswith("onnx."):
            return importlib.machinery.ModuleSpec(name, self, is_package=True)
        return None

    def create_module(self, spec):
        return _PlaceholderModule(spec.name)

    def exec_module(self, module):
        module.__path__ = []


def install() -> None:
    """Install the stand-in unless a real ``onnx`` is importable."""
    if any(isinstance(f, _OnnxFinder) for f in sys.meta_path):
        return
    try:
        import onnx  # noqa: F401
        return
    except ImportError:
        pass
    sys.meta_path.insert(0, _OnnxFinder())

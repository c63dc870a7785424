"""An ``onnx.backend``-style adapter that runs ONNX models on a B200.

The reference ships ``EmxOnnxCgenBackend`` (src/emx_onnx_cgen/onnx_backend/
backend.py:549-660): ``prepare(model, device)`` compiles the model into a C
executable and returns a rep whose ``run(inputs)`` serialises the inputs,
runs the executable and decodes its outputs.  This module keeps that surface
-- the class methods ``is_compatible``, ``prepare``, ``run_model`` and
``supports_device``, the module-level aliases and ``backend_name`` -- with a
launch plan as the compiled form:

* ``prepare`` reads the model (no ``onnx`` package needed), pins its dynamic
  dimensions (``input_dims``, the command line's ``--input-dim`` forms),
  lowers it and emits the plan, then loads it on the GPU the device string
  names: ``"CUDA"`` (device 0) or ``"CUDA:<n>"``.  The reference accepts
  ``"CPU"`` only; this backend has no CPU path and rejects ``"CPU"``.
* ``rep.run(inputs)`` takes the inputs in the graph's input order (a
  sequence, like the reference) or by name (a dict) and returns the outputs
  in graph output order.  Every call is one run of the plan through the C ABI.
* A model is an ONNX ``ModelProto`` (anything with ``SerializeToString``), its
  serialised bytes, or a path.  An op without a B200 kernel raises
  ``UnsupportedOpError`` from ``prepare``, as the reference's compile step
  raises its own ``UnsupportedOpError``.

When the ``onnx`` package is importable, the classes derive from
``onnx.backend.base.Backend`` / ``BackendRep`` so onnx's backend test runner
accepts them; otherwise they are plain classes with the same methods.
"""
from __future__ import annotations

import re
from collections.abc import Mapping, Sequence
from pathlib import Path

import numpy as np

from .lowering import lower
from .onnx_reader import infer_types, read_onnx, read_onnx_bytes
from .plan import NP, B200PlanEmitter

try:  # the optional base classes of onnx's backend API
    from onnx.backend.base import Backend as _BackendBase, BackendRep as _RepBase
except ImportError:  # onnx is not installed: same methods, no base class
    _BackendBase, _RepBase = object, object

backend_name = "emx-onnx-cgen-b200"
_DEVICE = re.compile(r"^CUDA(?::(\d+))?$")


def parse_device(device: str) -> int:
    """CUDA ordinal of an onnx.backend device string ("CUDA", "CUDA:1")."""
    m = _DEVICE.match(str(device).strip().upper())
    if not m:
        raise RuntimeError(f"Unsupported device: {device} (this backend runs on CUDA devices only)")
    return int(m.group(1) or 0)


def _model_bytes(model) -> bytes | Path:
    if isinstance(model, (str, Path)):
        return Path(model)
    if isinstance(model, (bytes, bytearray, memoryview)):
        return bytes(model)
    if hasattr(model, "SerializeToString"):
        return model.SerializeToString()
    raise TypeError(f"expected a ModelProto, serialized bytes or a path, got {type(model).__name__}")


def compile_plan(model, input_dims: Mapping[str, int] | None = None, emitter: B200PlanEmitter | None = None):
    """ONNX model (ModelProto, bytes or path) -> launch plan, on the host (no GPU needed)."""
    src = _model_bytes(model)
    dims = dict(input_dims or {})
    spec = read_onnx(src, dims) if isinstance(src, Path) else read_onnx_bytes(src, dims)
    return (emitter or B200PlanEmitter()).emit_plan(lower(infer_types(spec)))


class B200BackendRep(_RepBase):
    """A prepared model: its plan loaded on one GPU."""

    def __init__(self, plan, device: int):
        from .runtime import Session  # loads the CUDA library; fails loudly without it

        self.plan = plan
        self.device = device
        self._session = Session(plan, device=device)

    @property
    def input_names(self) -> list[str]:
        return list(self.plan.input_names)

    @property
    def output_names(self) -> list[str]:
        return list(self.plan.output_names)

    def run(self, inputs, **kwargs) -> list[np.ndarray]:
        if isinstance(inputs, Mapping):
            named = dict(inputs)
            missing = [n for n in self.plan.input_names if n not in named]
            if missing:
                raise ValueError(f"missing inputs {missing}")
        else:
            seq = list(inputs) if isinstance(inputs, Sequence) or hasattr(inputs, "__iter__") else [inputs]
            if len(seq) != len(self.plan.input_names):
                raise ValueError(f"expected {len(self.plan.input_names)} inputs "
                                 f"({', '.join(self.plan.input_names)}), got {len(seq)}")
            named = dict(zip(self.plan.input_names, seq))
        arrays = {}
        for name, shape, dt in zip(self.plan.input_names, self.plan.input_shapes, self.plan.input_dtypes):
            a = np.asarray(named[name])
            want = np.dtype(NP[dt])
            if a.dtype != want:
                raise TypeError(f"input {name!r}: dtype {a.dtype}, the model wants {want}")
            if tuple(a.shape) != tuple(shape):
                raise ValueError(f"input {name!r}: shape {tuple(a.shape)}, the plan was built for {tuple(shape)}")
            arrays[name] = a
        outs = self._session.run(arrays)
        return [outs[n] for n in self.plan.output_names]

    def close(self) -> None:
        self._session.close()


class B200Backend(_BackendBase):
    """onnx.backend entry points (class methods, as in the reference)."""

    @classmethod
    def is_compatible(cls, model, device: str = "CUDA", **kwargs) -> bool:
        try:
            parse_device(device)
            compile_plan(model, kwargs.get("input_dims"))
        except Exception:  # noqa: BLE001 -- any reason the model cannot be planned
            return False
        return True

    @classmethod
    def prepare(cls, model, device: str = "CUDA", **kwargs) -> B200BackendRep:
        ordinal = parse_device(device)
        emitter = kwargs.pop("emitter", None)
        plan = compile_plan(model, kwargs.pop("input_dims", None), emitter)
        return B200BackendRep(plan, ordinal)

    @classmethod
    def run_model(cls, model, inputs, device: str = "CUDA", **kwargs) -> list[np.ndarray]:
        rep = cls.prepare(model, device=device, **kwargs)
        try:
            return rep.run(inputs)
        finally:
            rep.close()

    @classmethod
    def supports_device(cls, device: str) -> bool:
        try:
            parse_device(device)
        except RuntimeError:
            return False
        return True


prepare = B200Backend.prepare
run_model = B200Backend.run_model
supports_device = B200Backend.supports_device
is_compatible = B200Backend.is_compatible

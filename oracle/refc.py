"""TEST INFRASTRUCTURE ONLY: the reference's own generated C as the parity oracle.

This module drives the reference compiler (its ``src`` directory, read-only:
the directory the ``EMX_REFERENCE_SRC`` environment variable names, else a
``reference/src`` checkout beside this repository's) to lower a
``GraphSpec`` and emit its C translation unit, exactly the way the
reference's CLI does between ``Compiler._lower_model`` (``compiler.py:514``)
and ``CEmitter.emit_model`` / ``collect_weight_data``
(``codegen/c_emitter.py:1312``, ``:4398``).  The emitted C is compiled with
``gcc -std=c99 -O2`` (no ``-march``, no ``-ffast-math``) into a shared
library under ``oracle/_ref/`` and called through ctypes with the generated
ABI ``_Bool <model>_load(const char *)`` / ``void <model>(inputs..., outputs...)``
(``docs/output-format.md:132-193``).

Only ``tests/``, ``__graft_entry__`` and ``bench.py``'s CPU-baseline legs use
this, and only to check results against.  The reference itself is needed only to
*generate* the C (in the build container); the compiled libraries in
``oracle/_ref/`` run without it.
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"
_SRC_ENV = os.environ.get("EMX_REFERENCE_SRC", "")
REFERENCE_SRC = Path(_SRC_ENV) if _SRC_ENV else HERE.parent.parent / "reference" / "src"

sys.path.insert(0, str(HERE.parent))
from emx_onnx_cgen_b200.spec import GraphSpec, NP_DTYPE  # noqa: E402

CFLAGS = ["-std=c99", "-O2", "-fPIC", "-shared", "-w"]


def reference_available() -> bool:
    """True when the reference's ``src`` directory is present."""
    return (REFERENCE_SRC / "emx_onnx_cgen" / "compiler.py").is_file()


def _import_reference():
    from oracle import onnx_shim  # noqa: WPS433
    onnx_shim.install()
    if str(REFERENCE_SRC) not in sys.path:
        sys.path.insert(0, str(REFERENCE_SRC))
    from shared.scalar_types import ScalarType
    from emx_onnx_cgen.compiler import Compiler, CompilerOptions
    from emx_onnx_cgen.ir import model as ir
    return ScalarType, Compiler, CompilerOptions, ir


class _ModelHeaderSource:
    """Duck-typed stand-in for the ``ModelProto`` fields read by
    ``Compiler._build_header`` (compiler.py:1082-1138)."""

    metadata_props = ()
    opset_import = ()
    doc_string = ""
    producer_name = ""
    producer_version = ""
    domain = ""
    model_version = 0
    ir_version = 10

    class graph:  # noqa: N801
        name = "g"
        doc_string = ""

    def SerializeToString(self) -> bytes:  # noqa: N802
        return b"synthetic"


def to_reference_graph(spec: GraphSpec):
    ScalarType, _, _, ir = _import_reference()

    def tt(dtype: str, shape):
        return ir.TensorType(dtype=ScalarType(dtype), shape=tuple(int(s) for s in shape),
                             dim_params=(None,) * len(shape))

    inits = tuple(
        ir.Initializer(name, tt(_suffix(arr), arr.shape), arr)
        for name, arr in spec.initializers.items()
    )
    return ir.Graph(
        inputs=tuple(ir.Value(t.name, tt(t.dtype, t.shape)) for t in spec.inputs),
        outputs=tuple(ir.Value(t.name, tt(t.dtype, t.shape)) for t in spec.outputs),
        nodes=tuple(ir.Node(n.op_type, n.name, tuple(n.inputs), tuple(n.outputs), dict(n.attrs),
                            n.domain) for n in spec.nodes),
        initializers=inits,
        values=tuple(ir.Value(t.name, tt(t.dtype, t.shape)) for t in spec.values),
        opset_imports=tuple(spec.opset_imports),
    )


def _suffix(arr: np.ndarray) -> str:
    for k, v in NP_DTYPE.items():
        if arr.dtype == v:
            return k
    raise ValueError(arr.dtype)


def lower(spec: GraphSpec, model_name: str | None = None, **options):
    """The reference's ``LoweredModel`` for ``spec`` (Compiler._lower_model)."""
    _, Compiler, CompilerOptions, _ = _import_reference()
    opts = CompilerOptions(model_name=model_name or spec.name, model_checksum="0" * 64, **options)
    compiler = Compiler(opts)
    return compiler, compiler._lower_model(_ModelHeaderSource(), to_reference_graph(spec))


def emit_c(spec: GraphSpec, out_dir: Path, model_name: str | None = None, **options):
    """Write ``<name>.c`` (+ ``<name>.bin`` when weights exceed the reference's
    large-weight threshold) and return their paths."""
    name = model_name or spec.name
    compiler, lowered = lower(spec, name, **options)
    src = compiler._emitter.emit_model(
        lowered, emit_testbench=False, testbench_inputs=None, testbench_outputs=None,
        testbench_optional_inputs=None, variable_dim_inputs={}, variable_dim_outputs={})
    weights = compiler._emitter.collect_weight_data(lowered.constants)
    out_dir.mkdir(parents=True, exist_ok=True)
    c_path = out_dir / f"{name}.c"
    c_path.write_text(src)
    bin_path = None
    if weights:
        bin_path = out_dir / f"{name}.bin"
        bin_path.write_bytes(weights)
    return c_path, bin_path


def compile_so(c_path: Path, so_path: Path | None = None) -> Path:
    so_path = so_path or c_path.with_suffix(".so")
    std = "-std=c2x" if "_BitInt(" in c_path.read_text() else None
    flags = [f if not (f == "-std=c99" and std) else std for f in CFLAGS]
    subprocess.run(["gcc", *flags, str(c_path), "-o", str(so_path), "-lm"], check=True)
    return so_path


def build(spec: GraphSpec, tag: str, out_dir: Path = REF_DIR, **options) -> Path:
    """Emit + compile; writes ``<tag>.c``, ``<tag>.so``, optional ``<tag>.bin`` and
    ``<tag>.json`` (I/O signature) under ``out_dir``.  Returns the .so path."""
    c_path, bin_path = emit_c(spec, out_dir, tag, **options)
    so = compile_so(c_path)
    meta = {
        "name": tag,
        "inputs": [[t.name, t.dtype, list(t.shape)] for t in spec.inputs],
        "outputs": [[t.name, t.dtype, list(t.shape)] for t in spec.outputs],
        "bin": bin_path.name if bin_path else None,
    }
    (out_dir / f"{tag}.json").write_text(json.dumps(meta))
    return so


class RefCModel:
    """A compiled reference model: ``run(inputs) -> outputs`` through the
    generated ABI.  Thread-safe for concurrent ``run`` calls after ``load``
    (the generated code keeps weights in read-only globals and allocates its
    temporaries per call, c_emitter.py:2744-2789)."""

    def __init__(self, tag: str, out_dir: Path = REF_DIR):
        meta = json.loads((out_dir / f"{tag}.json").read_text())
        self.meta = meta
        self.lib = ctypes.CDLL(str(out_dir / f"{tag}.so"))
        self.fn = getattr(self.lib, tag)
        self.fn.restype = None
        load = getattr(self.lib, f"{tag}_load")
        load.restype = ctypes.c_bool
        load.argtypes = [ctypes.c_char_p]
        path = str(out_dir / meta["bin"]) if meta["bin"] else ""
        if not load(path.encode()):
            raise RuntimeError(f"{tag}_load failed")

    def run(self, inputs: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
        args = []
        keep = []
        for name, dt, shape in self.meta["inputs"]:
            a = np.ascontiguousarray(inputs[name], dtype=NP_DTYPE[dt]).reshape(shape)
            keep.append(a)
            args.append(a.ctypes.data_as(ctypes.c_void_p))
        outs = {}
        for name, dt, shape in self.meta["outputs"]:
            o = np.zeros(shape, dtype=NP_DTYPE[dt])
            outs[name] = o
            args.append(o.ctypes.data_as(ctypes.c_void_p))
        self.fn(*args)
        return outs

    def run_into(self, in_ptrs: list[int], out_ptrs: list[int]) -> None:
        self.fn(*[ctypes.c_void_p(p) for p in (*in_ptrs, *out_ptrs)])

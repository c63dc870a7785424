"""The C-ABI library loads and exports every symbol include/emx_b200.h declares;
host-side error paths that need no GPU return the documented status codes."""
import ctypes
import re
from pathlib import Path

import pytest

from emx_onnx_cgen_b200 import runtime

HEADER = Path(__file__).resolve().parents[1] / "include" / "emx_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(emx_b200_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for s in ("emx_b200_plan_load", "emx_b200_run", "emx_b200_sync", "emx_b200_last_error",
              "emx_b200_plan_free"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    lib = runtime.load_library()
    for s in declared_symbols():
        assert hasattr(lib, s), s


def test_version():
    assert re.match(r"\d+\.\d+\.\d+", runtime.version())


def test_corrupt_plan_rejected_without_gpu():
    lib = runtime.load_library()
    out = ctypes.c_void_p()
    bad = b"\x00" * 64
    rc = lib.emx_b200_plan_load_mem(bad, len(bad), None, 0, 0, ctypes.byref(out))
    assert rc == 2  # EMX_ERR_PLAN_FORMAT
    assert b"magic" in lib.emx_b200_last_error()
    rc = lib.emx_b200_plan_load(b"x", 1, None, 0, ctypes.byref(out))
    assert rc == 2
    assert not out.value


def test_truncated_plan_rejected():
    from emx_onnx_cgen_b200 import lowering, workloads as W
    from emx_onnx_cgen_b200.plan import B200PlanEmitter
    plan = B200PlanEmitter().emit_plan(lowering.lower(W.qconv_stack_int8(batch=1, height=8, width=8).graph))
    lib = runtime.load_library()
    out = ctypes.c_void_p()
    blob = plan.plan_bytes[:-8]
    assert lib.emx_b200_plan_load_mem(blob, len(blob), None, 0, 0, ctypes.byref(out)) == 2
    blob = bytearray(plan.plan_bytes)
    blob[4] = 99  # version
    assert lib.emx_b200_plan_load_mem(bytes(blob), len(blob), None, 0, 0, ctypes.byref(out)) == 2
    assert b"version" in lib.emx_b200_last_error()


def test_missing_weights_file_reported(tmp_path):
    from emx_onnx_cgen_b200 import lowering, workloads as W
    from emx_onnx_cgen_b200.plan import B200PlanEmitter
    plan = B200PlanEmitter().emit_plan(lowering.lower(W.qconv_stack_int8(batch=1, height=8, width=8).graph))
    lib = runtime.load_library()
    out = ctypes.c_void_p()
    rc = lib.emx_b200_plan_load(plan.plan_bytes, len(plan.plan_bytes), str(tmp_path / "none.bin").encode(), 0,
                                ctypes.byref(out))
    assert rc == 3  # EMX_ERR_WEIGHTS
    short = tmp_path / "short.bin"
    short.write_bytes(plan.weight_bytes[:-1])
    rc = lib.emx_b200_plan_load(plan.plan_bytes, len(plan.plan_bytes), str(short).encode(), 0, ctypes.byref(out))
    assert rc == 3 and b"short read" in lib.emx_b200_last_error()


def test_null_arguments():
    lib = runtime.load_library()
    assert lib.emx_b200_plan_load_mem(None, 0, None, 0, 0, None) == 1
    assert lib.emx_b200_run(None, None, None, 0, -1, None) == 1
    assert lib.emx_b200_sync(None) == 1
    assert lib.emx_b200_set_host_io_chunks(None, 4) == 1
    assert lib.emx_b200_set_graphs(None, 1) == 1
    lib.emx_b200_plan_free(None)

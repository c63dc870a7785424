"""ctypes binding of libemx_b200.so (include/emx_b200.h) and a per-device Session.

This is the "thin ctypes C-ABI" the Python driver uses; it is also the model
for a binding in any other host language.  The library
must have been built (``python -m emx_onnx_cgen_b200.build``); there is no
fallback: a missing library raises ``RuntimeError`` at first use.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import numpy as np

from .plan import NP, Plan

LIB_PATH = Path(__file__).resolve().parent / "libemx_b200.so"

EMX_OK = 0
STATUS_NAMES = {0: "EMX_OK", 1: "EMX_ERR_INVALID_ARGUMENT", 2: "EMX_ERR_PLAN_FORMAT", 3: "EMX_ERR_WEIGHTS",
                4: "EMX_ERR_CUDA", 5: "EMX_ERR_UNSUPPORTED", 6: "EMX_ERR_DEVICE_TIMEOUT",
                7: "EMX_ERR_OUT_OF_MEMORY"}

EXPORTED = ("emx_b200_version", "emx_b200_last_error", "emx_b200_plan_load", "emx_b200_plan_load_mem",
            "emx_b200_run", "emx_b200_sync", "emx_b200_plan_free", "emx_b200_plan_info",
            "emx_b200_launch_count", "emx_b200_set_profiling", "emx_b200_op_times", "emx_b200_set_graphs",
            "emx_b200_set_host_io_chunks", "emx_b200_set_host_io_overlap", "emx_b200_join",
            "emx_b200_set_wait_budget", "emx_b200_set_fault")

FAULT_DROP_CHAIN_PROGRESS = 1


class EmxError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class PlanInfo(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("n_inputs", ctypes.c_int32), ("n_outputs", ctypes.c_int32),
                ("n_ops", ctypes.c_int32), ("batch", ctypes.c_int64), ("arena_bytes", ctypes.c_int64),
                ("weight_bytes", ctypes.c_int64), ("launches_per_run", ctypes.c_int64)]


_lib = None
_lock = threading.Lock()


def load_library(path: Path | None = None) -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path or LIB_PATH)
        if not p.exists():
            raise RuntimeError(f"{p} not found: build it with `python -m emx_onnx_cgen_b200.build`")
        lib = ctypes.CDLL(str(p))
        vp, sz, i64, i32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int64, ctypes.c_int
        lib.emx_b200_version.restype = ctypes.c_char_p
        lib.emx_b200_last_error.restype = ctypes.c_char_p
        lib.emx_b200_plan_load.argtypes = [vp, sz, ctypes.c_char_p, i32, ctypes.POINTER(vp)]
        lib.emx_b200_plan_load_mem.argtypes = [vp, sz, vp, sz, i32, ctypes.POINTER(vp)]
        lib.emx_b200_run.argtypes = [vp, ctypes.POINTER(vp), ctypes.POINTER(vp), i64, i64, vp]
        lib.emx_b200_sync.argtypes = [vp]
        lib.emx_b200_plan_free.argtypes = [vp]
        lib.emx_b200_plan_free.restype = None
        lib.emx_b200_plan_info.argtypes = [vp, ctypes.POINTER(PlanInfo)]
        lib.emx_b200_launch_count.argtypes = [vp]
        lib.emx_b200_launch_count.restype = i64
        lib.emx_b200_set_profiling.argtypes = [vp, i32]
        lib.emx_b200_set_graphs.argtypes = [vp, i32]
        lib.emx_b200_set_graphs.restype = i32
        lib.emx_b200_set_host_io_chunks.argtypes = [vp, i32]
        lib.emx_b200_set_host_io_chunks.restype = i32
        lib.emx_b200_set_host_io_overlap.argtypes = [vp, i32]
        lib.emx_b200_set_host_io_overlap.restype = i32
        lib.emx_b200_join.argtypes = [vp, vp]
        lib.emx_b200_join.restype = i32
        lib.emx_b200_set_wait_budget.argtypes = [vp, ctypes.c_uint64]
        lib.emx_b200_set_wait_budget.restype = i32
        lib.emx_b200_set_fault.argtypes = [vp, i32]
        lib.emx_b200_set_fault.restype = i32
        lib.emx_b200_op_times.argtypes = [vp, ctypes.POINTER(ctypes.c_double), ctypes.c_int32,
                                          ctypes.POINTER(i64)]
        for name in ("emx_b200_plan_load", "emx_b200_plan_load_mem", "emx_b200_run", "emx_b200_sync",
                     "emx_b200_plan_info", "emx_b200_set_profiling", "emx_b200_op_times"):
            getattr(lib, name).restype = i32
        _lib = lib
        return lib


def _check(status: int) -> None:
    if status != EMX_OK:
        msg = load_library().emx_b200_last_error().decode(errors="replace")
        raise EmxError(status, msg)


class Session:
    """One loaded plan on one device (the runtime counterpart of the generated
    ``<model>_load`` + ``<model>()`` pair)."""

    def __init__(self, plan: Plan, device: int = 0, weights_path: str | None = None):
        self.lib = load_library()
        self.plan = plan
        self.device = device
        self._blob = ctypes.create_string_buffer(plan.plan_bytes, len(plan.plan_bytes))
        handle = ctypes.c_void_p()
        if weights_path is not None:
            _check(self.lib.emx_b200_plan_load(self._blob, len(plan.plan_bytes), weights_path.encode(), device,
                                               ctypes.byref(handle)))
        else:
            wbuf = ctypes.create_string_buffer(plan.weight_bytes, max(1, len(plan.weight_bytes)))
            _check(self.lib.emx_b200_plan_load_mem(self._blob, len(plan.plan_bytes), wbuf,
                                                   len(plan.weight_bytes), device, ctypes.byref(handle)))
        self.handle = handle

    # -- raw pointer interface (host or device pointers)
    def run_ptrs(self, in_ptrs, out_ptrs, batch_begin: int = 0, batch_count: int = -1, stream: int = 0) -> None:
        ins = (ctypes.c_void_p * max(1, len(in_ptrs)))(*in_ptrs)
        outs = (ctypes.c_void_p * max(1, len(out_ptrs)))(*out_ptrs)
        _check(self.lib.emx_b200_run(self.handle, ins, outs, batch_begin, batch_count,
                                     ctypes.c_void_p(stream) if stream else None))

    def sync(self) -> None:
        _check(self.lib.emx_b200_sync(self.handle))

    # -- numpy convenience: host arrays in, host arrays out
    def run(self, inputs: dict[str, np.ndarray], batch_begin: int = 0, batch_count: int = -1) -> dict[str, np.ndarray]:
        p = self.plan
        keep, in_ptrs = [], []
        for name, shape, dt in zip(p.input_names, p.input_shapes, p.input_dtypes):
            a = np.ascontiguousarray(inputs[name], dtype=NP[dt])
            if a.shape != tuple(shape):
                raise ValueError(f"input {name}: shape {a.shape}, plan expects {tuple(shape)}")
            keep.append(a)
            in_ptrs.append(a.ctypes.data)
        outs = {}
        out_ptrs = []
        for name, shape, dt in zip(p.output_names, p.output_shapes, p.output_dtypes):
            o = np.zeros(shape, dtype=NP[dt])
            outs[name] = o
            out_ptrs.append(o.ctypes.data)
        self.run_ptrs(in_ptrs, out_ptrs, batch_begin, batch_count)
        self.sync()
        return outs

    def info(self) -> PlanInfo:
        inf = PlanInfo()
        _check(self.lib.emx_b200_plan_info(self.handle, ctypes.byref(inf)))
        return inf

    def set_graphs(self, enable: bool) -> None:
        _check(self.lib.emx_b200_set_graphs(self.handle, 1 if enable else 0))

    def set_host_io_overlap(self, enable: bool) -> None:
        """Overlap consecutive runs' uploads, kernels and downloads (page-locked host buffers)."""
        _check(self.lib.emx_b200_set_host_io_overlap(self.handle, 1 if enable else 0))

    def join(self, stream: int = 0) -> None:
        """Make `stream` wait for every download of the overlapped runs issued so far."""
        _check(self.lib.emx_b200_join(self.handle, ctypes.c_void_p(stream) if stream else None))

    def set_host_io_chunks(self, chunks: int) -> None:
        """Batch slices for pipelined page-locked host I/O (1 = off)."""
        _check(self.lib.emx_b200_set_host_io_chunks(self.handle, int(chunks)))

    def set_wait_budget(self, ns: int) -> None:
        """Budget of every bounded device-side wait, in ns (0 = the 2 s default)."""
        _check(self.lib.emx_b200_set_wait_budget(self.handle, int(ns)))

    def set_fault(self, hooks: int) -> None:
        """Failure-detection test hooks (FAULT_* bits; 0 = none)."""
        _check(self.lib.emx_b200_set_fault(self.handle, int(hooks)))

    def set_profiling(self, enable: bool) -> None:
        _check(self.lib.emx_b200_set_profiling(self.handle, 1 if enable else 0))

    def op_times(self) -> tuple[list[float], int]:
        """(accumulated ms per op, number of profiled runs)."""
        n = len(self.plan.ops)
        buf = (ctypes.c_double * max(1, n))()
        runs = ctypes.c_int64()
        _check(self.lib.emx_b200_op_times(self.handle, buf, n, ctypes.byref(runs)))
        return list(buf)[:n], int(runs.value)

    def launch_count(self) -> int:
        return int(self.lib.emx_b200_launch_count(self.handle))

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.emx_b200_plan_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def version() -> str:
    return load_library().emx_b200_version().decode()

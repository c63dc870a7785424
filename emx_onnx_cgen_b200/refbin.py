"""The reference's external weight file (``<model>.bin``) as a weight source.

The reference's C emitter keeps small constants inline in the generated C
and writes the others, in ``LoweredModel.constants`` order, as concatenated
C-order arrays into ``<model>.bin`` (codegen/c_emitter.py:4230-4268
``_partition_constants``, :4398-4407 ``collect_weight_data``): constants are
taken smallest first (ties in constant order) into the inline set while the
inline total stays within the threshold (``--large-weight-threshold``,
default 100 KiB); string constants are always inline; everything else goes
to the file.  ``constants_from_bin`` reads such a file back into the
constants of a lowered model, so a plan can be built from the same artefact
the generated C loads.
"""
from __future__ import annotations

import dataclasses

import numpy as np

from .spec import NP_DTYPE

DEFAULT_LARGE_WEIGHT_THRESHOLD = 100 * 1024


def _suffix(dt) -> str:
    return str(getattr(dt, "value", dt))


def _np(const) -> np.dtype:
    return NP_DTYPE[_suffix(const.dtype)]


def _nbytes(const) -> int:
    return int(np.prod(const.shape, dtype=np.int64)) * _np(const).itemsize


def partition_constants(constants, threshold: int = DEFAULT_LARGE_WEIGHT_THRESHOLD):
    """(inline, large) in constant order, by the reference's rule."""
    if threshold <= 0:
        return tuple(constants), ()
    order = sorted(enumerate(constants),
                   key=lambda it: (0 if _suffix(it[1].dtype) == "string" else _nbytes(it[1]), it[0]))
    inline_ids, total = set(), 0
    for idx, c in order:
        if _suffix(c.dtype) == "string":
            inline_ids.add(idx)
            continue
        nb = _nbytes(c)
        if total + nb <= threshold:
            inline_ids.add(idx)
            total += nb
    inline = tuple(c for i, c in enumerate(constants) if i in inline_ids)
    large = tuple(c for i, c in enumerate(constants) if i not in inline_ids)
    return inline, large


def weight_bin_bytes(constants, threshold: int = DEFAULT_LARGE_WEIGHT_THRESHOLD) -> bytes:
    """The bytes the reference writes to ``<model>.bin`` for these constants."""
    _, large = partition_constants(constants, threshold)
    return b"".join(np.ascontiguousarray(np.asarray(c.data, dtype=_np(c))).tobytes() for c in large)


def constants_from_bin(model, data: bytes, threshold: int = DEFAULT_LARGE_WEIGHT_THRESHOLD):
    """A copy of ``model`` whose large constants hold the values read from
    ``data`` (a ``<model>.bin`` written for the same model and threshold)."""
    _, large = partition_constants(model.constants, threshold)
    need = sum(_nbytes(c) for c in large)
    if len(data) != need:
        raise ValueError(f"weight file holds {len(data)} bytes, the model's large constants need {need}")
    pos, values = 0, {}
    for c in large:
        nb = _nbytes(c)
        values[c.name] = np.frombuffer(data[pos:pos + nb], dtype=_np(c)).reshape(c.shape).copy()
        pos += nb
    consts = tuple(dataclasses.replace(c, data=values[c.name]) if c.name in values else c for c in model.constants)
    return dataclasses.replace(model, constants=consts)

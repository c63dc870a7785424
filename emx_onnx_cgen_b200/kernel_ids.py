"""Kernel ids and plan-parameter slot numbers, read from ``csrc/kernels.h``.

The C++ header is the single source of truth; this module parses its enum
blocks at import time so the plan emitter and the runtime can never disagree
on a slot number.  Every enumerator becomes a module attribute
(``K_QCONV_TC``, ``QC_OC``, ...); ``NAMES`` maps kernel id -> name.
"""
from __future__ import annotations

import re
from pathlib import Path

_HEADER = Path(__file__).resolve().parent / "csrc" / "kernels.h"


def _parse(text: str) -> dict[str, int]:
    text = re.sub(r"//[^\n]*", "", text)
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    values: dict[str, int] = {}
    for body in re.findall(r"enum\s*(?:\w+\s*)?(?::\s*\w+\s*)?\{([^}]*)\}", text):
        nxt = 0
        for item in body.split(","):
            item = item.strip()
            if not item:
                continue
            if "=" in item:
                name, val = (s.strip() for s in item.split("=", 1))
                nxt = int(val, 0)
            else:
                name = item
            values[name] = nxt
            nxt += 1
    return values


ENUMS = _parse(_HEADER.read_text())
globals().update(ENUMS)
IP_BATCHED_SLOT = 39  # kernels.h: IP_BATCHED = EMX_OP_MAX_IPARAMS - 1
NAMES = {v: k[2:].lower() for k, v in ENUMS.items() if k.startswith("K_")}

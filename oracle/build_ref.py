"""TEST INFRASTRUCTURE ONLY: recipe that builds ``oracle/_ref/`` -- the
reference's own generated C for the CPU-baseline slices of each workload.

For every target the reference compiler (read from its source tree, the
directory ``EMX_REFERENCE_SRC`` names, else ``reference/src`` beside this
repository, via the onnx shim)
lowers the workload graph at a slice size and emits C, which is compiled with
``gcc -std=c99 -O2 -fPIC -shared``.  The slice keeps the full per-row problem
and shrinks only the independent batch/row dimension, along which the
reference's loop nests are independent (gemm_op.c.j2:2, qlinear_conv_op.c.j2:2,
matmul_nbits_op.c.j2:2, attention_op.c.j2:48-51, lstm_op.c.j2:33): running the
slice ``batch / slice`` times is the full workload.

Outputs go to ``oracle/_ref/<tag>.{c,so,json[,bin]}`` (git-ignored; the
compiled files travel with the repository snapshot to the GPU hosts, which run
them without the reference).

    python oracle/build_ref.py [tag ...]
"""
from __future__ import annotations

import json
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

from emx_onnx_cgen_b200 import workloads as W  # noqa: E402
from oracle import refc  # noqa: E402

# tag -> (builder, slice kwargs, rows per full workload covered by one call, full rows)
TARGETS = {
    "ref_qconv_b1": ("qconv_stack_int8", dict(batch=1), 1, 32),
    "ref_mlp_m64": ("mlp_fp32", dict(m=64), 64, 64),
    "ref_nbits_m1": ("llama_mlp_int4", dict(m=1), 1, 2048),
    "ref_attn_b1h1": ("attention_fp16", dict(batch=1, heads=1), 1, 8 * 32),
    "ref_lstm_b1": ("lstm_fp32", dict(batch=1), 1, 256),
}


def build(tags=None) -> None:
    refc.REF_DIR.mkdir(exist_ok=True)
    index_path = refc.REF_DIR / "index.json"
    index = json.loads(index_path.read_text()) if index_path.exists() else {}
    for tag in tags or TARGETS:
        builder, kwargs, rows, full_rows = TARGETS[tag]
        t0 = time.time()
        wl = W.BUILDERS[builder](**kwargs)
        refc.build(wl.graph, tag)
        index[tag] = {"builder": builder, "kwargs": kwargs, "rows_per_call": rows, "full_rows": full_rows}
        print(f"{tag}: built in {time.time() - t0:.1f}s", flush=True)
    index_path.write_text(json.dumps(index, indent=1))


if __name__ == "__main__":
    if not refc.reference_available():
        raise SystemExit(f"reference source not found at {refc.REFERENCE_SRC}")
    build(sys.argv[1:] or None)

"""Run one workload's launch plan a few times on cuda:0 (the command profilers wrap).

    python -m emx_onnx_cgen_b200.profile_run --workload qconv_stack_int8 --iters 5 [--batch 8] [--kw JSON]

Device-resident inputs, no host copies, one synchronisation at the end, so a
profiler sees only this library's kernels after the first plan load.  Prints
the mean per-op CUDA-event time of a separate profiled pass.
"""
from __future__ import annotations

import argparse
import json

import numpy as np


def main() -> None:
    import torch

    from . import kernel_ids as K, lowering, workloads as W
    from .plan import NP, B200PlanEmitter
    from .runtime import Session

    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="qconv_stack_int8")
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--batch", type=int, default=0, help="override the workload's batch/rows (0: default)")
    ap.add_argument("--kw", default="", help='builder arguments as JSON, e.g. \'{"shape": [16384, 4096]}\'')
    ap.add_argument("--emit", default="", help='plan emitter options as JSON, e.g. \'{"attention_mode": "tensor"}\'')
    args = ap.parse_args()
    kw = {k: tuple(v) if isinstance(v, list) else v for k, v in json.loads(args.kw).items()} if args.kw else {}
    if args.batch:
        key = {"qconv_stack_int8": "batch", "mlp_fp32": "m", "llama_mlp_int4": "m", "attention_fp16": "batch",
               "lstm_fp32": "batch"}[args.workload]
        kw[key] = args.batch
    wl = W.BUILDERS[args.workload](**kw)
    plan = B200PlanEmitter(**(json.loads(args.emit) if args.emit else {})).emit_plan(lowering.lower(wl.graph))
    sess = Session(plan, device=0)
    x = wl.make_inputs(0)
    ins = [torch.from_numpy(np.ascontiguousarray(x[n])).cuda() for n in plan.input_names]
    outs = [torch.empty(s, dtype=getattr(torch, np.dtype(NP[d]).name), device="cuda")
            for s, d in zip(plan.output_shapes, plan.output_dtypes)]
    stream = torch.cuda.Stream()
    ip, op = [t.data_ptr() for t in ins], [t.data_ptr() for t in outs]
    for _ in range(args.iters):
        sess.run_ptrs(ip, op, stream=stream.cuda_stream)
    sess.sync()
    sess.set_profiling(True)
    for _ in range(3):
        sess.run_ptrs(ip, op, stream=stream.cuda_stream)
        sess.sync()
    ms, runs = sess.op_times()
    print(json.dumps({f"{i}:{K.NAMES[o.kernel]}": t / runs for i, (t, o) in enumerate(zip(ms, plan.ops))}))
    sess.close()


if __name__ == "__main__":
    main()

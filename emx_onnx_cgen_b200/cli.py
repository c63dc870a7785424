"""Command line of the B200 backend: ``python -m emx_onnx_cgen_b200 ...``.

Mirrors the reference CLI's ``compile`` and ``verify`` commands
(src/emx_onnx_cgen/cli.py:1005-1260) with a B200 launch plan as the target
instead of C source:

``compile MODEL.onnx [-o DIR]``
    read the model, pin dynamic dimensions (``--input-dim``, both of the
    reference's forms), lower it and write ``<name>.plan``, ``<name>.weights``
    and ``<name>.json`` (see ``plan.save_plan``).  ``--weights-bin FILE``
    takes the large constants from a ``<model>.bin`` the reference wrote for
    the same model (``--large-weight-threshold`` as there, default 102400).
``run PLAN --inputs IN.npz --outputs OUT.npz``
    run a compiled plan (``PLAN`` = the path without extension) on one GPU.
``verify MODEL.onnx|PLAN --inputs IN.npz --expected EXP.npz``
    compile (or load), run, and compare with expected outputs by the
    reference's metric: ``--max-ulp`` (default 100) and ``--atol-eps``
    (default 1.0) for floating outputs, exact for integer ones.  Prints
    ``OK (max ULP n)`` and exits 0, or the failing outputs and exits 1.
``export WORKLOAD OUT.onnx``
    write one of the built-in workload graphs as an ONNX file
    (``--param k=v`` sets builder arguments; ``--inputs-out`` writes seeded
    inputs as .npz).

Exit codes: 0 success, 1 verification mismatch, 2 usage or model error.
"""
from __future__ import annotations

import argparse
import ast
import sys
from pathlib import Path

import numpy as np

from . import workloads as W
from .lowering import UnsupportedOpError, lower
from .onnx_reader import OnnxFormatError, infer_types, read_onnx
from .plan import B200PlanEmitter, load_plan, save_plan
from .refbin import DEFAULT_LARGE_WEIGHT_THRESHOLD, constants_from_bin
from .verify import check_output

WORKLOADS = {n: getattr(W, n) for n in (
    "qconv_stack_int8", "llama_mlp_int4", "mlp_fp32", "lstm_fp32", "attention_fp16", "matmul_nbits_f16",
    "swish_mul_f16", "qlinear_matmul_u8", "matmul_integer_u8", "conv_f32", "softmax_f32", "quant_dequant")}


class CliError(Exception):
    pass


def parse_input_dims(items) -> dict[str, int]:
    """``--input-dim`` values: ``name=V`` or ``value:axis=V`` (V >= 1)."""
    out = {}
    for item in items or ():
        key, sep, val = item.partition("=")
        if not sep or not key or not val.isdigit() or int(val) < 1:
            raise CliError(f"--input-dim {item!r}: expected NAME=INT or INPUT:AXIS=INT with INT >= 1")
        if ":" in key:
            name, _, axis = key.rpartition(":")
            if not name or not axis.isdigit():
                raise CliError(f"--input-dim {item!r}: bad axis")
        out[key] = int(val)
    return out


def _emitter(args) -> B200PlanEmitter:
    return B200PlanEmitter(use_tensor_cores=not args.no_tensor_cores,
                           nbits_rounded_dequant=args.nbits_rounded_dequant,
                           attention_mode=getattr(args, "attention_mode", "exact"))


def compile_model(model_path, dim_values=None, weights_bin=None, threshold=DEFAULT_LARGE_WEIGHT_THRESHOLD,
                  model_name=None, emitter=None):
    """ONNX file -> Plan (in memory)."""
    try:
        spec = infer_types(read_onnx(model_path, dim_values))
    except OnnxFormatError as e:
        raise CliError(f"{model_path}: {e}") from e
    if model_name:
        spec.name = model_name
    try:
        model = lower(spec)
    except UnsupportedOpError as e:
        raise CliError(f"{model_path}: {e}") from e
    if weights_bin is not None:
        try:
            model = constants_from_bin(model, Path(weights_bin).read_bytes(), threshold)
        except ValueError as e:
            raise CliError(f"{weights_bin}: {e}") from e
    return (emitter or B200PlanEmitter()).emit_plan(model)


def _load_npz(path) -> dict[str, np.ndarray]:
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def _session(plan, device, weights_path=None):
    from .runtime import Session  # loads the CUDA library: fails loudly when it is missing
    return Session(plan, device=device, weights_path=weights_path)


def _plan_and_weights(target: Path, args):
    if target.suffix == ".onnx":
        plan = compile_model(target, parse_input_dims(args.input_dim), args.weights_bin,
                             args.large_weight_threshold, emitter=_emitter(args))
        return plan, None
    prefix = target.with_suffix("") if target.suffix in (".plan", ".json", ".weights") else target
    if not prefix.with_suffix(".plan").exists():
        raise CliError(f"{target}: neither an .onnx file nor a compiled plan ({prefix}.plan)")
    return load_plan(prefix)


def _check_inputs(plan, inputs):
    missing = [n for n in plan.input_names if n not in inputs]
    if missing:
        raise CliError(f"inputs file lacks {missing} (has {sorted(inputs)})")


def cmd_compile(args) -> int:
    plan = compile_model(args.model, parse_input_dims(args.input_dim), args.weights_bin,
                         args.large_weight_threshold, args.model_name, _emitter(args))
    out = Path(args.output) if args.output else args.model.parent
    paths = save_plan(plan, out, args.model_name or plan.name)
    print(plan.describe())
    print(" ".join(str(p) for p in paths.values()))
    return 0


def cmd_run(args) -> int:
    plan, wpath = _plan_and_weights(Path(args.plan), args)
    inputs = _load_npz(args.inputs)
    _check_inputs(plan, inputs)
    sess = _session(plan, args.device, wpath)
    outs = sess.run(inputs)
    np.savez(args.outputs, **outs)
    print(f"{plan.name}: {len(outs)} outputs -> {args.outputs}")
    return 0


def cmd_verify(args) -> int:
    plan, wpath = _plan_and_weights(Path(args.model), args)
    inputs, expected = _load_npz(args.inputs), _load_npz(args.expected)
    _check_inputs(plan, inputs)
    sess = _session(plan, args.device, wpath)
    outs = sess.run(inputs)
    checks = []
    for name in plan.output_names:
        if name not in expected:
            raise CliError(f"expected-outputs file lacks {name!r}")
        checks.append(check_output(name, outs[name], expected[name], args.max_ulp, args.atol_eps))
    worst = max((c.max_ulp or 0 for c in checks), default=0)
    if all(c.ok for c in checks):
        print(f"OK (max ULP {worst})")
        return 0
    for c in checks:
        if not c.ok:
            print(c.message)
    return 1


def _param(v: str):
    try:
        return ast.literal_eval(v)
    except (ValueError, SyntaxError):
        return v


def cmd_export(args) -> int:
    from .onnx_writer import write_onnx
    params = {}
    for item in args.param or ():
        k, sep, v = item.partition("=")
        if not sep:
            raise CliError(f"--param {item!r}: expected KEY=VALUE")
        params[k] = _param(v)
    try:
        wl = WORKLOADS[args.workload](**params)
    except (TypeError, ValueError) as e:
        raise CliError(f"{args.workload}: {e}") from e
    write_onnx(wl.graph, args.output)
    print(f"{args.workload} -> {args.output}")
    if args.inputs_out:
        np.savez(args.inputs_out, **wl.make_inputs(args.seed))
        print(f"inputs (seed {args.seed}) -> {args.inputs_out}")
    return 0


def _common(p):
    p.add_argument("--target", choices=["b200"], default="b200",
                   help="emit target: a B200 launch plan (the reference CLI's C target stays with the reference)")
    p.add_argument("--input-dim", action="append", default=[],
                   help="pin a dynamic dimension: NAME=INT (every axis named NAME) or INPUT:AXIS=INT")
    p.add_argument("--weights-bin", type=Path, default=None,
                   help="take the large constants from the reference's <model>.bin")
    p.add_argument("--large-weight-threshold", type=int, default=DEFAULT_LARGE_WEIGHT_THRESHOLD,
                   help="the threshold the .bin was written with (default: 102400; 0 = all inline)")
    p.add_argument("--no-tensor-cores", action="store_true",
                   help="plan the integer convolutions on the CUDA-core kernels")
    p.add_argument("--nbits-rounded-dequant", action="store_true",
                   help="MatMulNBits: one fp16 MMA per K slice on rounded dequantised weights (faster, "
                        "not bit-compatible with the reference's fp32 dequantisation)")
    p.add_argument("--attention-mode", choices=["exact", "tensor"], default="exact",
                   help="Attention: the reference's fp16 rounding bit for bit (exact), or tensor cores with "
                        "fp32 accumulation for 128-wide heads (tensor)")


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="python -m emx_onnx_cgen_b200", description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="command", required=True)
    c = sub.add_parser("compile", help="compile an ONNX model into a B200 launch plan")
    c.add_argument("model", type=Path)
    c.add_argument("-o", "--output", default=None, help="output directory (default: the model's directory)")
    c.add_argument("--model-name", default=None, help="plan file stem / model name (default: the graph name)")
    _common(c)
    c.set_defaults(func=cmd_compile)
    r = sub.add_parser("run", help="run a compiled plan (or an .onnx model) on one GPU")
    r.add_argument("plan", help="plan path without extension, or an .onnx model")
    r.add_argument("--inputs", required=True)
    r.add_argument("--outputs", required=True)
    r.add_argument("--device", type=int, default=0)
    _common(r)
    r.set_defaults(func=cmd_run)
    v = sub.add_parser("verify", help="run on the GPU and compare with expected outputs")
    v.add_argument("model", help="an .onnx model or a compiled plan path")
    v.add_argument("--inputs", required=True)
    v.add_argument("--expected", required=True)
    v.add_argument("--max-ulp", type=int, default=100)
    v.add_argument("--atol-eps", type=float, default=1.0)
    v.add_argument("--device", type=int, default=0)
    _common(v)
    v.set_defaults(func=cmd_verify)
    e = sub.add_parser("export", help="write a built-in workload graph as an ONNX file")
    e.add_argument("workload", choices=sorted(WORKLOADS))
    e.add_argument("output")
    e.add_argument("--param", action="append", default=[], help="builder argument KEY=VALUE (Python literal)")
    e.add_argument("--inputs-out", default=None, help="also write seeded inputs (.npz)")
    e.add_argument("--seed", type=int, default=0)
    e.set_defaults(func=cmd_export)
    return ap


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    try:
        return args.func(args)
    except CliError as e:
        print(f"error: {e}", file=sys.stderr)
        return 2


if __name__ == "__main__":
    sys.exit(main())

"""Generate the golden input/output vectors in this directory.

Each case builds a small instance of one workload graph (or reads one of the
reference's own test models), has the REFERENCE
compiler (imported from its source tree through the test-only onnx shim in
``oracle/onnx_shim.py``) lower it and emit C, compiles that C with
``gcc -std=c99 -O2`` and runs it on seeded inputs.  The graph's initializers,
inputs and the reference outputs are stored as ``<case>.npz``; ``cases.json``
records the builder arguments.  The fixtures pin both the oracle restatement
(``oracle/oracle.c``) and the CUDA kernels without needing the reference at
test time.

Run from the repository root with the reference's ``src`` directory in
``EMX_REFERENCE_SRC`` (default: ``reference/src`` beside this repository)::

    python tests/golden/make_golden.py [case ...]   # all cases, or only the named ones
"""
from __future__ import annotations

import json
import platform
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from emx_onnx_cgen_b200 import workloads as W  # noqa: E402
from oracle import refc  # noqa: E402

# (case name, builder, kwargs, input seed)
CASES = [
    ("qconv_b2_c64_12x12", "qconv_stack_int8", dict(batch=2, channels=64, height=12, width=12), 0),
    ("qconv_b1_c64_7x9_lowgain", "qconv_stack_int8",
     dict(batch=1, channels=64, height=7, width=9, wscale_range=(0.0001, 0.001)), 1),
    ("qconv_b1_c16_5x5_3conv", "qconv_stack_int8",
     dict(batch=1, channels=16, height=5, width=5, n_convs=3, wscale_range=(0.0001, 0.001)), 2),
    ("qconv_b2_c32_16x16_lowgain", "qconv_stack_int8",
     dict(batch=2, channels=32, height=16, width=16, wscale_range=(0.0001, 0.001)), 3),
    ("mlp_m4_k32_h64", "mlp_fp32", dict(m=4, k=32, hidden=64), 0),
    ("mlp_m5_k48_h80", "mlp_fp32", dict(m=5, k=48, hidden=80), 1),
    ("nbits_m4_k64_n96", "llama_mlp_int4", dict(m=4, hidden=64, inter=96), 0),
    ("nbits_m3_k128_n160", "llama_mlp_int4", dict(m=3, hidden=128, inter=160), 1),
    ("attn_b1_h2_t16_d8", "attention_fp16", dict(batch=1, heads=2, seq=16, head_dim=8), 0),
    ("attn_b1_h2_t64_d128", "attention_fp16", dict(batch=1, heads=2, seq=64, head_dim=128), 1),
    ("attn_b1_h1_t33_d64", "attention_fp16", dict(batch=1, heads=1, seq=33, head_dim=64), 2),
    ("lstm_t3_b2_i8_h16", "lstm_fp32", dict(seq=3, batch=2, input_size=8, hidden=16), 0),
    ("lstm_t5_b3_i16_h32", "lstm_fp32", dict(seq=5, batch=3, input_size=16, hidden=32), 1),
    ("nbits1_m5_k96_n40_zpblock_bias", "matmul_nbits_f16",
     dict(m=5, k=96, n=40, block=32, zero_points="block", bias=True), 0),
    ("nbits1_m3_k64_n24_zpcol_b16", "matmul_nbits_f16", dict(m=3, k=64, n=24, block=16, zero_points="column"), 1),
    ("nbits1_m2_k256_n16_b128", "matmul_nbits_f16", dict(m=2, k=256, n=16, block=128), 2),
    # accuracy_level 4: the int8 activation path (matmul_nbits_int8_op.c.j2)
    ("nbits8_m5_k96_n40_zpblock_bias", "matmul_nbits_f16",
     dict(m=5, k=96, n=40, block=32, zero_points="block", bias=True, accuracy_level=4), 0),
    ("nbits8_m3_k64_n24_zpcol_b16", "matmul_nbits_f16",
     dict(m=3, k=64, n=24, block=16, zero_points="column", accuracy_level=4), 1),
    ("nbits8_m4_k80_n16_partial", "matmul_nbits_f16", dict(m=4, k=80, n=16, block=32, accuracy_level=4), 2),
    ("nbits8_m2_k256_n24_b128", "matmul_nbits_f16", dict(m=2, k=256, n=24, block=128, accuracy_level=4), 3),
    ("swishmul_8x24", "swish_mul_f16", dict(shape=(8, 24)), 0),
    ("swishmul_5x16_alpha1702", "swish_mul_f16", dict(shape=(5, 16), alpha=1.702), 1),
    ("qmm_m5_k40_n24", "qlinear_matmul_u8", dict(m=5, k=40, n=24), 0),
    ("qmm_m3_k17_n9_u8b", "qlinear_matmul_u8", dict(m=3, k=17, n=9, a_zero=100, b_dtype="u8", b_zero=120), 1),
    ("qmm_m4_k20_n7_intrequant", "qlinear_matmul_u8", dict(m=4, k=20, n=7, scales=(0.5, 0.25, 4.0)), 2),
    ("mmi_m4_k33_n10", "matmul_integer_u8", dict(m=4, k=33, n=10), 0),
    # K a multiple of 16: the tensor-core path
    ("qmm_m6_k64_n40", "qlinear_matmul_u8", dict(m=6, k=64, n=40), 3),
    ("qmm_m5_k48_n20_u8b_intrequant", "qlinear_matmul_u8",
     dict(m=5, k=48, n=20, a_zero=7, b_dtype="u8", b_zero=130, scales=(0.5, 0.25, 4.0)), 4),
    ("mmi_m4_k32_n24", "matmul_integer_u8", dict(m=4, k=32, n=24), 1),
    ("conv_b2_c4_9x7_s2", "conv_f32", dict(batch=2, cin=4, cout=6, h=9, w=7, stride=2, pad=1), 0),
    ("conv_b1_c4_8x8_g2_d2", "conv_f32", dict(batch=1, cin=4, cout=4, h=8, w=8, pad=2, dilation=2, group=2), 1),
    ("softmax_4x37", "softmax_f32", dict(shape=(4, 37)), 0),
    ("softmax_3x5x6_axis1", "softmax_f32", dict(shape=(3, 5, 6), axis=1), 1),
    ("qdq_u8_6x11", "quant_dequant", dict(shape=(6, 11)), 0),
    ("qdq_i8_4x9", "quant_dequant", dict(shape=(4, 9), out_dtype="i8", zero=-3, scale=0.05), 1),
    ("maxpool_i8_2x8x13x11_k3x2_s2x1", "pool8", dict(), 0),
    ("maxpool_u8_1x4x9x9_d2_ceil", "pool8",
     dict(shape=(1, 4, 9, 9), kernel=(3, 3), strides=(2, 2), pads=(1, 1, 0, 0), dilations=(2, 2), ceil_mode=1,
          dtype="u8"), 1),
    ("maxpool_i8_same_upper", "pool8",
     dict(shape=(2, 3, 10, 7), kernel=(4, 3), strides=(3, 2), auto_pad="SAME_UPPER"), 2),
    ("qavgpool_i8_2x8x13x11_k3x2", "pool8", dict(kind="avg"), 0),
    ("qavgpool_u8_pad_count", "pool8",
     dict(shape=(2, 5, 12, 10), kind="avg", kernel=(3, 3), strides=(2, 2), pads=(1, 1, 1, 1),
          count_include_pad=1, dtype="u8", x_zero=128, y_zero=120, x_scale=0.02, y_scale=0.015), 1),
    ("qavgpool_i8_to_u8_ceil", "pool8",
     dict(shape=(1, 6, 11, 9), kind="avg", kernel=(2, 2), strides=(2, 2), pads=(0, 0, 0, 0), ceil_mode=1,
          y_dtype="u8", y_zero=128, y_scale=0.05), 2),
    ("qsoftmax_u8_6x37", "qlinear_softmax8", dict(), 0),
    ("qsoftmax_i8_4x5x12_axis1", "qlinear_softmax8",
     dict(shape=(4, 5, 12), axis=1, dtype="i8", x_zero=-5, x_scale=0.11, y_zero=-128), 1),
    ("qsoftmax_u8_3x4x6_opset11", "qlinear_softmax8",
     dict(shape=(3, 4, 6), axis=1, opset=11, x_scale=0.03, x_zero=100), 2),
    ("transpose_f32_2x3x4x5", "transpose", dict(), 0),
    ("transpose_u8_perm_rev", "transpose", dict(shape=(3, 5, 7), perm=(2, 0, 1), dtype="u8"), 1),
]

# whole models from the reference's own test tree: (case name, path inside the
# reference project, input seed).  The graph is stored with the fixture (nodes
# in cases.json, initializers in the .npz), so tests need neither the model
# file nor the reference.
MODEL_CASES = [
    ("kws_qoperator", "tests/onnx/micro_kws_m_static_qoperator.onnx", 0),
]
MODEL_SAMPLES = 32  # seeded input sets per model, stacked on a leading sample axis


def _json_attr(v):
    if isinstance(v, (bool, int, float, str)):
        return v
    if isinstance(v, (list, tuple)) and all(isinstance(x, (bool, int, float, str)) for x in v):
        return list(v)
    raise TypeError(f"attribute value {v!r} has no JSON form")


def graph_json(spec) -> dict:
    return {
        "name": spec.name,
        "inputs": [[t.name, t.dtype, list(t.shape)] for t in spec.inputs],
        "outputs": [[t.name, t.dtype, list(t.shape)] for t in spec.outputs],
        "values": [[t.name, t.dtype, list(t.shape)] for t in spec.values],
        "nodes": [[n.op_type, n.name, list(n.inputs), list(n.outputs),
                   {k: _json_attr(v) for k, v in n.attrs.items()}, n.domain] for n in spec.nodes],
        "opset_imports": [list(o) for o in spec.opset_imports],
    }


def _smooth_field(rng, shape, lo: float, hi: float) -> np.ndarray:
    """Gaussian-filtered noise over the last two axes (a spectrogram-like
    field), its mean and spread drawn inside [lo, hi]."""
    f = np.fft.fft2(rng.standard_normal(shape))
    ky = np.fft.fftfreq(shape[-2])[:, None]
    kx = np.fft.fftfreq(shape[-1])[None, :]
    f *= np.exp(-(ky ** 2 + kx ** 2) * rng.uniform(20, 120))
    x = np.real(np.fft.ifft2(f))
    x = x / (x.std() + 1e-12)
    mid, half = (lo + hi) / 2, (hi - lo) / 2
    return mid + rng.uniform(-0.2, 0.2) * half + x * half * rng.uniform(0.25, 0.5)


def model_inputs(spec, seed: int) -> dict:
    """Seeded inputs over the range the model's first quantizer covers: every
    fourth set uniform over that whole range and a little past both ends (so
    saturation is hit), the others smooth fields laid out as the image the
    input is reshaped to (noise alone drives the keyword model to one class)."""
    rng = np.random.default_rng(seed)
    out = {}
    for t in spec.inputs:
        lo, hi, image = -1.0, 1.0, tuple(t.shape)
        names = {t.name}
        for n in spec.nodes:
            if n.op_type == "Reshape" and n.inputs[0] in names:
                names.add(n.outputs[0])
                tgt = [int(v) for v in np.asarray(spec.initializers[n.inputs[1]]).reshape(-1)]
                if len(tgt) == 4 and -1 not in tgt[1:]:
                    image = tuple(tgt[1:])
            if n.op_type == "QuantizeLinear" and n.inputs[0] in names:
                s = float(np.asarray(spec.initializers[n.inputs[1]]).reshape(-1)[0])
                zp = np.asarray(spec.initializers[n.inputs[2]]).reshape(-1)[0]
                qlo, qhi = (-128, 127) if zp.dtype == np.int8 else (0, 255)
                lo, hi = (qlo - 2 - int(zp)) * s, (qhi + 2 - int(zp)) * s
                break
        if seed % 4 == 3 or len(image) < 2:
            x = rng.uniform(lo, hi, size=t.shape)
        else:
            x = _smooth_field(rng, image, lo, hi).reshape(t.shape)
        out[t.name] = x.astype(np.float32)
    return out


def main() -> None:
    if not refc.reference_available():
        raise SystemExit(f"reference source not found at {refc.REFERENCE_SRC}")
    gcc = subprocess.run(["gcc", "--version"], capture_output=True, text=True).stdout.splitlines()[0]
    libc = " ".join(platform.libc_ver())
    index = {"generator": "reference generated C, gcc -std=c99 -O2", "gcc": gcc, "libc": libc,
             "cases": {}}
    only = set(sys.argv[1:])
    if only and (HERE / "cases.json").exists():
        index["cases"] = json.loads((HERE / "cases.json").read_text())["cases"]
    with tempfile.TemporaryDirectory() as tmp:
        for name, builder, kwargs, seed in CASES:
            if only and name not in only:
                continue
            wl = W.BUILDERS[builder](**kwargs)
            tag = "g_" + name
            refc.build(wl.graph, tag, Path(tmp))
            model = refc.RefCModel(tag, Path(tmp))
            inputs = wl.make_inputs(seed)
            outputs = model.run(inputs)
            arrays = {f"init:{k}": v for k, v in wl.graph.initializers.items()}
            arrays.update({f"in:{k}": v for k, v in inputs.items()})
            arrays.update({f"out:{k}": v for k, v in outputs.items()})
            np.savez_compressed(HERE / f"{name}.npz", **arrays)
            index["cases"][name] = {"builder": builder,
                                    "kwargs": {k: list(v) if isinstance(v, tuple) else v
                                               for k, v in kwargs.items()},
                                    "seed": seed}
            print(name, {k: v.shape for k, v in outputs.items()})
        from emx_onnx_cgen_b200.onnx_reader import infer_types, read_onnx
        for name, rel, seed in MODEL_CASES:
            if only and name not in only:
                continue
            spec = infer_types(read_onnx(refc.REFERENCE_SRC.parent / rel))
            tag = "g_" + name
            refc.build(spec, tag, Path(tmp))
            model = refc.RefCModel(tag, Path(tmp))
            runs = []
            for i in range(MODEL_SAMPLES):
                inputs = model_inputs(spec, seed + i)
                runs.append((inputs, model.run(inputs)))
            arrays = {f"init:{k}": v for k, v in spec.initializers.items()}
            arrays.update({f"in:{k}": np.stack([r[0][k] for r in runs]) for k in runs[0][0]})
            arrays.update({f"out:{k}": np.stack([r[1][k] for r in runs]) for k in runs[0][1]})
            outputs = runs[0][1]
            np.savez_compressed(HERE / f"{name}.npz", **arrays)
            index["cases"][name] = {"model": rel, "seed": seed, "samples": MODEL_SAMPLES,
                                    "graph": graph_json(spec)}
            print(name, {k: v.shape for k, v in outputs.items()})
    (HERE / "cases.json").write_text(json.dumps(index, indent=1) + "\n")


if __name__ == "__main__":
    main()

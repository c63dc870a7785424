"""ONNX Attention (opset 23) fp16 on the B200 kernel: bit-identical to the
reference's generated C (golden fixtures) and to the CPU restatement, which
repeats the reference's statement-by-statement fp16 rounding.  Covers causal
and non-causal, sequence lengths off the 16-row / 64- and 128-key tiles,
head sizes 8..128 (both kernels), and inputs with inf / NaN / overflowing scores (the path that
evaluates masked keys with the reference's mask arithmetic)."""
import numpy as np
import pytest

from emx_onnx_cgen_b200 import workloads as W
from emx_onnx_cgen_b200.runtime import Session
from golden_util import cases, load
from gpu_util import assert_bitexact, plan_for, require_gpu
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(n for n in cases() if n.startswith("attn")))
def test_golden(name):
    require_gpu()
    wl, inputs, ref = load(name)
    out = Session(plan_for(wl)).run(inputs)
    assert_bitexact(out["Y"], ref["Y"], name)


@pytest.mark.parametrize("kw", [
    dict(batch=2, heads=3, seq=100, head_dim=64),
    dict(batch=1, heads=2, seq=257, head_dim=128),
    dict(batch=1, heads=1, seq=77, head_dim=32, causal=False),
    dict(batch=3, heads=1, seq=16, head_dim=8),
    dict(batch=1, heads=1, seq=1, head_dim=16),
    dict(batch=1, heads=2, seq=70, head_dim=12),  # D not a multiple of 8: the 64-key-tile kernel
])
def test_vs_port(kw):
    require_gpu()
    wl = W.attention_fp16(**kw)
    x = wl.make_inputs(5)
    ref = oracle.run_graph(wl.graph, x)["Y"]
    out = Session(plan_for(wl)).run(x)["Y"]
    assert_bitexact(out, ref, str(kw))


@pytest.mark.parametrize("case", ["inf_k", "nan_v", "overflow", "neg_zero_v"])
def test_specials(case):
    require_gpu()
    wl = W.attention_fp16(batch=1, heads=2, seq=40, head_dim=16)
    x = wl.make_inputs(7)
    if case == "inf_k":
        x["K"][0, 0, 30, 3] = np.inf          # a masked key for rows < 30
    elif case == "nan_v":
        x["V"][0, 1, 35, 5] = np.nan
    elif case == "overflow":
        x["Q"][0, 0] *= np.float16(60)        # partial scores beyond fp16 range
        x["K"][0, 0] *= np.float16(60)
    elif case == "neg_zero_v":
        x["V"][0, 0, 0, :] = -0.0
        x["V"][0, 0, 1:, :] = np.abs(x["V"][0, 0, 1:, :])
    ref = oracle.run_graph(wl.graph, x)["Y"]
    out = Session(plan_for(wl)).run(x)["Y"]
    assert_bitexact(out, ref, case)


def test_full_size_heads():
    """Q, K, V [8, 32, 2048, 128], causal: heads are independent, so the CPU
    restatement checks a sample of (batch, head) pairs."""
    require_gpu()
    wl = W.attention_fp16()
    x = wl.make_inputs(0)
    out = Session(plan_for(wl)).run(x)["Y"]
    one = W.attention_fp16(batch=1, heads=1)
    for b, h in [(0, 0), (7, 31)]:
        xi = {k: np.ascontiguousarray(v[b:b + 1, h:h + 1]) for k, v in x.items()}
        ref = oracle.run_graph(one.graph, xi)["Y"]
        assert_bitexact(out[b:b + 1, h:h + 1], ref, f"b={b} h={h}")

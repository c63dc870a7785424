"""The onnx.backend-style adapter on the host: device strings, planning from a
ModelProto-like object / bytes / path (the same plan bytes as the in-memory
emitter), dynamic dimensions, and rejection of CPU devices and of ops
without a B200 kernel (reference surface:
src/emx_onnx_cgen/onnx_backend/backend.py:549-660)."""
import pytest

from emx_onnx_cgen_b200 import onnx_backend as ob, workloads as W
from emx_onnx_cgen_b200.lowering import UnsupportedOpError
from emx_onnx_cgen_b200.onnx_writer import write_onnx, write_onnx_bytes
from emx_onnx_cgen_b200.spec import GraphSpec, NodeSpec, TensorSpec
from gpu_util import plan_for


class _Proto:
    """Stands in for onnx.ModelProto: only SerializeToString is used."""

    def __init__(self, data: bytes):
        self._data = data

    def SerializeToString(self) -> bytes:  # noqa: N802
        return self._data


@pytest.mark.parametrize("device,ordinal", [("CUDA", 0), ("cuda:0", 0), ("CUDA:3", 3), (" CUDA:1 ", 1)])
def test_device_strings(device, ordinal):
    assert ob.parse_device(device) == ordinal
    assert ob.supports_device(device)


@pytest.mark.parametrize("device", ["CPU", "GPU", "CUDA:x", "", "cuda:-1"])
def test_rejected_devices(device):
    assert not ob.supports_device(device)
    with pytest.raises(RuntimeError, match="Unsupported device"):
        ob.parse_device(device)
    assert not ob.is_compatible(b"", device)


def test_plan_from_each_model_form(tmp_path):
    wl = W.qconv_stack_int8(batch=2, channels=32, height=8, width=8)
    want = plan_for(wl)
    data = write_onnx_bytes(wl.graph)
    write_onnx(wl.graph, tmp_path / "m.onnx")
    for model in (data, bytearray(data), _Proto(data), tmp_path / "m.onnx", str(tmp_path / "m.onnx")):
        got = ob.compile_plan(model)
        assert got.plan_bytes == want.plan_bytes and got.weight_bytes == want.weight_bytes
    assert ob.is_compatible(_Proto(data), "CUDA")
    with pytest.raises(TypeError):
        ob.compile_plan(12345)


def test_dynamic_batch_pinned():
    wl = W.mlp_fp32(m=4, k=64, hidden=128)
    g = wl.graph
    dyn = {t.name: {0: "batch"} for t in (*g.inputs, *g.outputs)}
    plan = ob.compile_plan(write_onnx_bytes(g, dim_params=dyn), input_dims={"batch": 4})
    assert plan.plan_bytes == plan_for(wl).plan_bytes


def test_unsupported_op_is_reported():
    g = GraphSpec(name="hard", inputs=[TensorSpec("x", "f32", (4,))], outputs=[TensorSpec("y", "f32", (4,))],
                  nodes=[NodeSpec("Hardmax", "n0", ("x",), ("y",), {}, None)], initializers={}, values=[],
                  opset_imports=(("", 17),))
    data = write_onnx_bytes(g)
    with pytest.raises(UnsupportedOpError):
        ob.compile_plan(data)
    assert not ob.is_compatible(data, "CUDA")

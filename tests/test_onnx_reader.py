"""The ONNX reader (no `onnx` package): wire-format round trips on
hand-built messages, and -- where the reference source tree is present --
its in-tree model fixtures parsed, lowered by the reference compiler, and
(for the ops this backend has kernels for) planned identically from both
lowerings."""
import struct
from pathlib import Path

import numpy as np
import pytest

from emx_onnx_cgen_b200 import lowering, workloads as W
from emx_onnx_cgen_b200.onnx_reader import OnnxFormatError, infer_types, read_onnx, read_onnx_bytes
from emx_onnx_cgen_b200.plan import B200PlanEmitter
from oracle import refc


def _key(num, wt):
    return _vint((num << 3) | wt)


def _vint(v):
    out = bytearray()
    v &= (1 << 64) - 1
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _ld(num, payload: bytes):
    return _key(num, 2) + _vint(len(payload)) + payload


def _str(num, s):
    return _ld(num, s.encode())


def _tensor_msg(name, arr, raw=True):
    dt = {np.float32: 1, np.uint8: 2, np.int8: 3, np.int32: 6, np.int64: 7, np.float16: 10}[arr.dtype.type]
    m = b"".join(_key(1, 0) + _vint(d) for d in arr.shape) + _key(2, 0) + _vint(dt) + _str(8, name)
    if raw:
        m += _ld(9, arr.tobytes())
    elif arr.dtype == np.float32:
        m += _ld(4, arr.astype("<f4").tobytes())
    else:
        m += _ld(7 if arr.dtype == np.int64 else 5, b"".join(_vint(int(v)) for v in arr.reshape(-1)))
    return m


def _vi(name, elem, dims):
    """ValueInfoProto: name, TypeProto{tensor_type{elem_type, shape{dim*}}}."""
    shape = b"".join(_ld(1, _key(1, 0) + _vint(d) if isinstance(d, int) else _str(2, d)) for d in dims)
    tensor_type = _key(1, 0) + _vint(elem) + _ld(2, shape)
    return _str(1, name) + _ld(2, _ld(1, tensor_type))


def _model():
    w = np.arange(12, dtype=np.float32).reshape(3, 4)
    node = (_str(1, "X") + _str(1, "W") + _str(2, "Y") + _str(3, "mm") + _str(4, "Gemm")
            + _ld(5, _str(1, "transB") + _key(3, 0) + _vint(1) + _key(20, 0) + _vint(2))
            + _ld(5, _str(1, "alpha") + _key(2, 5) + struct.pack("<f", 0.5) + _key(20, 0) + _vint(1))
            + _ld(5, _str(1, "perm") + _ld(8, _vint(2) + _vint(0)) + _key(20, 0) + _vint(7)))
    graph = (_ld(1, node) + _str(2, "g") + _ld(5, _tensor_msg("W", w))
             + _ld(5, _tensor_msg("b", np.array([-1, 2], np.int64), raw=False))
             + _ld(11, _vi("X", 1, ["batch", 4])) + _ld(12, _vi("Y", 1, ["batch", 3])))
    opset = _ld(8, _str(1, "") + _key(2, 0) + _vint(17))
    return _key(1, 0) + _vint(8) + _ld(7, graph) + opset, w


def test_reader_decodes_hand_built_model():
    data, w = _model()
    g = read_onnx_bytes(data, dim_values={"batch": 5})
    assert g.name == "g" and g.opset_imports == (("", 17),)
    assert [(t.name, t.dtype, t.shape) for t in g.inputs] == [("X", "f32", (5, 4))]
    assert [(t.name, t.shape) for t in g.outputs] == [("Y", (5, 3))]
    np.testing.assert_array_equal(g.initializers["W"], w)
    np.testing.assert_array_equal(g.initializers["b"], np.array([-1, 2], np.int64))
    n = g.nodes[0]
    assert n.op_type == "Gemm" and n.inputs == ("X", "W") and n.outputs == ("Y",)
    assert n.attrs["transB"] == 1 and n.attrs["alpha"] == 0.5 and n.attrs["perm"] == [2, 0]


def test_reader_errors():
    data, _ = _model()
    with pytest.raises(OnnxFormatError, match="symbolic dimension"):
        read_onnx_bytes(data)
    with pytest.raises(OnnxFormatError):
        read_onnx_bytes(data[: len(data) // 2], dim_values={"batch": 1})


FIXTURES = Path(refc.REFERENCE_SRC).parent / "tests" / "onnx"


@pytest.mark.parametrize("name", ["micro_kws_m_static_qoperator.onnx", "micro_kws_m_static_fp32.onnx",
                                  "micro_kws_m_qoperator_avg_pool.onnx"])
def test_reference_fixture_lowers(name):
    if not (FIXTURES / name).exists():
        pytest.skip("reference fixtures not present")
    g = infer_types(read_onnx(FIXTURES / name))
    model, lowered = refc.lower(g)
    assert len(lowered.ops) >= len(g.nodes) - 2  # the reference may fold reshapes
    assert tuple(lowered.output_shapes[0]) == (1, 10)

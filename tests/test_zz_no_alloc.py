"""The allocation-free standalone QLinearConv entry point
(emx_b200_qlinear_conv3x3_noalloc, static device scratch) against the plan
entry point (emx_b200_run) on the same single QLinearConv: identical output
bytes on two calls in a row, over the accepted channel pairs (c == oc and
c != oc), both input zero points (0: raw bytes, 128: recentred), with and
without a bias, on a created stream and on the legacy default stream (NULL);
the device's free memory does not move across calls; and a clear rejection
of a geometry larger than the static scratch.  Collected last so that it also
runs after every other GPU test has used the library."""
import ctypes

import numpy as np
import pytest

from emx_onnx_cgen_b200 import kernel_ids as K
from emx_onnx_cgen_b200.runtime import Session, load_library
from emx_onnx_cgen_b200.spec import GraphSpec, NodeSpec, TensorSpec
from emx_onnx_cgen_b200.workloads import Workload
from gpu_util import assert_bitexact, plan_for, require_gpu

pytestmark = pytest.mark.gpu

EMX_OK, EMX_ERR_INVALID_ARGUMENT = 0, 1


def _noalloc(lib):
    f = lib.emx_b200_qlinear_conv3x3_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_int,
                  ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    lib.emx_b200_last_error.restype = ctypes.c_char_p
    return f


def single_conv(n, c, oc, h, w, x_zero, with_bias, seed=3):
    """One QLinearConv 3x3 / stride 1 / pads 1: uint8 NCHW in and out, int8
    weights with per-channel scales (low gain, so outputs are not saturated)."""
    rng = np.random.default_rng(seed)
    inits = {
        "xs": np.asarray(0.02, np.float32).reshape(()), "xz": np.asarray(x_zero, np.uint8).reshape(()),
        "w": rng.integers(-127, 128, (oc, c, 3, 3)).astype(np.int8),
        "ws": rng.uniform(0.0001, 0.001, oc).astype(np.float32), "wz": np.zeros(oc, np.int8),
        "ys": np.asarray(0.02, np.float32).reshape(()), "yz": np.asarray(3, np.uint8).reshape(()),
    }
    ins = ["X", "xs", "xz", "w", "ws", "wz", "ys", "yz"]
    if with_bias:
        inits["b"] = rng.integers(-1000, 1001, oc).astype(np.int32)
        ins.append("b")
    g = GraphSpec(name="single_qconv", inputs=[TensorSpec("X", "u8", (n, c, h, w))],
                  outputs=[TensorSpec("Y", "u8", (n, oc, h, w))],
                  nodes=[NodeSpec("QLinearConv", "conv", tuple(ins), ("Y",),
                                  {"kernel_shape": [3, 3], "pads": [1, 1, 1, 1], "strides": [1, 1]})],
                  initializers=inits, opset_imports=(("", 17),))

    def make_inputs(s=0):
        return {"X": np.random.default_rng(s).integers(0, 256, (n, c, h, w)).astype(np.uint8)}

    return Workload("single_qconv", g, make_inputs, {"X": 0, "Y": 0}, {})


CASES = [  # n, c, oc, h, w, x_zero, bias
    (2, 64, 64, 12, 12, 128, True),
    (3, 32, 32, 9, 17, 128, True),
    (1, 128, 128, 7, 5, 128, True),
    (2, 32, 64, 10, 11, 128, True),
    (2, 64, 32, 8, 9, 0, True),
    (1, 64, 128, 6, 13, 0, False),
    (2, 128, 64, 5, 7, 128, False),
    (3, 64, 64, 11, 6, 0, False),
]


@pytest.mark.parametrize("stream_kind", ["created", "null"])
@pytest.mark.parametrize("n,c,oc,h,w,x_zero,bias", CASES)
def test_noalloc_matches_plan_entry_point(n, c, oc, h, w, x_zero, bias, stream_kind):
    require_gpu()
    import torch
    wl = single_conv(n, c, oc, h, w, x_zero, bias)
    plan = plan_for(wl)
    assert any(op.kernel == K.K_QCONV_TC for op in plan.ops), "the plan path must use the tensor-core conv"
    g = wl.graph.initializers
    x = wl.make_inputs(11)["X"]
    ref = Session(plan).run({"X": x})["Y"]

    lib = load_library()
    f = _noalloc(lib)
    dev = torch.device("cuda", 0)
    d_x = torch.from_numpy(x).to(dev)
    d_w = torch.from_numpy(g["w"]).to(dev)
    d_ws = torch.from_numpy(g["ws"]).to(dev)
    d_b = torch.from_numpy(g["b"]).to(dev) if bias else None
    d_y = [torch.full(ref.shape, 7, dtype=torch.uint8, device=dev) for _ in range(2)]
    stream = torch.cuda.Stream(dev) if stream_kind == "created" else None
    handle = ctypes.c_void_p(stream.cuda_stream) if stream is not None else None
    torch.cuda.synchronize()

    def call(out):
        rc = f(d_x.data_ptr(), d_w.data_ptr(), d_ws.data_ptr(), d_b.data_ptr() if bias else None,
               float(g["xs"][()]), x_zero, float(g["ys"][()]), int(g["yz"][()]), n, c, h, w, oc,
               out.data_ptr(), handle)
        assert rc == EMX_OK, lib.emx_b200_last_error()

    call(d_y[0])  # first call on this device may set up the scratch address
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info(dev)[0]
    for k in range(2):
        call(d_y[k])
        torch.cuda.synchronize()
        assert_bitexact(d_y[k].cpu().numpy(), ref, f"call {k + 1}")
    for _ in range(4):
        call(d_y[1])
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(dev)[0] == free_before, "device free memory changed across calls"


def test_noalloc_rejects_geometry_beyond_scratch():
    require_gpu()
    import torch
    lib = load_library()
    f = _noalloc(lib)
    dev = torch.device("cuda", 0)
    d = torch.zeros(16, dtype=torch.uint8, device=dev)  # never read: the call is rejected first
    rc = f(d.data_ptr(), d.data_ptr(), d.data_ptr(), None, 0.02, 128, 0.02, 0, 64, 64, 56, 56, 64,
           d.data_ptr(), None)
    assert rc == EMX_ERR_INVALID_ARGUMENT
    msg = lib.emx_b200_last_error().decode()
    assert "needs" in msg and "static scratch holds" in msg, msg

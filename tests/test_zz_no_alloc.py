"""The allocation-free standalone QLinearConv entry point
(emx_b200_qlinear_conv3x3_noalloc, static device scratch) against the plan
entry point (emx_b200_run) on the same single QLinearConv: identical output
bytes on two calls in a row, and a clear rejection of a geometry larger than
the static scratch.  Collected last so that it also runs after every other
GPU test has used the library."""
import ctypes

import numpy as np
import pytest

from emx_onnx_cgen_b200 import workloads as W
from emx_onnx_cgen_b200.runtime import Session, load_library
from gpu_util import assert_bitexact, plan_for, require_gpu

pytestmark = pytest.mark.gpu

EMX_OK, EMX_ERR_INVALID_ARGUMENT = 0, 1


def _noalloc(lib):
    f = lib.emx_b200_qlinear_conv3x3_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_int,
                  ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    return f


@pytest.mark.parametrize("n,c,h,w", [(2, 64, 12, 12), (3, 32, 9, 17), (1, 128, 7, 5)])
def test_noalloc_matches_plan_entry_point(n, c, h, w):
    require_gpu()
    import torch
    wl = W.qconv_stack_int8(batch=n, channels=c, height=h, width=w, n_convs=1,
                            wscale_range=(0.0001, 0.001))
    g = wl.graph.initializers
    x = wl.make_inputs(11)["X"]
    ref = Session(plan_for(wl)).run({"X": x})["Y"]

    lib = load_library()
    f = _noalloc(lib)
    dev = torch.device("cuda", 0)
    d_x = torch.from_numpy(x).to(dev)
    d_w = torch.from_numpy(g["w0"]).to(dev)
    d_ws = torch.from_numpy(g["ws0"]).to(dev)
    d_b = torch.from_numpy(g["b0"]).to(dev)
    stream = torch.cuda.Stream(dev)
    for call in range(2):
        d_y = torch.full(ref.shape, 7, dtype=torch.uint8, device=dev)
        rc = f(d_x.data_ptr(), d_w.data_ptr(), d_ws.data_ptr(), d_b.data_ptr(), float(g["x_scale"][()]),
               int(g["x_zero"][()]), float(g["h_scale"][()]), int(g["h_zero"][()]), n, c, h, w, c,
               d_y.data_ptr(), ctypes.c_void_p(stream.cuda_stream))
        assert rc == EMX_OK, lib.emx_b200_last_error()
        stream.synchronize()
        assert_bitexact(d_y.cpu().numpy(), ref, f"call {call + 1}")


def test_noalloc_rejects_geometry_beyond_scratch():
    require_gpu()
    import torch
    lib = load_library()
    lib.emx_b200_last_error.restype = ctypes.c_char_p
    f = _noalloc(lib)
    dev = torch.device("cuda", 0)
    d = torch.zeros(16, dtype=torch.uint8, device=dev)  # never read: the call is rejected first
    rc = f(d.data_ptr(), d.data_ptr(), d.data_ptr(), None, 0.02, 128, 0.02, 0, 64, 64, 56, 56, 64,
           d.data_ptr(), None)
    assert rc == EMX_ERR_INVALID_ARGUMENT
    msg = lib.emx_b200_last_error().decode()
    assert "needs" in msg and "static scratch holds" in msg, msg

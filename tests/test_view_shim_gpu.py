"""The reference-signature C++ launchers (include/atomflow_view_ops.h), called
with reference-layout View structs exactly as src/core/engine.cu calls them."""
import ctypes

import numpy as np
import pytest

import oracle
from tests._util import assert_fp16_parity, make_gemv_case, normal_f32

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_launch_w8a16_gemv_view():
    from atomflow_b200._lib import DataType, lib, make_view
    L = lib()
    N, K = 5120, 3072
    x, q, s = make_gemv_case(77, 1, N, K)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    qd = torch.from_numpy(q).cuda()
    sd = torch.from_numpy(s.view(np.int16)).cuda()
    yd = torch.zeros(1, N, dtype=torch.int16, device="cuda")
    vx = make_view(xd.data_ptr(), DataType.FP16, [1, K])
    vw = make_view(qd.data_ptr(), DataType.FP8_E4M3, [N, K])
    vs = make_view(sd.data_ptr(), DataType.FP16, [N, K // 128])
    vy = make_view(yd.data_ptr(), DataType.FP16, [1, N])
    st = torch.cuda.current_stream().cuda_stream
    L.launch_w8a16_gemv(ctypes.byref(vx), ctypes.byref(vw), ctypes.byref(vs), ctypes.byref(vy), 128, st)
    torch.cuda.synchronize()
    assert L.af_view_last_status() == 0
    assert_fp16_parity(yd.cpu().numpy().view(np.uint16), oracle.gemv_f64(x, q, s, "group", with_l2=True), "view")
    # the drop-in is bit-identical to the reference kernel
    np.testing.assert_array_equal(yd.cpu().numpy().view(np.uint16).reshape(-1), oracle.gemv_refmath(x, q, s, 8).reshape(-1))
    # a wrong dtype is rejected, recorded, and launches nothing
    vbad = make_view(qd.data_ptr(), DataType.FP16, [N, K])
    L.launch_w8a16_gemv(ctypes.byref(vx), ctypes.byref(vbad), ctypes.byref(vs), ctypes.byref(vy), 128, st)
    assert L.af_view_last_status() == 1


def test_launch_argmax_and_linear_gemm_view():
    from atomflow_b200._lib import DataType, lib, make_view
    L = lib()
    V = 128256
    v = normal_f32(1, V)
    v[99999] = 11.0
    vd = torch.from_numpy(v).cuda()
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    lv = make_view(vd.data_ptr(), DataType.FP32, [1, V])
    st = torch.cuda.current_stream().cuda_stream
    # default: the reference launcher's result, ids < 65536 only (argmax.cu:72-73, 115-117)
    want_ref = int(np.argmax(v.reshape(-1)[:65536]))
    L.launch_argmax(ctypes.byref(lv), ctypes.c_void_p(out.data_ptr()), st)
    torch.cuda.synchronize()
    assert L.af_view_last_status() == 0 and int(out.item()) == want_ref
    R = oracle.ref()
    if R is not None:   # the reference's own launch_argmax on the same logits
        ro = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert R.afref_argmax(vd.data_ptr(), V, ro.data_ptr(), st) == 0
        torch.cuda.synchronize()
        assert int(ro.item()) == want_ref
    assert L.af_view_set_argmax_mode(0) == 1
    try:
        L.launch_argmax(ctypes.byref(lv), ctypes.c_void_p(out.data_ptr()), st)
        torch.cuda.synchronize()
        assert L.af_view_last_status() == 0 and int(out.item()) == 99999
    finally:
        assert L.af_view_set_argmax_mode(1) == 0
    assert L.af_view_set_argmax_mode(7) == -1
    M, N, K = 4, 256, 512
    x, q, _ = make_gemv_case(5, M, N, K, kind="none")
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    qd = torch.from_numpy(q).cuda()
    yd = torch.zeros(M, N, dtype=torch.int16, device="cuda")
    vi = make_view(xd.data_ptr(), DataType.FP16, [M, K])
    vw = make_view(qd.data_ptr(), DataType.FP8_E4M3, [N, K])
    vo = make_view(yd.data_ptr(), DataType.FP16, [M, N])
    L.launch_linear_gemm(ctypes.byref(vi), ctypes.byref(vw), ctypes.byref(vo), None, st)
    torch.cuda.synchronize()
    assert L.af_view_last_status() == 0
    assert_fp16_parity(yd.cpu().numpy().view(np.uint16), oracle.gemv_f64(x, q, None, "none", with_l2=True), "linear")
